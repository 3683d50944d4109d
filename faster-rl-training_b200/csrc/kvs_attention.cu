// RoPE at explicit logical positions, and the exact-arithmetic (SIMT) attention
// kernels used for fp32 / fp64 models and for shapes the tensor-core kernels do
// not cover.
//
// Reference: kvstreams/rope.py:21-46 (RotaryEmbedding, apply_rope) and
// kvstreams/model.py:50-75 (Attention.forward): GQA by repeat_interleave
// (head h reads kv head h // (n_heads / n_kv_heads)), scores * head_dim**-0.5,
// masked softmax over keys, probabilities times values.
#include <initializer_list>

#include "kvs_common.cuh"
#include "kvs_rope.cuh"

#include <algorithm>
#include <mutex>
#include <vector>

using namespace kvs;

namespace {

// ------------------------------------------------------------------ RoPE
// in place (src == dst) or copying; one thread per rotated pair (i, i + D/2).  src rows
// (tokens) are src_stride elements apart, dst rows packed.
template <typename T, typename F>
__global__ void rope_kernel(const T* __restrict__ src, T* __restrict__ dst, const int64_t* __restrict__ pos,
                            int n_tokens, int n_heads, int D, const F* __restrict__ inv_freq, int64_t src_stride,
                            int64_t dst_stride) {
  const int half = D >> 1;
  const int64_t total = (int64_t)n_tokens * n_heads * half;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    const int64_t th = idx / half;
    const int t = (int)(th / n_heads);
    const int64_t base = (int64_t)t * dst_stride + (th - (int64_t)t * n_heads) * D;
    const int64_t sbase = (int64_t)t * src_stride + (th - (int64_t)t * n_heads) * D;
    using A = typename Acc<T>::type;
    A a = to_acc(src[sbase + i]), b = to_acc(src[sbase + i + half]);
    A r0, r1;
    rope_rotate<A, F>(a, b, pos[t], inv_freq[i], r0, r1);
    dst[base + i] = from_acc<T>(r0);
    dst[base + i + half] = from_acc<T>(r1);
  }
}

// RoPE of new keys written straight into the pool, values copied alongside
// (apply_rope on k, model.py:63, then PagedKVCache.write, paged_cache.py:167-171).
template <typename T, typename F>
__global__ void rope_write_kv_kernel(kvs_cache c, int layer, const int32_t* __restrict__ blocks,
                                     const int32_t* __restrict__ offsets, const T* __restrict__ k,
                                     const T* __restrict__ v, const int64_t* __restrict__ pos, int n_tokens,
                                     const F* __restrict__ inv_freq, int64_t kv_stride) {
  const int D = c.head_dim, half = D >> 1, H = c.n_kv_heads;
  const int64_t total = (int64_t)n_tokens * H * half;
  T* K = static_cast<T*>(c.k);
  T* V = static_cast<T*>(c.v);
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    const int64_t th = idx / half;
    const int h = (int)(th % H);
    const int t = (int)(th / H);
    const int64_t row = ((int64_t)layer * c.num_blocks + blocks[t]) * c.block_size + offsets[t];
    const int64_t dst = (row * H + h) * D;
    const int64_t src = (int64_t)t * kv_stride + (int64_t)h * D;
    using A = typename Acc<T>::type;
    A a = to_acc(k[src + i]), b = to_acc(k[src + i + half]);
    A r0, r1;
    rope_rotate<A, F>(a, b, pos[t], inv_freq[i], r0, r1);
    K[dst + i] = from_acc<T>(r0);
    K[dst + i + half] = from_acc<T>(r1);
    V[dst + i] = v[src + i];
    V[dst + i + half] = v[src + i + half];
  }
}

// 16 bytes of T as accumulator values (and back, rounded as from_acc rounds)
template <typename T> struct Pack16;
template <> struct Pack16<float> {
  static constexpr int n = 4;
  static __device__ void unpack(const uint4& u, float (&x)[4]) {
    x[0] = __uint_as_float(u.x), x[1] = __uint_as_float(u.y), x[2] = __uint_as_float(u.z), x[3] = __uint_as_float(u.w);
  }
  static __device__ uint4 pack(const float (&x)[4]) {
    return make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]), __float_as_uint(x[3]));
  }
};
template <> struct Pack16<double> {
  static constexpr int n = 2;
  static __device__ void unpack(const uint4& u, double (&x)[2]) {
    x[0] = __hiloint2double((int)u.y, (int)u.x), x[1] = __hiloint2double((int)u.w, (int)u.z);
  }
  static __device__ uint4 pack(const double (&x)[2]) {
    return make_uint4((unsigned)__double2loint(x[0]), (unsigned)__double2hiint(x[0]), (unsigned)__double2loint(x[1]),
                      (unsigned)__double2hiint(x[1]));
  }
};
template <typename H, typename H2>
struct PackHalf16 {
  static constexpr int n = 8;
  static __device__ float2 to2(uint32_t w) {
    H2 v;
    memcpy(&v, &w, 4);
    return make_float2(to_acc<H>(v.x), to_acc<H>(v.y));
  }
  static __device__ uint32_t from2(float a, float b) {
    H2 v;
    v.x = from_acc<H>(a);
    v.y = from_acc<H>(b);
    uint32_t w;
    memcpy(&w, &v, 4);
    return w;
  }
  static __device__ void unpack(const uint4& u, float (&x)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = to2(w[k]);
      x[2 * k] = f.x, x[2 * k + 1] = f.y;
    }
  }
  static __device__ uint4 pack(const float (&x)[8]) {
    return make_uint4(from2(x[0], x[1]), from2(x[2], x[3]), from2(x[4], x[5]), from2(x[6], x[7]));
  }
};
template <> struct Pack16<__nv_bfloat16> : PackHalf16<__nv_bfloat16, __nv_bfloat162> {};
template <> struct Pack16<__half> : PackHalf16<__half, __half2> {};

// The same rotations with one angle per (token, frequency) shared by every head: thread ->
// (token, chunk of V = 16 / sizeof(T) consecutive frequencies), sin / cos computed once, then
// 16-byte loads of the chunk from both halves of each head.  Rows and heads 16-byte aligned.
template <typename T, typename F>
__global__ void rope_heads_kernel(const T* __restrict__ src, T* __restrict__ dst, const int64_t* __restrict__ pos,
                                  int n_tokens, int n_heads, int D, const F* __restrict__ inv_freq,
                                  int64_t src_stride, int64_t dst_stride) {
  using A = typename Acc<T>::type;
  using P = Pack16<T>;
  constexpr int V = P::n;
  const int half = D >> 1, chunks = half / V;
  const int64_t total = (int64_t)n_tokens * chunks;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / chunks);
    const int i0 = (int)(idx - (int64_t)t * chunks) * V;
    const int64_t p = pos[t];
    A sn[V], cs[V];
#pragma unroll
    for (int k = 0; k < V; ++k) rope_sincos<A, F>(p, inv_freq[i0 + k], sn[k], cs[k]);
    const T* srow = src + (int64_t)t * src_stride + i0;
    T* drow = dst + (int64_t)t * dst_stride + i0;
#pragma unroll 4
    for (int h = 0; h < n_heads; ++h) {
      const uint4 ulo = *reinterpret_cast<const uint4*>(srow + (int64_t)h * D);
      const uint4 uhi = *reinterpret_cast<const uint4*>(srow + (int64_t)h * D + half);
      A a[V], b[V], r0[V], r1[V];
      P::unpack(ulo, a);
      P::unpack(uhi, b);
#pragma unroll
      for (int k = 0; k < V; ++k) rope_apply(a[k], b[k], sn[k], cs[k], r0[k], r1[k]);
      *reinterpret_cast<uint4*>(drow + (int64_t)h * D) = P::pack(r0);
      *reinterpret_cast<uint4*>(drow + (int64_t)h * D + half) = P::pack(r1);
    }
  }
}

// rope_write_kv_kernel with the same thread layout
template <typename T, typename F>
__global__ void rope_heads_write_kv_kernel(kvs_cache c, int layer, const int32_t* __restrict__ blocks,
                                           const int32_t* __restrict__ offsets, const T* __restrict__ k,
                                           const T* __restrict__ v, const int64_t* __restrict__ pos, int n_tokens,
                                           const F* __restrict__ inv_freq, int64_t kv_stride) {
  using A = typename Acc<T>::type;
  using P = Pack16<T>;
  constexpr int V = P::n;
  const int D = c.head_dim, half = D >> 1, H = c.n_kv_heads, chunks = half / V;
  T* K = static_cast<T*>(c.k);
  T* Vp = static_cast<T*>(c.v);
  const int64_t total = (int64_t)n_tokens * chunks;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(idx / chunks);
    const int i0 = (int)(idx - (int64_t)t * chunks) * V;
    const int64_t p = pos[t];
    A sn[V], cs[V];
#pragma unroll
    for (int q = 0; q < V; ++q) rope_sincos<A, F>(p, inv_freq[i0 + q], sn[q], cs[q]);
    const int64_t row = ((int64_t)layer * c.num_blocks + blocks[t]) * c.block_size + offsets[t];
    const T* krow = k + (int64_t)t * kv_stride + i0;
    const T* vrow = v + (int64_t)t * kv_stride + i0;
    T* kdst = K + row * H * D + i0;
    T* vdst = Vp + row * H * D + i0;
#pragma unroll 2
    for (int h = 0; h < H; ++h) {
      const int64_t o = (int64_t)h * D;
      const uint4 ulo = *reinterpret_cast<const uint4*>(krow + o);
      const uint4 uhi = *reinterpret_cast<const uint4*>(krow + o + half);
      const uint4 vlo = *reinterpret_cast<const uint4*>(vrow + o);
      const uint4 vhi = *reinterpret_cast<const uint4*>(vrow + o + half);
      A a[V], b[V], r0[V], r1[V];
      P::unpack(ulo, a);
      P::unpack(uhi, b);
#pragma unroll
      for (int q = 0; q < V; ++q) rope_apply(a[q], b[q], sn[q], cs[q], r0[q], r1[q]);
      *reinterpret_cast<uint4*>(kdst + o) = P::pack(r0);
      *reinterpret_cast<uint4*>(kdst + o + half) = P::pack(r1);
      *reinterpret_cast<uint4*>(vdst + o) = vlo;
      *reinterpret_cast<uint4*>(vdst + o + half) = vhi;
    }
  }
}

// whether the 16-byte-chunk kernels apply: every head row and half-row starts on 16 bytes
template <typename T>
bool rope_vec_ok(int D, std::initializer_list<int64_t> strides, std::initializer_list<const void*> ptrs) {
  constexpr int V = 16 / (int)sizeof(T);
  if ((D / 2) % V != 0) return false;
  for (int64_t stride : strides)
    if ((stride * (int64_t)sizeof(T)) % 16 != 0) return false;
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) % 16 != 0) return false;
  return true;
}

template <typename A>
__device__ __forceinline__ A warp_allreduce_sum(A x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename A> __device__ __forceinline__ A exp_acc(A x);
template <> __device__ __forceinline__ float exp_acc<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double exp_acc<double>(double x) { return exp(x); }

// Online softmax state of one (query, head) held by a warp; lanes own head dims
// lane, lane+32, ...  Keys are visited in increasing cache order.
template <typename T, int DPL>
struct OnlineRow {
  using A = typename Acc<T>::type;
  A q[DPL], acc[DPL];
  A m, l;
  __device__ __forceinline__ void init(const T* qrow, int D) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int d = lane + 32 * k;
      q[k] = d < D ? to_acc(qrow[d]) : A(0);
      acc[k] = A(0);
    }
    m = -INFINITY;
    l = A(0);
  }
  __device__ __forceinline__ void visit(const T* krow, const T* vrow, int D, A scale) {
    const int lane = threadIdx.x & 31;
    A part = A(0);
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) part += q[k] * to_acc(krow[d]);
    }
    const A s = warp_allreduce_sum(part) * scale;
    const A m_new = s > m ? s : m;
    const A alpha = exp_acc<A>(m - m_new);
    const A p = exp_acc<A>(s - m_new);
    l = l * alpha + p;
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) acc[k] = acc[k] * alpha + p * to_acc(vrow[d]);
    }
    m = m_new;
  }
  __device__ __forceinline__ void store(T* orow, int D) const {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < DPL; ++k) {
      const int d = lane + 32 * k;
      if (d < D) orow[d] = from_acc<T>(acc[k] / l);
    }
  }
};

// ------------------------------------------------------------------ paged (generic)
// One warp per (new token, query head).  Query i of a sequence with T new tokens
// and n live entries (new ones included) sees cache entries [0, n - T + i].
template <typename T, int DPL>
__global__ void __launch_bounds__(128)
paged_attn_generic_kernel(kvs_cache c, kvs_batch b, int layer, const T* __restrict__ q, T* __restrict__ out,
                          int n_heads, double scale) {
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= b.total_tokens * n_heads) return;
  const int j = gw / n_heads, h = gw % n_heads;
  int i = j;
  if (b.cu_tokens) {
    int lo = 0, hi = b.num_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (b.cu_tokens[mid] <= j) lo = mid; else hi = mid - 1;
    }
    i = lo;
  }
  const int slot = b.seq_slots[i];
  const int t0 = b.cu_tokens ? b.cu_tokens[i] : i;
  const int t1 = b.cu_tokens ? b.cu_tokens[i + 1] : i + 1;
  const int n = c.lengths[slot];
  const int visible = n - (t1 - t0) + (j - t0) + 1;
  const int D = c.head_dim, Hkv = c.n_kv_heads, bs = c.block_size;
  const int hk = h / (n_heads / Hkv);
  const T* K = static_cast<const T*>(c.k);
  const T* V = static_cast<const T*>(c.v);
  const int32_t* table = c.tables + (int64_t)slot * c.max_blocks;
  OnlineRow<T, DPL> row;
  row.init(q + ((int64_t)j * n_heads + h) * D, D);
  using A = typename Acc<T>::type;
  const A sc = (A)scale;
  for (int e = 0; e < visible; ++e) {
    const int64_t r = ((int64_t)layer * c.num_blocks + table[e / bs]) * bs + e % bs;
    const int64_t off = (r * Hkv + hk) * D;
    row.visit(K + off, V + off, D, sc);
  }
  row.store(out + ((int64_t)j * n_heads + h) * D, D);
}

// ------------------------------------------------------------------ replay (generic)
// One warp per (stream b, query t, head h); key s is visible iff s <= t and
// t < evicted_at[b][s] (replay.py:62), padded rows t >= len see only s == t
// (replay.py:221-222).
template <typename T, int DPL>
__global__ void __launch_bounds__(128)
replay_generic_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                      const int64_t* __restrict__ ev, const int32_t* __restrict__ lengths, T* __restrict__ out,
                      float* __restrict__ row_lse, int B, int Tn, int Hq, int Hkv, int D, double scale) {
  const int64_t gw = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= (int64_t)B * Tn * Hq) return;
  const int h = (int)(gw % Hq);
  const int t = (int)((gw / Hq) % Tn);
  const int b = (int)(gw / ((int64_t)Hq * Tn));
  const int hk = h / (Hq / Hkv);
  const int len = lengths[b];
  const int64_t qo = (((int64_t)b * Tn + t) * Hq + h) * D;
  OnlineRow<T, DPL> row;
  row.init(q + qo, D);
  using A = typename Acc<T>::type;
  const A sc = (A)scale;
  const int64_t* e = ev + (int64_t)b * Tn;
  if (t >= len) {
    const int64_t ko = (((int64_t)b * Tn + t) * Hkv + hk) * D;
    row.visit(k + ko, v + ko, D, sc);
  } else {
    for (int s = 0; s <= t; ++s) {
      if (!(t < e[s])) continue;
      const int64_t ko = (((int64_t)b * Tn + s) * Hkv + hk) * D;
      row.visit(k + ko, v + ko, D, sc);
    }
  }
  row.store(out + qo, D);
  if (row_lse != nullptr && (threadIdx.x & 31) == 0) {  // natural-log sum-exp in log2 units
    const int T_pad = (Tn + 127) / 128 * 128;
    row_lse[((int64_t)b * Hq + h) * T_pad + t] = (float)((row.m + log((double)row.l)) * 1.4426950408889634);
  }
}

template <typename T>
int launch_paged_generic(const kvs_cache& c, const kvs_batch& b, int layer, const void* q, void* out,
                         int n_heads, double scale, cudaStream_t st) {
  const int warps = b.total_tokens * n_heads;
  const int grid = (warps + 3) / 4;
  const T* qq = static_cast<const T*>(q);
  T* oo = static_cast<T*>(out);
  if (c.head_dim <= 32) paged_attn_generic_kernel<T, 1><<<grid, 128, 0, st>>>(c, b, layer, qq, oo, n_heads, scale);
  else if (c.head_dim <= 64) paged_attn_generic_kernel<T, 2><<<grid, 128, 0, st>>>(c, b, layer, qq, oo, n_heads, scale);
  else if (c.head_dim <= 128) paged_attn_generic_kernel<T, 4><<<grid, 128, 0, st>>>(c, b, layer, qq, oo, n_heads, scale);
  else if (c.head_dim <= 256) paged_attn_generic_kernel<T, 8><<<grid, 128, 0, st>>>(c, b, layer, qq, oo, n_heads, scale);
  else return KVS_E_UNSUPPORTED;
  return launch_rc();
}

template <typename T>
int launch_replay_generic(const kvs_replay_args& a, cudaStream_t st) {
  const int64_t warps = (int64_t)a.batch * a.seq_len * a.n_heads;
  const int64_t grid = (warps + 3) / 4;
  if (grid > INT32_MAX) return KVS_E_UNSUPPORTED;
  const T* q = static_cast<const T*>(a.q);
  const T* k = static_cast<const T*>(a.k);
  const T* v = static_cast<const T*>(a.v);
  T* o = static_cast<T*>(a.out);
#define KVS_REPLAY(DPL)                                                                             \
  replay_generic_kernel<T, DPL><<<(unsigned)grid, 128, 0, st>>>(q, k, v, a.evicted_at, a.lengths, o, a.row_lse, \
                                                                a.batch, \
                                                                a.seq_len, a.n_heads, a.n_kv_heads,    \
                                                                a.head_dim, a.scale)
  if (a.head_dim <= 32) KVS_REPLAY(1);
  else if (a.head_dim <= 64) KVS_REPLAY(2);
  else if (a.head_dim <= 128) KVS_REPLAY(4);
  else if (a.head_dim <= 256) KVS_REPLAY(8);
  else return KVS_E_UNSUPPORTED;
#undef KVS_REPLAY
  return launch_rc();
}

template <typename T, typename F>
int launch_rope(const void* src, void* dst, const int64_t* pos, int n_tokens, int n_heads, int D,
                const void* inv_freq, cudaStream_t st, int64_t src_stride, int64_t dst_stride) {
  const int64_t total = (int64_t)n_tokens * n_heads * (D / 2);
  if (total == 0) return KVS_OK;
  const int64_t sstride = src_stride ? src_stride : (int64_t)n_heads * D;
  const int64_t dstride = dst_stride ? dst_stride : (int64_t)n_heads * D;
  if (rope_vec_ok<T>(D, {sstride, dstride}, {src, dst})) {
    const int64_t units = (int64_t)n_tokens * (D / 2 / Pack16<T>::n);
    const int grid = (int)std::min<int64_t>((units + 255) / 256, 148 * 64);
    rope_heads_kernel<T, F><<<grid, 256, 0, st>>>(static_cast<const T*>(src), static_cast<T*>(dst), pos, n_tokens,
                                                  n_heads, D, static_cast<const F*>(inv_freq), sstride, dstride);
    return launch_rc();
  }
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
  rope_kernel<T, F><<<grid, 256, 0, st>>>(static_cast<const T*>(src), static_cast<T*>(dst), pos, n_tokens,
                                          n_heads, D, static_cast<const F*>(inv_freq), sstride, dstride);
  return launch_rc();
}

template <typename T, typename F>
int launch_rope_write(const kvs_cache& c, int layer, const int32_t* blocks, const int32_t* offsets,
                      const void* k, const void* v, const int64_t* pos, int n_tokens, const void* inv_freq,
                      cudaStream_t st, int64_t kv_stride) {
  const int64_t total = (int64_t)n_tokens * c.n_kv_heads * (c.head_dim / 2);
  if (total == 0) return KVS_OK;
  const int64_t kstride = kv_stride ? kv_stride : (int64_t)c.n_kv_heads * c.head_dim;
  if (rope_vec_ok<T>(c.head_dim, {kstride}, {k, v, c.k, c.v})) {
    const int64_t units = (int64_t)n_tokens * (c.head_dim / 2 / Pack16<T>::n);
    const int grid = (int)std::min<int64_t>((units + 255) / 256, 148 * 64);
    rope_heads_write_kv_kernel<T, F><<<grid, 256, 0, st>>>(c, layer, blocks, offsets, static_cast<const T*>(k),
                                                           static_cast<const T*>(v), pos, n_tokens,
                                                           static_cast<const F*>(inv_freq), kstride);
    return launch_rc();
  }
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
  rope_write_kv_kernel<T, F><<<grid, 256, 0, st>>>(c, layer, blocks, offsets, static_cast<const T*>(k),
                                                   static_cast<const T*>(v), pos, n_tokens,
                                                   static_cast<const F*>(inv_freq),
                                                   kv_stride ? kv_stride : (int64_t)c.n_kv_heads * c.head_dim);
  return launch_rc();
}

int rope_dispatch(const void* src, void* dst, int dtype, const int64_t* pos, int n_tokens, int n_heads, int D,
                  const void* inv_freq, cudaStream_t st, int64_t src_stride = 0, int64_t dst_stride = 0) {
  switch (dtype) {
    case KVS_F32:
      return launch_rope<float, float>(src, dst, pos, n_tokens, n_heads, D, inv_freq, st, src_stride, dst_stride);
    case KVS_F64:
      return launch_rope<double, double>(src, dst, pos, n_tokens, n_heads, D, inv_freq, st, src_stride, dst_stride);
    case KVS_BF16:
      return launch_rope<__nv_bfloat16, float>(src, dst, pos, n_tokens, n_heads, D, inv_freq, st, src_stride,
                                               dst_stride);
    case KVS_F16:
      return launch_rope<__half, float>(src, dst, pos, n_tokens, n_heads, D, inv_freq, st, src_stride, dst_stride);
  }
  return KVS_E_UNSUPPORTED;
}

}  // namespace

// Exact generic decode: rope(q) into out, rope(k)+v into the pool, then attention
// reading q from out (each warp reads its own row before overwriting it).
// RoPE of q (into a->out) and of the new k, and the append of k/v to their slots
int kvs_rope_append(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a, cudaStream_t st) {
  const int n = b->total_tokens;
  int rc = rope_dispatch(a->q, a->out, c->dtype, a->positions, n, a->n_heads, c->head_dim, a->inv_freq, st,
                         a->q_stride);
  if (rc) return rc;
  const int64_t ks = a->kv_stride;
  switch (c->dtype) {
    case KVS_F32: return launch_rope_write<float, float>(*c, a->layer, a->slot_blocks, a->slot_offsets, a->k_new, a->v_new, a->positions, n, a->inv_freq, st, ks);
    case KVS_F64: return launch_rope_write<double, double>(*c, a->layer, a->slot_blocks, a->slot_offsets, a->k_new, a->v_new, a->positions, n, a->inv_freq, st, ks);
    case KVS_BF16: return launch_rope_write<__nv_bfloat16, float>(*c, a->layer, a->slot_blocks, a->slot_offsets, a->k_new, a->v_new, a->positions, n, a->inv_freq, st, ks);
    case KVS_F16: return launch_rope_write<__half, float>(*c, a->layer, a->slot_blocks, a->slot_offsets, a->k_new, a->v_new, a->positions, n, a->inv_freq, st, ks);
  }
  return KVS_E_UNSUPPORTED;
}

int kvs_decode_generic(const kvs_cache* c, const kvs_batch* b, const kvs_decode_args* a, cudaStream_t st) {
  const int rc = kvs_rope_append(c, b, a, st);
  if (rc) return rc;
  return kvs_paged_attention(c, b, a->layer, a->out, a->out, a->n_heads, a->scale, reinterpret_cast<kvs_stream_t>(st));
}

int kvs_replay_generic(const kvs_replay_args* a, cudaStream_t st) {
  switch (a->dtype) {
    case KVS_F32: return launch_replay_generic<float>(*a, st);
    case KVS_F64: return launch_replay_generic<double>(*a, st);
    case KVS_BF16: return launch_replay_generic<__nv_bfloat16>(*a, st);
    case KVS_F16: return launch_replay_generic<__half>(*a, st);
  }
  return KVS_E_UNSUPPORTED;
}

// ====================================================================== C ABI

KVS_API size_t kvs_abi_struct_size(int which) {
  switch (which) {
    case 0: return sizeof(kvs_cache);
    case 1: return sizeof(kvs_batch);
    case 2: return sizeof(kvs_decode_args);
    case 3: return sizeof(kvs_replay_args);
    case 4: return sizeof(kvs_segments);
  }
  return 0;
}

KVS_API int kvs_abi_version(void) { return KVS_ABI_VERSION; }

KVS_API int kvs_device_sm_count(void) {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev];
}

KVS_API int kvs_rope(void* x, int32_t dtype, const int64_t* positions, int32_t n_tokens, int32_t n_heads,
                     int32_t head_dim, const void* inv_freq, kvs_stream_t stream) {
  if (!x || !positions || !inv_freq || n_tokens < 0 || n_heads <= 0 || head_dim <= 0 || head_dim % 2)
    return KVS_E_ARG;
  return rope_dispatch(x, x, dtype, positions, n_tokens, n_heads, head_dim, inv_freq, to_cuda(stream));
}

KVS_API int kvs_rope_copy(const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int32_t dtype,
                          const int64_t* positions, int32_t n_tokens, int32_t n_heads, int32_t head_dim,
                          const void* inv_freq, kvs_stream_t stream) {
  const int64_t row = (int64_t)n_heads * head_dim;
  if (!src || !dst || !positions || !inv_freq || n_tokens < 0 || n_heads <= 0 || head_dim <= 0 || head_dim % 2 ||
      src_stride < 0 || (src_stride != 0 && src_stride < row) || dst_stride < 0 || (dst_stride != 0 && dst_stride < row))
    return KVS_E_ARG;
  return rope_dispatch(src, dst, dtype, positions, n_tokens, n_heads, head_dim, inv_freq, to_cuda(stream),
                       src_stride, dst_stride);
}

KVS_API int kvs_paged_attention(const kvs_cache* c, const kvs_batch* b, int32_t layer, const void* q, void* out,
                                int32_t n_heads, double scale, kvs_stream_t stream) {
  if (!c || !b || !q || !out || layer < 0 || layer >= c->n_layers || n_heads <= 0 ||
      n_heads % c->n_kv_heads)
    return KVS_E_ARG;
  if (b->total_tokens == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  switch (c->dtype) {
    case KVS_F32: return launch_paged_generic<float>(*c, *b, layer, q, out, n_heads, scale, st);
    case KVS_F64: return launch_paged_generic<double>(*c, *b, layer, q, out, n_heads, scale, st);
    case KVS_BF16: return launch_paged_generic<__nv_bfloat16>(*c, *b, layer, q, out, n_heads, scale, st);
    case KVS_F16: return launch_paged_generic<__half>(*c, *b, layer, q, out, n_heads, scale, st);
  }
  return KVS_E_UNSUPPORTED;
}
