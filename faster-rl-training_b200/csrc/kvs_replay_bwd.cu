// Backward of the masked replay attention (the gradient the trainer needs through
// token_logprobs, training/logprobs.py:10-25 -> model.py:71-74 under the replay.py:62 mask).
// Exact SIMT kernels for every dtype (float accumulation for half types, double for f64):
//
//   P = softmax(scale * Q K^T) over the visible keys of each row, O = P V (the forward)
//   D_t = sum_d dO_t O_t,   dS = P o (dO V^T - D),   dQ = scale dS K,
//   dK = scale dS^T Q  (summed over the query heads of each KV head),   dV = P^T dO
//
// visible(t, s) = s <= t && t < evicted_at[b][s] for t < lengths[b]; a padded row t >= len
// sees s == t only (collate, replay.py:221-222).  Three launches: row statistics (log-sum-exp
// of the scores, D), dQ (one warp per query row and head), dK/dV (one warp per key and KV
// head, over the rows that see the key and the heads of its group).
#include "kvs_common.cuh"

#include <cmath>

using namespace kvs;

namespace {

template <typename A> __device__ __forceinline__ A warp_sum(A x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
template <typename A> __device__ __forceinline__ A exp_a(A x);
template <> __device__ __forceinline__ float exp_a<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double exp_a<double>(double x) { return exp(x); }
template <typename A> __device__ __forceinline__ A log_a(A x);
template <> __device__ __forceinline__ float log_a<float>(float x) { return logf(x); }
template <> __device__ __forceinline__ double log_a<double>(double x) { return log(x); }

// the lane's DPL elements of a head vector (element lane + 32 k)
template <typename T, int DPL>
__device__ __forceinline__ void load_row(const T* p, int D, typename Acc<T>::type (&r)[DPL]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < DPL; ++k) {
    const int d = lane + 32 * k;
    r[k] = d < D ? to_acc(p[d]) : typename Acc<T>::type(0);
  }
}
template <typename T, int DPL>
__device__ __forceinline__ typename Acc<T>::type dot_row(const typename Acc<T>::type (&a)[DPL], const T* p, int D) {
  using A = typename Acc<T>::type;
  const int lane = threadIdx.x & 31;
  A s = A(0);
#pragma unroll
  for (int k = 0; k < DPL; ++k) {
    const int d = lane + 32 * k;
    if (d < D) s += a[k] * to_acc(p[d]);
  }
  return warp_sum(s);
}

// row statistics: lse[b][t][h] = log sum_s exp(scale q.k_s) over the visible keys,
// dd[b][t][h] = sum_d dO O
template <typename T, int DPL>
__global__ void __launch_bounds__(128)
replay_bwd_stats_kernel(const T* __restrict__ q, const T* __restrict__ k, const int64_t* __restrict__ ev,
                        const int32_t* __restrict__ lengths, const T* __restrict__ o, const T* __restrict__ dout,
                        typename Acc<T>::type* __restrict__ lse, typename Acc<T>::type* __restrict__ dd, int B,
                        int Tn, int Hq, int Hkv, int D, double scale) {
  using A = typename Acc<T>::type;
  const int64_t gw = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= (int64_t)B * Tn * Hq) return;
  const int h = (int)(gw % Hq), t = (int)((gw / Hq) % Tn), b = (int)(gw / ((int64_t)Hq * Tn));
  const int hk = h / (Hq / Hkv), len = lengths[b];
  const int64_t qo = (((int64_t)b * Tn + t) * Hq + h) * D;
  A qr[DPL];
  load_row<T, DPL>(q + qo, D, qr);
  const A sc = (A)scale;
  const int64_t* e = ev + (int64_t)b * Tn;
  A m = -INFINITY, l = A(0);
  auto visit = [&](int s) {
    const A x = dot_row<T, DPL>(qr, k + (((int64_t)b * Tn + s) * Hkv + hk) * D, D) * sc;
    const A mn = x > m ? x : m;
    l = l * exp_a<A>(m - mn) + exp_a<A>(x - mn);
    m = mn;
  };
  if (t >= len) {
    visit(t);
  } else {
    for (int s = 0; s <= t; ++s)
      if (t < e[s]) visit(s);
  }
  A orow[DPL];
  load_row<T, DPL>(o + qo, D, orow);
  const A dsum = dot_row<T, DPL>(orow, dout + qo, D);
  if ((threadIdx.x & 31) == 0) {
    lse[gw] = m + log_a<A>(l);
    dd[gw] = dsum;
  }
}

// dQ: one warp per (b, t, h)
template <typename T, int DPL>
__global__ void __launch_bounds__(128)
replay_bwd_dq_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                     const int64_t* __restrict__ ev, const int32_t* __restrict__ lengths, const T* __restrict__ dout,
                     const typename Acc<T>::type* __restrict__ lse, const typename Acc<T>::type* __restrict__ dd,
                     T* __restrict__ dq, int B, int Tn, int Hq, int Hkv, int D, double scale) {
  using A = typename Acc<T>::type;
  const int64_t gw = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= (int64_t)B * Tn * Hq) return;
  const int h = (int)(gw % Hq), t = (int)((gw / Hq) % Tn), b = (int)(gw / ((int64_t)Hq * Tn));
  const int hk = h / (Hq / Hkv), len = lengths[b];
  const int64_t qo = (((int64_t)b * Tn + t) * Hq + h) * D;
  A qr[DPL], dor[DPL], acc[DPL];
  load_row<T, DPL>(q + qo, D, qr);
  load_row<T, DPL>(dout + qo, D, dor);
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = A(0);
  const A sc = (A)scale, L = lse[gw], Dt = dd[gw];
  const int64_t* e = ev + (int64_t)b * Tn;
  const int lane = threadIdx.x & 31;
  auto visit = [&](int s) {
    const int64_t ko = (((int64_t)b * Tn + s) * Hkv + hk) * D;
    const A p = exp_a<A>(dot_row<T, DPL>(qr, k + ko, D) * sc - L);
    const A ds = p * (dot_row<T, DPL>(dor, v + ko, D) - Dt);
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) acc[i] += ds * to_acc(k[ko + d]);
    }
  };
  if (t >= len) {
    visit(t);
  } else {
    for (int s = 0; s <= t; ++s)
      if (t < e[s]) visit(s);
  }
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int d = lane + 32 * i;
    if (d < D) dq[qo + d] = from_acc<T>(acc[i] * sc);
  }
}

// dK, dV: one warp per (b, s, hk); rows t that see key s: s <= t < min(len, evicted_at[s])
// (real rows), or t == s when s is itself a padded row
template <typename T, int DPL>
__global__ void __launch_bounds__(128)
replay_bwd_dkdv_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                       const int64_t* __restrict__ ev, const int32_t* __restrict__ lengths,
                       const T* __restrict__ dout, const typename Acc<T>::type* __restrict__ lse,
                       const typename Acc<T>::type* __restrict__ dd, T* __restrict__ dk, T* __restrict__ dv, int B,
                       int Tn, int Hq, int Hkv, int D, double scale) {
  using A = typename Acc<T>::type;
  const int64_t gw = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= (int64_t)B * Tn * Hkv) return;
  const int hk = (int)(gw % Hkv), s = (int)((gw / Hkv) % Tn), b = (int)(gw / ((int64_t)Hkv * Tn));
  const int G = Hq / Hkv, len = lengths[b];
  const int64_t ko = (((int64_t)b * Tn + s) * Hkv + hk) * D;
  A kr[DPL], vr[DPL], ak[DPL], av[DPL];
  load_row<T, DPL>(k + ko, D, kr);
  load_row<T, DPL>(v + ko, D, vr);
#pragma unroll
  for (int i = 0; i < DPL; ++i) ak[i] = av[i] = A(0);
  const A sc = (A)scale;
  const int lane = threadIdx.x & 31;
  int t0 = s, t1;  // rows [t0, t1)
  if (s >= len) {
    t1 = s + 1;
  } else {
    const int64_t e = ev[(int64_t)b * Tn + s];
    t1 = (int)(e < (int64_t)len ? e : (int64_t)len);
  }
  for (int t = t0; t < t1; ++t) {
    for (int g = 0; g < G; ++g) {
      const int h = hk * G + g;
      const int64_t row = ((int64_t)b * Tn + t) * Hq + h;
      const T* qt = q + row * D;
      const T* dot = dout + row * D;
      const A p = exp_a<A>(dot_row<T, DPL>(kr, qt, D) * sc - lse[row]);
      const A ds = p * (dot_row<T, DPL>(vr, dot, D) - dd[row]);
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        if (d < D) {
          av[i] += p * to_acc(dot[d]);
          ak[i] += ds * to_acc(qt[d]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < DPL; ++i) {
    const int d = lane + 32 * i;
    if (d < D) {
      dk[ko + d] = from_acc<T>(ak[i] * sc);
      dv[ko + d] = from_acc<T>(av[i]);
    }
  }
}

template <typename T>
int launch_backward(const kvs_replay_args& a, const void* dout, void* dq, void* dk, void* dv, cudaStream_t st) {
  using A = typename Acc<T>::type;
  const int64_t rows = (int64_t)a.batch * a.seq_len * a.n_heads;
  const int64_t keys = (int64_t)a.batch * a.seq_len * a.n_kv_heads;
  if ((rows + 3) / 4 > INT32_MAX || (keys + 3) / 4 > INT32_MAX) return KVS_E_UNSUPPORTED;
  A* lse = static_cast<A*>(a.scratch);
  A* ddv = lse + rows;
  const T* q = static_cast<const T*>(a.q);
  const T* k = static_cast<const T*>(a.k);
  const T* v = static_cast<const T*>(a.v);
  const T* o = static_cast<const T*>(a.out);
  const T* g = static_cast<const T*>(dout);
  const unsigned gr = (unsigned)((rows + 3) / 4), gk = (unsigned)((keys + 3) / 4);
  int rc = KVS_OK;
#define KVS_BWD(DPL)                                                                                             \
  do {                                                                                                           \
    replay_bwd_stats_kernel<T, DPL><<<gr, 128, 0, st>>>(q, k, a.evicted_at, a.lengths, o, g, lse, ddv, a.batch,  \
                                                        a.seq_len, a.n_heads, a.n_kv_heads, a.head_dim, a.scale); \
    if ((rc = launch_rc())) return rc;                                                                           \
    replay_bwd_dq_kernel<T, DPL><<<gr, 128, 0, st>>>(q, k, v, a.evicted_at, a.lengths, g, lse, ddv,              \
                                                     static_cast<T*>(dq), a.batch, a.seq_len, a.n_heads,         \
                                                     a.n_kv_heads, a.head_dim, a.scale);                         \
    if ((rc = launch_rc())) return rc;                                                                           \
    replay_bwd_dkdv_kernel<T, DPL><<<gk, 128, 0, st>>>(q, k, v, a.evicted_at, a.lengths, g, lse, ddv,            \
                                                       static_cast<T*>(dk), static_cast<T*>(dv), a.batch,        \
                                                       a.seq_len, a.n_heads, a.n_kv_heads, a.head_dim, a.scale); \
    return launch_rc();                                                                                          \
  } while (0)
  if (a.head_dim <= 32) KVS_BWD(1);
  if (a.head_dim <= 64) KVS_BWD(2);
  if (a.head_dim <= 128) KVS_BWD(4);
  if (a.head_dim <= 256) KVS_BWD(8);
#undef KVS_BWD
  return KVS_E_UNSUPPORTED;
}

size_t acc_bytes(int dtype) { return dtype == KVS_F64 ? 8 : 4; }

}  // namespace

size_t kvs_replay_tc_backward_scratch(int B, int T, int Hq);
int kvs_replay_tc_backward(const kvs_replay_args* a, const void* dout, void* dq, void* dk, void* dv, cudaStream_t st);
int kvs_replay_tc_backward_path(const kvs_replay_args* a, cudaStream_t st);

KVS_API int kvs_replay_backward_path(const kvs_replay_args* a, kvs_stream_t stream) {
  if (!a || a->batch <= 0 || a->seq_len <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 ||
      a->n_heads % a->n_kv_heads)
    return KVS_E_ARG;
  if (a->dtype != KVS_BF16 || (a->flags & 1)) return 0;
  return kvs_replay_tc_backward_path(a, to_cuda(stream));
}

KVS_API size_t kvs_replay_backward_scratch_bytes(int32_t batch, int32_t seq_len, int32_t n_heads, int32_t dtype) {
  if (batch <= 0 || seq_len <= 0 || n_heads <= 0) return 0;
  const size_t exact = align_up((size_t)2 * batch * seq_len * n_heads * acc_bytes(dtype), 256);
  if (dtype != KVS_BF16) return exact;
  const size_t tc = kvs_replay_tc_backward_scratch(batch, seq_len, n_heads);
  return tc > exact ? tc : exact;
}

KVS_API int kvs_replay_attention_backward(const kvs_replay_args* a, const void* dout, void* dq, void* dk, void* dv,
                                          kvs_stream_t stream) {
  if (!a || !dout || !dq || !dk || !dv || !a->q || !a->k || !a->v || !a->out || !a->evicted_at || !a->lengths ||
      a->batch < 0 || a->seq_len < 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->n_heads % a->n_kv_heads ||
      a->head_dim <= 0)
    return KVS_E_ARG;
  if (a->batch == 0 || a->seq_len == 0) return KVS_OK;
  if (!a->scratch ||
      a->scratch_bytes < kvs_replay_backward_scratch_bytes(a->batch, a->seq_len, a->n_heads, a->dtype))
    return KVS_E_SCRATCH;
  const cudaStream_t st = to_cuda(stream);
  if (a->dtype == KVS_BF16 && a->row_lse != nullptr && !(a->flags & 1)) {
    const int rc = kvs_replay_tc_backward(a, dout, dq, dk, dv, st);
    if (rc != KVS_E_UNSUPPORTED) return rc;
  }
  switch (a->dtype) {
    case KVS_F32: return launch_backward<float>(*a, dout, dq, dk, dv, st);
    case KVS_F64: return launch_backward<double>(*a, dout, dq, dk, dv, st);
    case KVS_BF16: return launch_backward<__nv_bfloat16>(*a, dout, dq, dk, dv, st);
    case KVS_F16: return launch_backward<__half>(*a, dout, dq, dk, dv, st);
  }
  return KVS_E_UNSUPPORTED;
}
