// Log-probabilities of target tokens from lm_head logits (training/logprobs.py:17-20):
// logp = x_t / T - log sum_v exp(x_v / T), in one pass over each logits row, and its
// gradient dlogits = g (onehot(t) - softmax(x / T)) / T.  The reference materialises
// log_softmax(logits / T) for every row and gathers from it; here the row is read once.

#include <algorithm>
#include <climits>
#include <cmath>
#include <cooperative_groups.h>

#include "kvs_common.cuh"

using namespace kvs;

namespace {

constexpr int kRowThreads = 256;

template <typename T> struct Vec;
template <> struct Vec<float> { using type = float4; static constexpr int n = 4; };
template <> struct Vec<double> { using type = double2; static constexpr int n = 2; };

__device__ __forceinline__ float exp_of(float x) { return __expf(x); }
__device__ __forceinline__ double exp_of(double x) { return exp(x); }
__device__ __forceinline__ float log_of(float x) { return logf(x); }
__device__ __forceinline__ double log_of(double x) { return log(x); }

// running (max, sum of exp(x - max)) of a set of values
template <typename A>
struct Lse {
  A m, s;
  __device__ void add(A x) {
    if (x > m) {
      s = s * exp_of(m - x) + A(1);
      m = x;
    } else {
      s += exp_of(x - m);
    }
  }
  __device__ void merge(A m2, A s2) {
    if (m2 > m) {
      s = s * exp_of(m - m2) + s2;
      m = m2;
    } else if (s2 > A(0)) {
      s += s2 * exp_of(m2 - m);
    }
  }
};

template <typename A>
__device__ Lse<A> block_lse(Lse<A> v) {
  __shared__ A sm[kRowThreads / 32], ss[kRowThreads / 32];
  for (int o = 16; o > 0; o >>= 1) {
    const A m2 = __shfl_xor_sync(0xffffffffu, v.m, o), s2 = __shfl_xor_sync(0xffffffffu, v.s, o);
    v.merge(m2, s2);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[w] = v.m;
    ss[w] = v.s;
  }
  __syncthreads();
  Lse<A> r{-INFINITY, A(0)};
  for (int i = 0; i < kRowThreads / 32; ++i) r.merge(sm[i], ss[i]);
  __syncthreads();
  return r;
}

// one CTA per row: lse of x / T over the row, logp of the target.  x / T is x * (1 / T)
// (within one ulp of the reference's division; exact for the usual T = 1, where it is x).
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
lse_gather_kernel(const T* __restrict__ logits, int64_t ld, int vocab, const int64_t* __restrict__ targets,
                  T inv_temp, T* __restrict__ logp, T* __restrict__ lse_out) {
  using V = typename Vec<T>::type;
  constexpr int NV = Vec<T>::n;
  const int64_t row = blockIdx.x;
  const T* x = logits + row * ld;
  Lse<T> acc{-INFINITY, T(0)};
  // aligned vector loads when the row allows them
  const bool vec = (reinterpret_cast<uintptr_t>(x) % sizeof(V)) == 0;
  const int nvec = vec ? vocab / NV : 0;
  const V* xv = reinterpret_cast<const V*>(x);
  // four vector loads in flight per thread; one max / rescale per vector, its exps independent
  constexpr int U = 4;
  for (int i0 = threadIdx.x; i0 < nvec; i0 += U * kRowThreads) {
    V q[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * kRowThreads;
      if (i < nvec) q[u] = __ldcs(xv + i);  // streamed once
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (i0 + u * kRowThreads >= nvec) break;
      T e[NV];
      const T* qe = reinterpret_cast<const T*>(&q[u]);
      T vm = -INFINITY;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        e[k] = qe[k] * inv_temp;
        vm = vm > e[k] ? vm : e[k];
      }
      if (vm > acc.m) {
        acc.s = acc.s * exp_of(acc.m - vm);
        acc.m = vm;
      }
      T part = T(0);
#pragma unroll
      for (int k = 0; k < NV; ++k) part += exp_of(e[k] - acc.m);
      acc.s += part;
    }
  }
  for (int i = nvec * NV + threadIdx.x; i < vocab; i += kRowThreads) acc.add(x[i] * inv_temp);
  const Lse<T> r = block_lse(acc);
  if (threadIdx.x == 0) {
    const T lse = r.m + log_of(r.s);
    const int64_t t = targets[row];
    logp[row] = (t >= 0 && t < vocab) ? x[t] * inv_temp - lse : T(NAN);
    if (lse_out) lse_out[row] = lse;
  }
}

// dlogits[r][v] = g[r] * (onehot(t_r)[v] - exp(x[r][v] / T - lse[r])) / T, written in OutT
template <typename T, typename OutT>
__global__ void __launch_bounds__(kRowThreads)
lse_gather_bwd_kernel(const T* __restrict__ logits, int64_t ld, int vocab, const int64_t* __restrict__ targets,
                      const T* __restrict__ lse, const T* __restrict__ grad, T inv_temp, OutT* __restrict__ dlogits,
                      int64_t ld_out) {
  const int64_t row = blockIdx.x;
  const T* x = logits + row * ld;
  OutT* d = dlogits + row * ld_out;
  const T l = lse[row], g = grad[row] * inv_temp;
  const int64_t t = targets[row];
  for (int i = threadIdx.x; i < vocab; i += kRowThreads) {
    const T p = exp_of(x[i] * inv_temp - l);
    const T v = g * ((i == t ? T(1) : T(0)) - p);
    if constexpr (sizeof(OutT) == 2) {
      if constexpr (std::is_same<OutT, __nv_bfloat16>::value) d[i] = __float2bfloat16_rn((float)v);
      else d[i] = __float2half_rn((float)v);
    } else {
      d[i] = (OutT)v;
    }
  }
}

// ---------------------------------------------------------------------------- sampling
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011): ten rounds of two 32x32->64-bit products mixed into the 4-word counter, the
// 2-word key advanced by a Weyl sequence between rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
  }
  return c;
}

// Gumbel noise -log(-log U) of one Philox word, U = ((bits >> 9) + 0.5) * 2^-23 in
// [2^-24, 1 - 2^-24] (exact in float).  The inner log needs full accuracy near U = 1 (logf);
// the outer one sees -log U in [6e-8, 16.7] and its result is added to x / T, where the
// intrinsic's few-ulp error is immaterial.
__device__ __forceinline__ float gumbel(uint32_t bits) {
  const float u = __uint2float_rn(bits >> 9) * 0x1p-23f + 0x1p-24f;
  return -__logf(-logf(u));
}

constexpr int kSampleCTAs = 4;  // CTAs per logits row: one thread-block cluster

template <typename A>
struct SamplePart {
  A m, s, key;
  int idx;
};

// the larger key; among equal keys the lower vocabulary index (torch.argmax's first maximum)
template <typename A>
__device__ __forceinline__ void take_best(A& key, int& idx, A k2, int i2) {
  if (k2 > key || (k2 == key && i2 < idx)) {
    key = k2;
    idx = i2;
  }
}

// entries 4g .. 4g+3 of a row (-inf beyond the vocabulary)
template <typename T>
__device__ __forceinline__ void load_group(const T* x, int g, int vocab, bool vec, T (&e)[4]) {
  const int i = 4 * g;
  if (vec && i + 3 < vocab) {
    if constexpr (sizeof(T) == 4) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(x) + g);
      e[0] = v.x, e[1] = v.y, e[2] = v.z, e[3] = v.w;
    } else {
      const double2* p = reinterpret_cast<const double2*>(x + i);
      const double2 a = __ldcs(p), b = __ldcs(p + 1);
      e[0] = a.x, e[1] = a.y, e[2] = b.x, e[3] = b.y;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) e[k] = i + k < vocab ? x[i + k] : T(-INFINITY);
  }
}

// One cluster of kSampleCTAs CTAs per row; CTA rank r takes a contiguous quarter of the
// row's 4-entry groups (one Philox block each).  Per thread: the running log-sum-exp of
// x / T and the best key (x when greedy, x / T + Gumbel noise otherwise); reduced over the
// CTA, then over the cluster by rank 0 reading the other CTAs' partials from their shared
// memory (distributed shared memory), which writes the token and its log-prob.
template <typename T>
__global__ void __cluster_dims__(kSampleCTAs, 1, 1) __launch_bounds__(kRowThreads)
sample_kernel(const T* __restrict__ logits, int64_t ld, int vocab, T inv_temp, int greedy, uint32_t k0, uint32_t k1,
              uint32_t off_lo, uint32_t off_hi, int64_t* __restrict__ tokens, T* __restrict__ logp) {
  namespace cg = cooperative_groups;
  __shared__ SamplePart<T> part;
  __shared__ T s_key[kRowThreads / 32];
  __shared__ int s_idx[kRowThreads / 32];
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const int64_t row = blockIdx.x / kSampleCTAs;
  const T* x = logits + row * ld;
  const int groups = (vocab + 3) >> 2;
  const int per = (groups + kSampleCTAs - 1) / kSampleCTAs;
  const int gbeg = (int)rank * per, gend = min(groups, gbeg + per);
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16) == 0;
  Lse<T> acc{-INFINITY, T(0)};
  T best = -INFINITY;
  int bidx = INT_MAX;
  constexpr int U = 4;  // groups in flight per thread
  for (int g0 = gbeg + threadIdx.x; g0 < gend; g0 += U * kRowThreads) {
    T e[U][4];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (g0 + u * kRowThreads < gend) load_group(x, g0 + u * kRowThreads, vocab, vec, e[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = g0 + u * kRowThreads;
      if (g >= gend) break;
      T z[4], vm = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        z[k] = e[u][k] * inv_temp;
        vm = vm > z[k] ? vm : z[k];
      }
      if (vm != T(-INFINITY)) {  // a group of -inf adds nothing (and would give inf - inf)
        if (vm > acc.m) {
          acc.s = acc.s * exp_of(acc.m - vm);
          acc.m = vm;
        }
        T ps = T(0);
#pragma unroll
        for (int k = 0; k < 4; ++k) ps += exp_of(z[k] - acc.m);
        acc.s += ps;
      }
      if (greedy) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (4 * g + k < vocab && e[u][k] > best) best = e[u][k], bidx = 4 * g + k;
      } else {
        const uint4 r = philox4x32_10(make_uint4((uint32_t)g, (uint32_t)row, off_lo, off_hi), k0, k1);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const T key = z[k] + T(gumbel(w[k]));
          if (4 * g + k < vocab && key > best) best = key, bidx = 4 * g + k;
        }
      }
    }
  }
  // a thread's entries come in increasing index order, so its strict '>' kept the first maximum
  const Lse<T> tot = block_lse(acc);
  for (int o = 16; o > 0; o >>= 1) {
    const T k2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bidx, o);
    take_best(best, bidx, k2, i2);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_key[w] = best;
    s_idx[w] = bidx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRowThreads / 32; ++i) take_best(best, bidx, s_key[i], s_idx[i]);
    part = SamplePart<T>{tot.m, tot.s, best, bidx};
  }
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    Lse<T> l{part.m, part.s};
    T key = part.key;
    int idx = part.idx;
    for (int r = 1; r < kSampleCTAs; ++r) {
      const SamplePart<T>* q = cluster.map_shared_rank(&part, r);
      l.merge(q->m, q->s);
      take_best(key, idx, q->key, q->idx);
    }
    if (idx < vocab) {
      tokens[row] = idx;
      logp[row] = x[idx] * inv_temp - (l.m + log_of(l.s));
    } else {
      tokens[row] = -1;
      logp[row] = T(NAN);
    }
  }
  cluster.sync();  // the other CTAs' shared memory stays alive until rank 0 has read it
}

}  // namespace

KVS_API int kvs_lse_gather(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab, const int64_t* targets,
                           double temperature, int32_t dtype, void* logp, void* lse, kvs_stream_t stream) {
  if (!logits || !targets || !logp || n_rows < 0 || vocab <= 0 || ld < vocab || !(temperature > 0)) return KVS_E_ARG;
  if (n_rows == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  if (dtype == KVS_F32)
    lse_gather_kernel<float><<<n_rows, kRowThreads, 0, st>>>(static_cast<const float*>(logits), ld, vocab, targets,
                                                           (float)(1.0 / temperature), static_cast<float*>(logp),
                                                           static_cast<float*>(lse));
  else if (dtype == KVS_F64)
    lse_gather_kernel<double><<<n_rows, kRowThreads, 0, st>>>(static_cast<const double*>(logits), ld, vocab, targets,
                                                            1.0 / temperature, static_cast<double*>(logp),
                                                            static_cast<double*>(lse));
  else
    return KVS_E_UNSUPPORTED;
  return launch_rc();
}

KVS_API int kvs_lse_gather_backward(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab,
                                    const int64_t* targets, const void* lse, const void* grad, double temperature,
                                    int32_t dtype, void* dlogits, int64_t ld_out, int32_t out_dtype,
                                    kvs_stream_t stream) {
  if (!logits || !targets || !lse || !grad || !dlogits || n_rows < 0 || vocab <= 0 || ld < vocab || ld_out < vocab ||
      !(temperature > 0))
    return KVS_E_ARG;
  if (n_rows == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  if (dtype == KVS_F32) {
    const float* x = static_cast<const float*>(logits);
    const float* l = static_cast<const float*>(lse);
    const float* g = static_cast<const float*>(grad);
    const float tf = (float)(1.0 / temperature);
    if (out_dtype == KVS_F32)
      lse_gather_bwd_kernel<float, float><<<n_rows, kRowThreads, 0, st>>>(x, ld, vocab, targets, l, g, tf,
                                                                         static_cast<float*>(dlogits), ld_out);
    else if (out_dtype == KVS_BF16)
      lse_gather_bwd_kernel<float, __nv_bfloat16><<<n_rows, kRowThreads, 0, st>>>(
          x, ld, vocab, targets, l, g, tf, static_cast<__nv_bfloat16*>(dlogits), ld_out);
    else if (out_dtype == KVS_F16)
      lse_gather_bwd_kernel<float, __half><<<n_rows, kRowThreads, 0, st>>>(x, ld, vocab, targets, l, g, tf,
                                                                          static_cast<__half*>(dlogits), ld_out);
    else
      return KVS_E_UNSUPPORTED;
  } else if (dtype == KVS_F64 && out_dtype == KVS_F64) {
    lse_gather_bwd_kernel<double, double><<<n_rows, kRowThreads, 0, st>>>(
        static_cast<const double*>(logits), ld, vocab, targets, static_cast<const double*>(lse),
        static_cast<const double*>(grad), 1.0 / temperature, static_cast<double*>(dlogits), ld_out);
  } else {
    return KVS_E_UNSUPPORTED;
  }
  return launch_rc();
}

KVS_API int kvs_sample(const void* logits, int64_t ld, int32_t n_rows, int32_t vocab, double temperature,
                       int32_t dtype, int32_t greedy, uint64_t seed, uint64_t offset, int64_t* tokens, void* logp,
                       kvs_stream_t stream) {
  if (!logits || !tokens || !logp || n_rows < 0 || vocab <= 0 || ld < vocab || !(temperature > 0)) return KVS_E_ARG;
  if ((int64_t)n_rows * kSampleCTAs > INT_MAX) return KVS_E_ARG;
  if (n_rows == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  const int grid = n_rows * kSampleCTAs;
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  const uint32_t o0 = (uint32_t)offset, o1 = (uint32_t)(offset >> 32);
  const int gr = greedy ? 1 : 0;
  if (dtype == KVS_F32)
    sample_kernel<float><<<grid, kRowThreads, 0, st>>>(static_cast<const float*>(logits), ld, vocab,
                                                       (float)(1.0 / temperature), gr, k0, k1, o0, o1, tokens,
                                                       static_cast<float*>(logp));
  else if (dtype == KVS_F64)
    sample_kernel<double><<<grid, kRowThreads, 0, st>>>(static_cast<const double*>(logits), ld, vocab,
                                                        1.0 / temperature, gr, k0, k1, o0, o1, tokens,
                                                        static_cast<double*>(logp));
  else
    return KVS_E_UNSUPPORTED;
  return launch_rc();
}
