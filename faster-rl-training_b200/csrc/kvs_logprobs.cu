// Log-probabilities of target tokens from lm_head logits (training/logprobs.py:17-20):
// logp = x_t / T - log sum_v exp(x_v / T), in one pass over each logits row, and its
// gradient dlogits = g (onehot(t) - softmax(x / T)) / T.  The reference materialises
// log_softmax(logits / T) for every row and gathers from it; here the row is read once.

#include <algorithm>
#include <cmath>

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
