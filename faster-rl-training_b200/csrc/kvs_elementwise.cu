// The two elementwise steps of each decoder layer (model.py:29-36, 78-86) as single passes for
// half-precision models: RMSNorm of a row (fp32 sum of squares, one rounding of x * rstd * w)
// and the SwiGLU product silu(gate) * up read from the fused gate|up projection output
// (fp32 arithmetic, one rounding).  PyTorch runs each of them as two or more kernels, and the
// decode step of a rollout batch (64 rows) is dominated by their fixed costs.

#include <algorithm>
#include <cmath>

#include "kvs_common.cuh"

using namespace kvs;

namespace {

template <typename T> __device__ __forceinline__ float tof(T x);
template <> __device__ __forceinline__ float tof<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float tof<__half>(__half x) { return __half2float(x); }
template <typename T> __device__ __forceinline__ T fromf(float x);
template <> __device__ __forceinline__ __nv_bfloat16 fromf<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half fromf<__half>(float x) { return __float2half_rn(x); }

constexpr int kNormThreads = 256;

// one CTA per row; 8 elements (16 bytes) per thread and step
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, float* __restrict__ rstd_out,
                int dim, int64_t ld_x, int64_t ld_y, float eps) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ld_x;
  T* yr = y + row * ld_y;
  float ss = 0.f;
  const int nvec = dim / 8;
  // the first kKeep vectors of each thread stay in registers for the second pass
  constexpr int kKeep = 4;
  uint4 keep[kKeep];
#pragma unroll
  for (int u = 0; u < kKeep; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    if (i < nvec) keep[u] = reinterpret_cast<const uint4*>(xr)[i];
  }
#pragma unroll
  for (int u = 0; u < kKeep; ++u) {
    if (threadIdx.x + u * kNormThreads >= nvec) break;
    const T* e = reinterpret_cast<const T*>(&keep[u]);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float f = tof(e[k]);
      ss += f * f;
    }
  }
  for (int i = threadIdx.x + kKeep * kNormThreads; i < nvec; i += kNormThreads) {
    const uint4 q = reinterpret_cast<const uint4*>(xr)[i];
    const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float f = tof(e[k]);
      ss += f * f;
    }
  }
  for (int i = nvec * 8 + threadIdx.x; i < dim; i += kNormThreads) {
    const float f = tof(xr[i]);
    ss += f * f;
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)dim + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[row] = r;
  auto emit = [&](int i, const uint4& q) {
    const uint4 wq = reinterpret_cast<const uint4*>(w)[i];
    const T* e = reinterpret_cast<const T*>(&q);
    const T* we = reinterpret_cast<const T*>(&wq);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < 8; ++k) oe[k] = fromf<T>(tof(e[k]) * r * tof(we[k]));
    reinterpret_cast<uint4*>(yr)[i] = o;
  };
#pragma unroll
  for (int u = 0; u < kKeep; ++u) {
    const int i = threadIdx.x + u * kNormThreads;
    if (i < nvec) emit(i, keep[u]);
  }
  for (int i = threadIdx.x + kKeep * kNormThreads; i < nvec; i += kNormThreads)
    emit(i, reinterpret_cast<const uint4*>(xr)[i]);
  for (int i = nvec * 8 + threadIdx.x; i < dim; i += kNormThreads) yr[i] = fromf<T>(tof(xr[i]) * r * tof(w[i]));
}

// RMSNorm backward with the forward's per-row rstd (model.py:29-36 differentiated):
//   gx[r] = rstd_r (gxn - xn mean_j(gxn xn)),  xn = x[r] rstd_r,  gxn = gy[r] w   (fp32, one rounding)
//   gw    = sum_r gy[r] xn[r]
// A CTA takes rows blockIdx.x, blockIdx.x + gridDim.x, ...; thread t owns the 16-byte chunks
// t and t + 512 (dim <= 8192) and keeps w and its gw sums in registers;
// each CTA writes its gw sums to its own row of `part`, summed in CTA order by rms_norm_gw_kernel
// (no float atomics: the result does not depend on scheduling).
constexpr int kBwdThreads = 512, kBwdChunks = 2;

template <typename T>
__global__ void __launch_bounds__(kBwdThreads, 1)
rms_norm_bwd_kernel(const T* __restrict__ x, const T* __restrict__ w, const float* __restrict__ rstd,
                    const T* __restrict__ gy, T* __restrict__ gx, float* __restrict__ part, int64_t n_rows, int dim,
                    int64_t ld_x, int64_t ld_gy, int64_t ld_gx) {
  const int nvec = dim / 8;
  float wf[kBwdChunks][8], acc[kBwdChunks][8];
#pragma unroll
  for (int u = 0; u < kBwdChunks; ++u) {
    const int i = threadIdx.x + u * kBwdThreads;
    uint4 wq = make_uint4(0, 0, 0, 0);
    if (i < nvec) wq = reinterpret_cast<const uint4*>(w)[i];
    const T* we = reinterpret_cast<const T*>(&wq);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      wf[u][k] = tof(we[k]);
      acc[u][k] = 0.f;
    }
  }
  __shared__ float red[kBwdThreads / 32];
  for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x) {
    const float r = rstd[row];
    uint4 xq[kBwdChunks], gq[kBwdChunks];
#pragma unroll
    for (int u = 0; u < kBwdChunks; ++u) {
      const int i = threadIdx.x + u * kBwdThreads;
      xq[u] = gq[u] = make_uint4(0, 0, 0, 0);
      if (i < nvec) {
        xq[u] = reinterpret_cast<const uint4*>(x + row * ld_x)[i];
        gq[u] = reinterpret_cast<const uint4*>(gy + row * ld_gy)[i];
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int u = 0; u < kBwdChunks; ++u) {
      const T* xe = reinterpret_cast<const T*>(&xq[u]);
      const T* ge = reinterpret_cast<const T*>(&gq[u]);
#pragma unroll
      for (int k = 0; k < 8; ++k) dot += (tof(ge[k]) * wf[u][k]) * (tof(xe[k]) * r);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dot;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kBwdThreads / 32; ++i) tot += red[i];
    __syncthreads();  // red is rewritten for the next row
    const float mean = tot / (float)dim;
#pragma unroll
    for (int u = 0; u < kBwdChunks; ++u) {
      const int i = threadIdx.x + u * kBwdThreads;
      if (i >= nvec) break;
      const T* xe = reinterpret_cast<const T*>(&xq[u]);
      const T* ge = reinterpret_cast<const T*>(&gq[u]);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float xn = tof(xe[k]) * r, g = tof(ge[k]);
        oe[k] = fromf<T>(r * (g * wf[u][k] - xn * mean));
        acc[u][k] += g * xn;
      }
      reinterpret_cast<uint4*>(gx + row * ld_gx)[i] = o;
    }
  }
#pragma unroll
  for (int u = 0; u < kBwdChunks; ++u) {
    const int i = threadIdx.x + u * kBwdThreads;
    if (i >= nvec) break;
    float4* dst = reinterpret_cast<float4*>(part + (int64_t)blockIdx.x * dim + i * 8);
    dst[0] = make_float4(acc[u][0], acc[u][1], acc[u][2], acc[u][3]);
    dst[1] = make_float4(acc[u][4], acc[u][5], acc[u][6], acc[u][7]);
  }
}

// gw[j] = sum over the CTAs' partial rows, in CTA order
__global__ void rms_norm_gw_kernel(const float* __restrict__ part, float* __restrict__ gw, int n_parts, int dim) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= dim) return;
  float s = 0.f;
  for (int c = 0; c < n_parts; ++c) s += part[(int64_t)c * dim + j];
  gw[j] = s;
}

int norm_bwd_ctas(int64_t n_rows) { return (int)std::max<int64_t>(1, std::min<int64_t>(n_rows, 148)); }

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

// out[r][j] = silu(gu[r][j]) * gu[r][F + j]; 8 outputs per thread
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t rows, int F, int64_t ld_gu,
                                int64_t ld_out) {
  const int nvec = F / 8;
  const int64_t total = rows * nvec;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / nvec;
    const int j = (int)(idx % nvec);
    const uint4 gq = reinterpret_cast<const uint4*>(gu + r * ld_gu)[j];
    const uint4 uq = reinterpret_cast<const uint4*>(gu + r * ld_gu + F)[j];
    const T* g = reinterpret_cast<const T*>(&gq);
    const T* u = reinterpret_cast<const T*>(&uq);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < 8; ++k) oe[k] = fromf<T>(silu_f(tof(g[k])) * tof(u[k]));
    reinterpret_cast<uint4*>(out + r * ld_out)[j] = o;
  }
}

// d gate = grad * up * s (1 + gate (1 - s)), d up = grad * silu(gate), s = sigmoid(gate)
template <typename T>
__global__ void silu_mul_bwd_kernel(const T* __restrict__ gu, const T* __restrict__ grad, T* __restrict__ dgu,
                                    int64_t rows, int F, int64_t ld_gu, int64_t ld_grad, int64_t ld_dgu) {
  const int nvec = F / 8;
  const int64_t total = rows * nvec;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / nvec;
    const int j = (int)(idx % nvec);
    const uint4 gq = reinterpret_cast<const uint4*>(gu + r * ld_gu)[j];
    const uint4 uq = reinterpret_cast<const uint4*>(gu + r * ld_gu + F)[j];
    const uint4 dq = reinterpret_cast<const uint4*>(grad + r * ld_grad)[j];
    const T* g = reinterpret_cast<const T*>(&gq);
    const T* u = reinterpret_cast<const T*>(&uq);
    const T* d = reinterpret_cast<const T*>(&dq);
    uint4 og, ou;
    T* oge = reinterpret_cast<T*>(&og);
    T* oue = reinterpret_cast<T*>(&ou);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float gf = tof(g[k]), uf = tof(u[k]), df = tof(d[k]);
      const float s = 1.f / (1.f + __expf(-gf));
      oge[k] = fromf<T>(df * uf * s * (1.f + gf * (1.f - s)));
      oue[k] = fromf<T>(df * gf * s);
    }
    reinterpret_cast<uint4*>(dgu + r * ld_dgu)[j] = og;
    reinterpret_cast<uint4*>(dgu + r * ld_dgu + F)[j] = ou;
  }
}

int grid_for(int64_t work) { return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 148 * 16)); }

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

KVS_API int kvs_rms_norm(const void* x, const void* weight, void* y, float* rstd, int64_t n_rows, int32_t dim,
                         int64_t ld_x, int64_t ld_y, double eps, int32_t dtype, kvs_stream_t stream) {
  if (!x || !weight || !y || n_rows < 0 || dim <= 0 || ld_x < dim || ld_y < dim) return KVS_E_ARG;
  if (dim % 8 || ld_x % 8 || ld_y % 8 || !al16(x) || !al16(weight) || !al16(y)) return KVS_E_UNSUPPORTED;
  if (n_rows == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  if (dtype == KVS_BF16)
    rms_norm_kernel<__nv_bfloat16><<<(unsigned)n_rows, kNormThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
        static_cast<__nv_bfloat16*>(y), rstd, dim, ld_x, ld_y, (float)eps);
  else if (dtype == KVS_F16)
    rms_norm_kernel<__half><<<(unsigned)n_rows, kNormThreads, 0, st>>>(
        static_cast<const __half*>(x), static_cast<const __half*>(weight), static_cast<__half*>(y), rstd, dim, ld_x,
        ld_y, (float)eps);
  else
    return KVS_E_UNSUPPORTED;
  return launch_rc();
}

KVS_API int kvs_silu_mul(const void* gu, void* out, int64_t n_rows, int32_t f, int64_t ld_gu, int64_t ld_out,
                         int32_t dtype, kvs_stream_t stream) {
  if (!gu || !out || n_rows < 0 || f <= 0 || ld_gu < 2 * (int64_t)f || ld_out < f) return KVS_E_ARG;
  if (f % 8 || ld_gu % 8 || ld_out % 8 || !al16(gu) || !al16(out)) return KVS_E_UNSUPPORTED;
  if (n_rows == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  const int grid = grid_for(n_rows * (f / 8));
  if (dtype == KVS_BF16)
    silu_mul_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(gu),
                                                       static_cast<__nv_bfloat16*>(out), n_rows, f, ld_gu, ld_out);
  else if (dtype == KVS_F16)
    silu_mul_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(gu), static_cast<__half*>(out), n_rows,
                                                 f, ld_gu, ld_out);
  else
    return KVS_E_UNSUPPORTED;
  return launch_rc();
}

KVS_API int kvs_silu_mul_backward(const void* gu, const void* grad, void* dgu, int64_t n_rows, int32_t f,
                                  int64_t ld_gu, int64_t ld_grad, int64_t ld_dgu, int32_t dtype,
                                  kvs_stream_t stream) {
  if (!gu || !grad || !dgu || n_rows < 0 || f <= 0 || ld_gu < 2 * (int64_t)f || ld_grad < f ||
      ld_dgu < 2 * (int64_t)f)
    return KVS_E_ARG;
  if (f % 8 || ld_gu % 8 || ld_grad % 8 || ld_dgu % 8 || !al16(gu) || !al16(grad) || !al16(dgu))
    return KVS_E_UNSUPPORTED;
  if (n_rows == 0) return KVS_OK;
  const cudaStream_t st = to_cuda(stream);
  const int grid = grid_for(n_rows * (f / 8));
  if (dtype == KVS_BF16)
    silu_mul_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(gu), static_cast<const __nv_bfloat16*>(grad),
        static_cast<__nv_bfloat16*>(dgu), n_rows, f, ld_gu, ld_grad, ld_dgu);
  else if (dtype == KVS_F16)
    silu_mul_bwd_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(gu), static_cast<const __half*>(grad),
                                                    static_cast<__half*>(dgu), n_rows, f, ld_gu, ld_grad, ld_dgu);
  else
    return KVS_E_UNSUPPORTED;
  return launch_rc();
}

KVS_API size_t kvs_rms_norm_backward_scratch_bytes(int64_t n_rows, int32_t dim) {
  if (n_rows <= 0 || dim <= 0) return 0;
  return (size_t)norm_bwd_ctas(n_rows) * (size_t)dim * sizeof(float);
}

KVS_API int kvs_rms_norm_backward(const void* x, const void* weight, const float* rstd, const void* gy, void* gx,
                                  float* gw, int64_t n_rows, int32_t dim, int64_t ld_x, int64_t ld_gy, int64_t ld_gx,
                                  int32_t dtype, void* scratch, size_t scratch_bytes, kvs_stream_t stream) {
  if (!x || !weight || !rstd || !gy || !gx || !gw || n_rows < 0 || dim <= 0 || ld_x < dim || ld_gy < dim ||
      ld_gx < dim)
    return KVS_E_ARG;
  if (dim % 8 || dim > 8 * kBwdThreads * kBwdChunks || ld_x % 8 || ld_gy % 8 || ld_gx % 8 || !al16(x) ||
      !al16(weight) || !al16(gy) || !al16(gx))
    return KVS_E_UNSUPPORTED;
  const cudaStream_t st = to_cuda(stream);
  if (n_rows == 0) return cudaMemsetAsync(gw, 0, (size_t)dim * sizeof(float), st) == cudaSuccess ? KVS_OK : KVS_E_LAUNCH;
  if (!scratch || scratch_bytes < kvs_rms_norm_backward_scratch_bytes(n_rows, dim) || !al16(scratch))
    return KVS_E_SCRATCH;
  const int grid = norm_bwd_ctas(n_rows);
  float* part = static_cast<float*>(scratch);
  if (dtype == KVS_BF16)
    rms_norm_bwd_kernel<__nv_bfloat16><<<grid, kBwdThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight), rstd,
        static_cast<const __nv_bfloat16*>(gy), static_cast<__nv_bfloat16*>(gx), part, n_rows, dim, ld_x, ld_gy, ld_gx);
  else if (dtype == KVS_F16)
    rms_norm_bwd_kernel<__half><<<grid, kBwdThreads, 0, st>>>(
        static_cast<const __half*>(x), static_cast<const __half*>(weight), rstd, static_cast<const __half*>(gy),
        static_cast<__half*>(gx), part, n_rows, dim, ld_x, ld_gy, ld_gx);
  else
    return KVS_E_UNSUPPORTED;
  int rc = launch_rc();
  if (rc) return rc;
  rms_norm_gw_kernel<<<(dim + 255) / 256, 256, 0, st>>>(part, gw, grid, dim);
  return launch_rc();
}
