// Shared helpers for the KV-streams sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kvs_b200.h"  // include/ (the build passes -I<repo>/include)

#define KVS_API extern "C" __attribute__((visibility("default")))

namespace kvs {

constexpr int64_t kNever = INT64_MAX;

inline cudaStream_t to_cuda(kvs_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Process-wide count of kernels this library launched (kvs_launch_count).
void count_launch();

// Host: count the launch just issued and convert its error into a return code.
inline int launch_rc() {
  count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KVS_OK : KVS_E_LAUNCH;
}

// First error wins: status[0] is set once, details only by the thread that set it.
__device__ __forceinline__ void set_status(int32_t* status, int code, int a, int b, int c) {
  if (atomicCAS(status, 0, code) == 0) {
    status[1] = a;
    status[2] = b;
    status[3] = c;
  }
}

// ---------------------------------------------------------------- element types
template <typename T> struct Acc { using type = float; };
template <> struct Acc<double> { using type = double; };

template <typename T> __device__ __forceinline__ typename Acc<T>::type to_acc(T x);
template <> __device__ __forceinline__ float to_acc<float>(float x) { return x; }
template <> __device__ __forceinline__ double to_acc<double>(double x) { return x; }
template <> __device__ __forceinline__ float to_acc<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <> __device__ __forceinline__ float to_acc<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_acc(typename Acc<T>::type x);
template <> __device__ __forceinline__ float from_acc<float>(float x) { return x; }
template <> __device__ __forceinline__ double from_acc<double>(double x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_acc<__half>(float x) { return __float2half_rn(x); }

// ---------------------------------------------------------------- block scan
// Exclusive prefix sum over one int per thread of a 1-D block (blockDim.x <= 1024,
// multiple of 32).  Returns the exclusive prefix; *total gets the block sum.
// `smem` must hold 33 ints.  Contains __syncthreads(): call from all threads.
__device__ __forceinline__ int block_exclusive_scan(int v, int* smem, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) smem[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? smem[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nwarps) smem[lane] = w;  // inclusive prefix of warp sums
    if (lane == 31) smem[32] = w;
  }
  __syncthreads();
  int warp_prefix = warp > 0 ? smem[warp - 1] : 0;
  int result = warp_prefix + x - v;
  if (total) *total = smem[32];
  __syncthreads();
  return result;
}

__device__ __forceinline__ long long block_sum_ll(long long v, long long* smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  long long r = 0;
  for (int w = 0; w < nwarps; ++w) r += smem[w];
  __syncthreads();
  return r;
}

__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ __forceinline__ size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace kvs
