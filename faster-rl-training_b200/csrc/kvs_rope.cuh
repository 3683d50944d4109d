// Rotary embedding of one (x[i], x[i + D/2]) pair at a logical position.
//
// Follows kvstreams/rope.py:26-34,42-46: inv_freq[i] = 1 / theta**(2i/D) computed
// in float64 and stored as float32 (the host passes that table), the angle is
// float(position) * inv_freq[i] rounded once, and
//   out[i]       = x[i] * cos - x[i + D/2] * sin
//   out[i + D/2] = x[i + D/2] * cos + x[i] * sin
// with each product and the sum rounded separately, as the reference's
// elementwise tensor ops do.  float64 models use the same table widened to double
// and double arithmetic.  Every kernel that rotates (decode append, decode query,
// replay) calls this one function, so inference and replay rotate identically.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace kvs {

// sin and cos of the angle float(position) * inv_freq[i], the product rounded once
template <typename A, typename F>
__device__ __forceinline__ void rope_sincos(int64_t pos, F inv_freq, A& s, A& c);

template <>
__device__ __forceinline__ void rope_sincos<float, float>(int64_t pos, float inv_freq, float& s, float& c) {
  sincosf(__fmul_rn((float)pos, inv_freq), &s, &c);
}

template <>
__device__ __forceinline__ void rope_sincos<double, double>(int64_t pos, double inv_freq, double& s, double& c) {
  sincos(__dmul_rn((double)pos, inv_freq), &s, &c);
}

// the rotation of one pair by a precomputed angle, each product and sum rounded separately
__device__ __forceinline__ void rope_apply(float a, float b, float s, float c, float& r0, float& r1) {
  r0 = __fadd_rn(__fmul_rn(a, c), __fmul_rn(-b, s));
  r1 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

__device__ __forceinline__ void rope_apply(double a, double b, double s, double c, double& r0, double& r1) {
  r0 = __dadd_rn(__dmul_rn(a, c), __dmul_rn(-b, s));
  r1 = __dadd_rn(__dmul_rn(b, c), __dmul_rn(a, s));
}

template <typename A, typename F>
__device__ __forceinline__ void rope_rotate(A a, A b, int64_t pos, F inv_freq, A& r0, A& r1) {
  A s, c;
  rope_sincos<A, F>(pos, inv_freq, s, c);
  rope_apply(a, b, s, c, r0, r1);
}

}  // namespace kvs
