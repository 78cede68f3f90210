// Shared device/host helpers for libtessattn (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tx {

// Device status word values (written by kernels whose bounded waits give up).
// Low byte: kind; bits 8..23: site id (which wait gave up), for the error message.
enum : int {
  kStatusOk = 0,
  kStatusTimeout = 3,
  kStatusBadArg = 1,
};

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t bits) {
  return __uint_as_float(uint32_t(bits) << 16);
}

// Round-to-nearest-even float -> bf16 bit pattern (NaN kept quiet).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}

// Two floats -> packed bf16x2 (lo in bits 0..15), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float *p, size_t i) { return p[i]; }
  static __device__ __forceinline__ void store(float *p, size_t i, float v) { p[i] = v; }
};
template <> struct Elem<uint16_t> {
  static __device__ __forceinline__ float load(const uint16_t *p, size_t i) {
    return bf16_bits_to_f32(p[i]);
  }
  static __device__ __forceinline__ void store(uint16_t *p, size_t i, float v) {
    p[i] = f32_to_bf16_bits(v);
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// sin and cos of a float angle (a RoPE angle, position x inverse frequency): Cody-Waite
// reduction by 2*pi (2*pi split into a float head and a float tail; each product k * part
// is exact inside its fma) to [-pi, pi], then the hardware approximations, accurate to
// about 2^-21 absolute on that interval.  (A quadrant reduction with Taylor polynomials on
// the FMA pipe was measured slower inside the attention kernel.)
__device__ __forceinline__ void rope_sincos(float angle, float *sn, float *cs) {
  const float k = rintf(angle * 0.159154943091895336f);
  float r = fmaf(k, -6.28318548202514648f, angle);
  r = fmaf(k, 1.74845553e-07f, r);
  __sincosf(r, sn, cs);
}

// GELU in the erf form, 0.5 v (1 + erf(v / sqrt 2)), with erf from the rational
// approximation 7.1.26 of Abramowitz and Stegun (|error| <= 1.5e-7), as the reference's
// gelu_f32 evaluates it (kernels.metal:381-391): for z = |v| / sqrt 2,
// t = 1 / (1 + 0.3275911 z), tail = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^(-z^2)
// = 1 - erf(z), and gelu = 0.5 v tail for v < 0, 0.5 v (2 - tail) otherwise.
__device__ __forceinline__ float gelu_erf(float v) {
  const float z = fabsf(v) * 0.70710678118654752f;
  const float t = 1.0f / (1.0f + 0.3275911f * z);
  const float poly =
      ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
       0.254829592f) * t;
  const float tail = poly * expf(-z * z);
  return 0.5f * v * (v < 0.0f ? tail : 2.0f - tail);
}

// Records the first failure in the context's status word.
__device__ __forceinline__ void report_status(int *status, int code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace tx
