// Philox4x32-10 counter-based generator and the fixed-order arithmetic the
// sampling/acceptance kernels share with the CPU oracle.
//
// Philox4x32-10: Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as
// easy as 1, 2, 3" (SC'11); multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key
// increments 0x9E3779B9 / 0xBB67AE85, ten rounds.
//
// fm_exp: e^x by Cody-Waite range reduction (x = n ln2 + r, ln2 split into a
// 16-bit head and a tail), the degree-7 Taylor polynomial of e^r in Horner
// form with fused multiply-adds, and an exact power-of-two scale (in two
// steps below 2^-126 and at 2^128).  Every operation is an explicitly
// rounded intrinsic, so host C with the same steps reproduces it bit for bit.
#pragma once

#include "common.cuh"

namespace fm {

struct Philox4 {
  uint32_t v[4];
};

__device__ __forceinline__ Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint64_t seed) {
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  Philox4 r;
  r.v[0] = c0;
  r.v[1] = c1;
  r.v[2] = c2;
  r.v[3] = c3;
  return r;
}

// uniform in [0, 1): top 24 bits of word 0 times 2^-24
__device__ __forceinline__ float philox_uniform(uint64_t seed, uint32_t a, uint32_t b, uint32_t c, uint32_t purpose) {
  const Philox4 r = philox4x32_10(a, b, c, purpose, seed);
  return __fmul_rn((float)(r.v[0] >> 8), 5.9604644775390625e-08f);
}

__device__ __forceinline__ float fm_exp(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return __int_as_float(0x7f800000);
  if (x < -103.972084f) return 0.0f;
  // n = x log2(e) rounded half-to-even (the value rintf gives) by the
  // 1.5 * 2^23 shifter, exact for |x log2(e)| < 2^22 (here <= 150); the
  // shifter's low mantissa bits are n as an integer, so no float->int
  // conversion is issued.
  const float t = __fadd_rn(__fmul_rn(x, 1.44269502162933349609f), 12582912.0f);
  const float n = __fsub_rn(t, 12582912.0f);
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.42860682030941723212e-6f, r);
  float p = 1.98412698e-4f;
  p = __fmaf_rn(p, r, 1.38888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333e-3f);
  p = __fmaf_rn(p, r, 4.16666667e-2f);
  p = __fmaf_rn(p, r, 1.66666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int e = __float_as_int(t) - 0x4B400000;
  // e = 128 (x <= 88.7228): scale by 2^127, then 2, so a product below FLT_MAX stays finite
  if (e > 127) return __fmul_rn(__fmul_rn(p, __uint_as_float(254u << 23)), 2.0f);
  if (e >= -126) return __fmul_rn(p, __uint_as_float((uint32_t)(e + 127) << 23));
  return __fmul_rn(__fmul_rn(p, __uint_as_float((uint32_t)(e + 126 + 127) << 23)), __uint_as_float(1u << 23));
}

// fm_exp of two lanes with the packed fp32x2 add / multiply / fma of sm_100:
// every lane rounds exactly as the scalar steps of fm_exp do (the same
// operations in the same order; -n * c == n * -c exactly), so each value is
// fm_exp's.  The fast path needs e = bits(t) - 0x4B400000 in [-126, 127] on
// both lanes, where fm_exp scales with one multiply; NaN, infinities, large
// inputs and the two-step scales (e < -126, e = 128) all fall outside, and
// such a pair is recomputed by fm_exp itself.  The scale 2^e is (bits(t) << 23) + bits(1.0f),
// as 0x4B400000 << 23 vanishes modulo 2^32.
__device__ __forceinline__ float2 fm_exp2(float2 x) {
  const float2 t = __fadd2_rn(__fmul2_rn(x, make_float2(1.44269502162933349609f, 1.44269502162933349609f)),
                              make_float2(12582912.0f, 12582912.0f));
  const float2 n = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  float2 r = __ffma2_rn(n, make_float2(-0.693145751953125f, -0.693145751953125f), x);
  r = __ffma2_rn(n, make_float2(-1.42860682030941723212e-6f, -1.42860682030941723212e-6f), r);
  float2 p = __ffma2_rn(make_float2(1.98412698e-4f, 1.98412698e-4f), r, make_float2(1.38888889e-3f, 1.38888889e-3f));
  p = __ffma2_rn(p, r, make_float2(8.33333333e-3f, 8.33333333e-3f));
  p = __ffma2_rn(p, r, make_float2(4.16666667e-2f, 4.16666667e-2f));
  p = __ffma2_rn(p, r, make_float2(1.66666667e-1f, 1.66666667e-1f));
  p = __ffma2_rn(p, r, make_float2(0.5f, 0.5f));
  p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
  p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
  const uint32_t b0 = __float_as_uint(t.x), b1 = __float_as_uint(t.y);
  // e + 126 = bits - (0x4B400000 - 126), in [0, 253] on the fast path
  if (max(b0 - 0x4B3FFF82u, b1 - 0x4B3FFF82u) > 253u) return make_float2(fm_exp(x.x), fm_exp(x.y));
  return __fmul2_rn(p, make_float2(__uint_as_float((b0 << 23) + 0x3F800000u), __uint_as_float((b1 << 23) + 0x3F800000u)));
}

// Box-Muller on Philox words: pair p (elements 2p, 2p+1) uses counter (p, 0, offset, 4)
__device__ __forceinline__ void normal_pair(uint64_t seed, uint32_t offset, long long p, float& z0, float& z1) {
  const Philox4 r = philox4x32_10((uint32_t)p, (uint32_t)(p >> 32), offset, 4u, seed);
  const float u1 = __fmul_rn((float)(r.v[0] >> 8) + 0.5f, 5.9604644775390625e-08f);
  const float u2 = __fmul_rn((float)(r.v[1] >> 8), 5.9604644775390625e-08f);
  const float rad = sqrtf(-2.0f * logf(u1));
  float sv, cv;
  sincospif(2.0f * u2, &sv, &cv);
  z0 = rad * cv;
  z1 = rad * sv;
}

}  // namespace fm
