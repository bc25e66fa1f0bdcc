// Device-side arithmetic of the sampler spec: the order key, the fixed-point
// weight, the exponential E() and Philox4x32-10.  Every float operation uses
// an explicit round-to-nearest intrinsic so nvcc cannot contract a multiply
// and an add into an FMA: the results must equal, bit for bit, the same
// binary32 operations performed one at a time on the host.
#pragma once
#include <cstdint>

namespace mstar {

constexpr float kL2E = 0x1.715476p+0f;  // log2(e) rounded to binary32
constexpr float kTwo32 = 4294967296.0f;

// E(y) ~ e^y for y <= 0: t = y*log2(e); t = n + f with n = floor(t);
// 2^f by its degree-8 Taylor series in Horner form (coefficients
// (ln 2)^k / k! rounded to binary32), clamped to 2 so E stays
// monotone across integer steps of t; result p * 2^n (exact scaling, n >= -64).
__device__ __forceinline__ float spec_exp(float y) {
  if (y == 0.0f) return 1.0f;
  const float t = __fmul_rn(y, kL2E);
  if (!(t >= -64.0f)) return 0.0f;
  const float n = floorf(t);
  const float f = __fsub_rn(t, n);
  float p = 0x1.62c022p-20f;
  p = __fadd_rn(__fmul_rn(p, f), 0x1.ffcbfcp-17f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.430912p-13f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.5d87fep-10f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.3b2ab6p-7f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.c6b08ep-5f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.ebfbep-3f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.62e43p-1f);
  p = __fadd_rn(__fmul_rn(p, f), 1.0f);
  p = fminf(p, 2.0f);
  const float scale = __int_as_float((127 + (int)n) << 23);  // 2^n, n in [-64, 0]
  return __fmul_rn(p, scale);
}

// Order-preserving key of a non-NaN float; -0 and +0 share a key.
__device__ __forceinline__ uint32_t okey(float x) {
  uint32_t b = __float_as_uint(x);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float okey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// e = E(x - m) (1 when x == m); w = rint(e * 2^32).
__device__ __forceinline__ float spec_e(float x, float m) {
  return (x == m) ? 1.0f : spec_exp(__fsub_rn(x, m));
}
__device__ __forceinline__ uint64_t spec_w_from_e(float e) {
  return (uint64_t)__float2ull_rn(__fmul_rn(e, kTwo32));
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11); first output word of
// counter (offset lo, offset hi, 0, 0) under key seed.
__device__ __forceinline__ uint32_t philox_word0(uint64_t seed, uint64_t offset) {
  uint32_t c0 = (uint32_t)offset, c1 = (uint32_t)(offset >> 32), c2 = 0u, c3 = 0u;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  return c0;
}

__device__ __forceinline__ float philox_uniform(uint64_t seed, uint64_t offset) {
  return __fmul_rn((float)(philox_word0(seed, offset) >> 8), 0x1.0p-24f);
}

// Draw point r in [0, W) for uniform u: floor(u * W) in binary64, clamped.
__device__ __forceinline__ uint64_t draw_point(float u, uint64_t W) {
  if (!(u > 0.0f) || W == 0) return 0;
  const double t = floor(__dmul_rn((double)u, (double)W));
  return (t >= (double)W) ? W - 1 : (uint64_t)t;
}

}  // namespace mstar
