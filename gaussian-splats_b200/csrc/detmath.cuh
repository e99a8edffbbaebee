// Deterministic float32 exp / log for the rasterizer kernels.
//
// Integer outputs (tile bounds and counts, per-pixel contributor counts)
// depend on exp/log results to the last bit, so the operator fixes one
// algorithm for each and evaluates it with IEEE float32 add/mul/div/sqrt and
// explicit fmaf only (the library is compiled with --fmad=false, so nothing
// else is fused). The CPU oracle evaluates the identical algorithm; a GPU test
// checks both agree bit for bit over a sweep of inputs.
//
// exp: Cody & Waite (1980) reduction x = n ln2 + r, |r| <= ln2/2, with ln2
//      split into a 16-significant-bit head (n * head exact for |n| < 256) and
//      a float tail; e^r from its degree-7 Taylor polynomial (truncation
//      error < 6e-9 relative) in Horner form; 2^n applied through the
//      exponent field (two steps below 2^-126 or above 2^127).
// log: x = 2^e m, m in [sqrt(1/2), sqrt(2)); log m = 2 atanh(s),
//      s = (m - 1)/(m + 1), from 2(s + s^3/3 + s^5/5 + s^7/7 + s^9/9);
//      log x = e ln2 + log m with the same ln2 split.
#pragma once

#include <cstdint>

namespace gs {

constexpr float kLn2Hi = 0.693145751953125f;        // 45426 / 65536
constexpr float kLn2Lo = 1.42860682030941723e-06f;  // ln 2 - kLn2Hi
constexpr float kLog2e = 1.44269504088896341f;

__device__ __forceinline__ float det_exp(float x) {
  if (x != x) return x;
  if (x > 88.8f) return __int_as_float(0x7f800000);
  if (x < -104.0f) return 0.0f;
  float n = rintf(x * kLog2e);
  float r = fmaf(-n, kLn2Hi, x);
  r = fmaf(-n, kLn2Lo, r);
  float p = 1.98412698e-4f;        // 1/5040
  p = fmaf(p, r, 1.38888889e-3f);  // 1/720
  p = fmaf(p, r, 8.33333333e-3f);  // 1/120
  p = fmaf(p, r, 4.16666667e-2f);  // 1/24
  p = fmaf(p, r, 1.66666667e-1f);  // 1/6
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int e = static_cast<int>(n);
  if (e > 127) { p *= 1.70141183e38f; e -= 127; }    // 2^127
  if (e < -126) { p *= 1.17549435e-38f; e += 126; }  // 2^-126
  return p * __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

// exp for arguments in [-87, 0] with no NaN: the compositing hot path, where
// the argument is -d^2/2 of a finite d^2 >= 0 already tested against a cutoff
// of at most 2 log(255) + 1e-3 (so x >= -5.6). 2^n is then a normal float
// (n >= -126), so det_exp's step for subnormal results is left out. Same bits
// as det_exp on that domain.
__device__ __forceinline__ float det_exp_nonpositive(float x) {
  // rintf(x log2e) without a conversion instruction: adding 1.5 * 2^23 to a
  // value below 2^22 in magnitude rounds it to the nearest integer, ties to
  // even, as rintf does; the integer is then also the sum's low bits.
  const float shifted = x * kLog2e + 12582912.0f;
  const float n = shifted - 12582912.0f;
  float r = fmaf(-n, kLn2Hi, x);
  r = fmaf(-n, kLn2Lo, r);
  float p = 1.98412698e-4f;
  p = fmaf(p, r, 1.38888889e-3f);
  p = fmaf(p, r, 8.33333333e-3f);
  p = fmaf(p, r, 4.16666667e-2f);
  p = fmaf(p, r, 1.66666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int e = __float_as_int(shifted) - 0x4B400000;  // n as an integer
  // p * 2^n: p lies in [0.7, 1.42] and n >= -126 keeps the product normal,
  // where the scaling is exact -- an add to p's exponent field.
  return __int_as_float(__float_as_int(p) + (e << 23));
}

__device__ __forceinline__ float det_log(float x) {
  if (!(x > 0.0f)) return x == 0.0f ? __int_as_float(0xff800000) : __int_as_float(0x7fc00000);
  if (x == __int_as_float(0x7f800000)) return x;
  int e = 0;
  uint32_t bits = __float_as_uint(x);
  if (bits < 0x00800000u) { x *= 8388608.0f; bits = __float_as_uint(x); e = -23; }
  e += static_cast<int>(bits >> 23) - 127;
  float m = __uint_as_float((bits & 0x007fffffu) | 0x3f800000u);
  if (m > 1.41421354f) { m *= 0.5f; e += 1; }
  float f = m - 1.0f;
  float s = f / (2.0f + f);
  float s2 = s * s;
  float poly = fmaf(s2, 2.22222222e-1f, 2.85714287e-1f);  // 2/9, 2/7
  poly = fmaf(poly, s2, 4.00000006e-1f);                    // 2/5
  poly = fmaf(poly, s2, 6.66666687e-1f);                    // 2/3
  float lm = fmaf(s * s2, poly, 2.0f * s);
  float fe = static_cast<float>(e);
  return fmaf(fe, kLn2Hi, fmaf(fe, kLn2Lo, lm));
}

__device__ __forceinline__ float det_sigmoid(float x) { return 1.0f / (1.0f + det_exp(-x)); }
__device__ __forceinline__ float det_rsqrt(float x) { return 1.0f / sqrtf(x); }

}  // namespace gs
