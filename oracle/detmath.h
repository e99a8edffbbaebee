/*
 * Deterministic float32 exp / log for the CPU oracle (test infrastructure).
 *
 * Integer outputs of the rasterizer (tile bounds, per-Gaussian tile counts,
 * per-pixel contributor counts) hinge on exp/log/sqrt results to the last
 * bit. libm and CUDA's math library do not promise the same bits, so the
 * operator's numeric contract fixes one algorithm for each transcendental and
 * both the CUDA kernels and this oracle evaluate it with IEEE-754 float32
 * add/mul/div/sqrt and explicit fused multiply-adds only. Compile with
 * -ffp-contract=off so that no other multiply-add is fused.
 *
 * exp: Cody & Waite (1980) argument reduction x = n ln2 + r, |r| <= ln2/2,
 *      with ln2 split into a 16-significant-bit head (so n * head is exact
 *      for |n| < 256) and a float tail; e^r from its degree-7 Taylor
 *      polynomial (truncation error < 6e-9 relative on |r| <= 0.347) in
 *      Horner form; scaling by 2^n through the exponent field.
 * log: x = 2^e m with m in [sqrt(1/2), sqrt(2)); log m = 2 atanh(s),
 *      s = (m - 1) / (m + 1), from the odd series 2(s + s^3/3 + ... + s^9/9)
 *      (truncation error < 3e-9 relative for |s| <= 0.1716);
 *      log x = e ln2 + log m with the same ln2 split.
 * The CUDA copy of these two functions lives in the library's detmath.cuh;
 * a GPU test checks both copies agree bit for bit over a sweep of inputs.
 */
#ifndef GSO_DETMATH_H
#define GSO_DETMATH_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#define GSO_LN2_HI 0.693145751953125f       /* 45426 / 65536 */
#define GSO_LN2_LO 1.42860682030941723e-06f /* ln 2 - GSO_LN2_HI */
#define GSO_LOG2E 1.44269504088896341f

static inline uint32_t gso_f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float gso_u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

static inline float gso_exp(float x) {
    if (x != x) return x;
    if (x > 88.8f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    float n = rintf(x * GSO_LOG2E);
    float r = fmaf(-n, GSO_LN2_HI, x);
    r = fmaf(-n, GSO_LN2_LO, r);
    float p = 1.98412698e-4f;        /* 1/5040 */
    p = fmaf(p, r, 1.38888889e-3f);  /* 1/720 */
    p = fmaf(p, r, 8.33333333e-3f);  /* 1/120 */
    p = fmaf(p, r, 4.16666667e-2f);  /* 1/24 */
    p = fmaf(p, r, 1.66666667e-1f);  /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int e = (int)n;
    if (e > 127) { p *= 1.70141183e38f; e -= 127; }   /* 2^127 */
    if (e < -126) { p *= 1.17549435e-38f; e += 126; } /* 2^-126 */
    return p * gso_u2f((uint32_t)(e + 127) << 23);
}

static inline float gso_log(float x) {
    if (!(x > 0.0f)) return x == 0.0f ? -INFINITY : NAN;
    if (x == INFINITY) return x;
    int e = 0;
    uint32_t bits = gso_f2u(x);
    if (bits < 0x00800000u) { x *= 8388608.0f; bits = gso_f2u(x); e = -23; }
    e += (int)(bits >> 23) - 127;
    float m = gso_u2f((bits & 0x007fffffu) | 0x3f800000u);
    if (m > 1.41421354f) { m *= 0.5f; e += 1; }
    float f = m - 1.0f;
    float s = f / (2.0f + f);
    float s2 = s * s;
    float poly = fmaf(s2, 2.22222222e-1f, 2.85714287e-1f); /* 2/9, 2/7 */
    poly = fmaf(poly, s2, 4.00000006e-1f);                   /* 2/5 */
    poly = fmaf(poly, s2, 6.66666687e-1f);                   /* 2/3 */
    float lm = fmaf(s * s2, poly, 2.0f * s);
    float fe = (float)e;
    return fmaf(fe, GSO_LN2_HI, fmaf(fe, GSO_LN2_LO, lm));
}

static inline float gso_sigmoid(float x) { return 1.0f / (1.0f + gso_exp(-x)); }
static inline float gso_rsqrt(float x) { return 1.0f / sqrtf(x); }

#endif
