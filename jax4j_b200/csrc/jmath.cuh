// Single-precision tanh and logistic sigmoid for the elementwise kernels and
// for the generated fused kernels.  J4C_MATH_DEFS is both compiled here (nvcc)
// and handed to NVRTC as text (J4C_MATH_SRC), so an eager op and the same op
// inside a fused chain compute the same bits.
//
// Both evaluate one exponential, e^y = 2^(y log2 e) with ex2.approx.ftz
// (PTX; 2 ulp) of the rounded product y * (float) log2 e, and one
// approximate reciprocal (rcp.approx.ftz, 1 ulp).  The reference evaluates
// them in double and narrows (core/ConcreteNDArray.java:657-664); its
// tolerance for them is 1e-5 relative.  Error bounds, in units of 2^-23
// relative (u): the product's rounding (2^-24) and (float) log2 e's own
// (0.11 u) shift the exponent by at most 0.61|y| u of relative error, so
// e^y is within 2 + 0.61|y| u; the bounds below use 2 + 1.2|y| u.
//
//   sigmoid(x) = 1 / (1 + e^-x):  e^-x within 2 + 1.2|x| u; the add keeps
//     the relative error of 1 + e (e / (1 + e) <= 1) and adds 0.5 u, the
//     reciprocal 1 u: <= 3.5 + 1.2|x| u, i.e. <= 1.9e-6 for |x| <= 10 and
//     <= 7.6e-6 for |x| <= 50 (sigmoid(-50) = 2e-22).  Beyond x < -87.3 the
//     reciprocal's result would be subnormal and is flushed to 0 (the true
//     value is below 1.2e-38).
//   tanh(x), a = |x|, sign restored at the end (tanh is odd; -0 stays -0):
//     a >= 1/4:  1 - 2 / (1 + e^2a).  v = 2 / (1 + e^2a) carries at most
//       (2 + 2.4a) e^2a / (1 + e^2a) + 1.5 u of relative error; tanh = 1 - v,
//       and v / tanh <= 3.1 at a = 1/4 and falls as e^-2a, so the result is
//       within ~10 u at a = 1/4 (13 u, 1.6e-6, is the bound tested) and
//       within ~1 u from a = 2 on.  e^2a = inf (a > 44) gives exactly 1.
//     a < 1/4:  the Taylor series a - a^3/3 + 2a^5/15 - 17a^7/315 +
//       62a^9/2835, evaluated as a + a^3 q(a^2) (one rounding on top of a);
//       the first omitted term, 1382 a^11 / 155925, is below 2.2e-9 of the
//       value, so the result is within ~1.5 u.
//   NaN propagates through both; tanh(+-inf) = +-1, sigmoid(+inf) = 1,
//   sigmoid(-inf) = 0.
#pragma once

#define J4C_MATH_DEFS                                                                              \
    __device__ __forceinline__ float j_rcp_approx(float d) {                                       \
        float r;                                                                                   \
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));                                      \
        return r;                                                                                  \
    }                                                                                              \
    __device__ __forceinline__ float j_ex2_approx(float y) {                                       \
        float r;                                                                                   \
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));                                      \
        return r;                                                                                  \
    }                                                                                              \
    /* e^-x = 2^(x * -log2 e) */                                                                   \
    __device__ __forceinline__ float j_sigmoid(float x) {                                          \
        return j_rcp_approx(__fadd_rn(1.0f, j_ex2_approx(__fmul_rn(x, -1.44269502162933349609375f)))); \
    }                                                                                              \
    /* e^2a = 2^(a * 2 log2 e); 2 * (float) log2 e is exact, so this is the */                     \
    /* rounded product 2a * (float) log2 e */                                                      \
    __device__ __forceinline__ float j_tanh(float x) {                                             \
        const float a = fabsf(x);                                                                  \
        const float e2a = j_ex2_approx(__fmul_rn(a, 2.8853900432586669921875f));                   \
        const float big = __fmaf_rn(-2.0f, j_rcp_approx(__fadd_rn(1.0f, e2a)), 1.0f);              \
        const float a2 = __fmul_rn(a, a);                                                          \
        float q = __fmaf_rn(a2, 0.021869488536155203f, -0.053968253968253971f);                    \
        q = __fmaf_rn(q, a2, 0.13333333333333333f);                                                \
        q = __fmaf_rn(q, a2, -0.33333333333333333f);                                               \
        const float small = __fmaf_rn(__fmul_rn(a2, a), q, a);                                     \
        return copysignf(a < 0.25f ? small : big, x);                                              \
    }

#define J4C_MATH_STR2(...) #__VA_ARGS__
#define J4C_MATH_STR(x) J4C_MATH_STR2(x)
#define J4C_MATH_SRC J4C_MATH_STR(J4C_MATH_DEFS)
