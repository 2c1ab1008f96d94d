// exp(x) for x <= 0 in IEEE fp64, table-driven.
//
// Method: P. T. P. Tang, "Table-driven implementation of the exponential
// function in IEEE floating-point arithmetic", ACM TOMS 15(2), 1989:
//   x = (32 m + j) ln2/32 + r,  |r| <= ln2/64,
//   exp(x) = 2^m * 2^(j/32) * exp(r),
// with k = 32 m + j = rint(32 x / ln2) taken from the low mantissa bits of
// x * 32/ln2 + 1.5 * 2^52, the reduction r = x - k ln2/32 done in two steps
// with a split ln2/32 (the FMA keeps each product exact), exp(r) - 1 from its
// Taylor series through r^6/720 (truncation < 4e-18 for |r| <= 0.0109), and
// 2^(j/32) from a 32-entry table of correctly rounded doubles.  2^m is built
// from its exponent bits, so no conversion instruction is needed.  Arguments
// below -708 return 0 (the true value is under exp(-708) = 3.31e-308; SOAP
// radial factors there vanish against every other term).
#pragma once

#include <cuda_runtime.h>

namespace mdsoap {

// 2^(j/32), j = 0..31, correctly rounded.
__device__ __constant__ const double kExp2Table[32] = {
    1.0, 1.0218971486541166, 1.0442737824274138, 1.0671404006768237, 1.0905077326652577, 1.1143867425958924,
    1.1387886347566916, 1.1637248587775775, 1.189207115002721, 1.215247359980469, 1.241857812073484,
    1.2690509571917332, 1.2968395546510096, 1.3252366431597413, 1.3542555469368927, 1.383909881963832,
    1.4142135623730951, 1.4451808069770467, 1.4768261459394993, 1.5091644275934228, 1.5422108254079407,
    1.5759808451078865, 1.6104903319492543, 1.645755478153965, 1.681792830507429, 1.718619298122478,
    1.7562521603732995, 1.7947090750031072, 1.8340080864093424, 1.8741676341103, 1.9152065613971474,
    1.9571441241754002};

// `table` is a shared-memory copy of kExp2Table (lanes index it freely).
__device__ __forceinline__ double exp_nonpositive(double x, const double* __restrict__ table) {
    constexpr double kInvLn2Over32 = 46.16624130844683;   // 32 / ln 2
    constexpr double kShift = 6755399441055744.0;         // 1.5 * 2^52
    constexpr double kLn2Over32Hi = 0.02166084939249829;  // ln 2 / 32, leading double
    constexpr double kLn2Over32Lo = 7.247021293269686e-19; // ln 2 / 32 - leading double
    const double t = fma(x, kInvLn2Over32, kShift);
    const int k = __double2loint(t);
    const double kd = t - kShift;
    double r = fma(kd, -kLn2Over32Hi, x);
    r = fma(kd, -kLn2Over32Lo, r);
    // exp(r) - 1 = r (1 + r/2 (1 + r/3 (1 + r/4 (1 + r/5 (1 + r/6)))))
    double p = fma(r, 1.0 / 720.0, 1.0 / 120.0);
    p = fma(r, p, 1.0 / 24.0);
    p = fma(r, p, 1.0 / 6.0);
    p = fma(r, p, 0.5);
    p = fma(r, p, 1.0);
    p = r * p;
    const double tj = table[k & 31];
    const double mant = fma(tj, p, tj);
    const int m = k >> 5;  // arithmetic shift: floor(k / 32)
    const double scale = __hiloint2double((m + 1023) << 20, 0);
    return x < -708.0 ? 0.0 : mant * scale;
}

// pref * exp(x) for x in [-708, 0] when the product is a normal double (the
// plan checks pref exp(x) >= 1e-300 over its whole argument range before it
// picks a kernel that calls this).  Same method as exp_nonpositive, with the
// prefactor folded into the table factor and 2^m applied by adding m to the
// exponent field (exact for normal results), so no clamp and no scaling
// multiply are needed:
//   PRECISE  two-step reduction and the series through r^6/720 (as above);
//   !PRECISE one-step reduction (the dropped k ln2/32 tail is below
//            |k| 7.3e-19 <= 2.4e-14 absolute in r) and the series through
//            r^5/120 (truncation < 2.2e-15): relative error a few 1e-14, for
//            float32 output rows.
template <bool PRECISE>
__device__ __forceinline__ double scaled_exp(double x, double pref, const double* __restrict__ table) {
    constexpr double kInvLn2Over32 = 46.16624130844683;
    constexpr double kShift = 6755399441055744.0;
    constexpr double kLn2Over32Hi = 0.02166084939249829;
    constexpr double kLn2Over32Lo = 7.247021293269686e-19;
    const double t = fma(x, kInvLn2Over32, kShift);
    const int k = __double2loint(t);
    const double kd = t - kShift;
    double r = fma(kd, -kLn2Over32Hi, x);
    double p;
    if constexpr (PRECISE) {
        r = fma(kd, -kLn2Over32Lo, r);
        p = fma(r, 1.0 / 720.0, 1.0 / 120.0);
        p = fma(r, p, 1.0 / 24.0);
    } else {
        p = fma(r, 1.0 / 120.0, 1.0 / 24.0);
    }
    p = fma(r, p, 1.0 / 6.0);
    p = fma(r, p, 0.5);
    p = fma(r, p, 1.0);
    p = r * p;
    const double tj = pref * table[k & 31];
    const double v = fma(tj, p, tj);
    return __hiloint2double(__double2hiint(v) + (k >> 5) * (1 << 20), __double2loint(v));
}

}  // namespace mdsoap
