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

// 2^(j/64), j = 0..63, correctly rounded (the even entries are kExp2Table's).
__device__ __constant__ const double kExp2Table64[64] = {
    1.0, 1.0108892860517005, 1.0218971486541166, 1.0330248790212284, 1.0442737824274138,
    1.0556451783605572, 1.0671404006768237, 1.0787607977571199, 1.0905077326652577, 1.102382583307841,
    1.1143867425958924, 1.1265216186082418, 1.1387886347566916, 1.1511892299529827, 1.1637248587775775,
    1.1763969916502812, 1.189207115002721, 1.202156731452703, 1.215247359980469, 1.22848053610687,
    1.241857812073484, 1.255380757024691, 1.2690509571917332, 1.2828700160787783, 1.2968395546510096,
    1.3109612115247644, 1.3252366431597413, 1.339667524053303, 1.3542555469368927, 1.3690024229745905,
    1.383909881963832, 1.3989796725383112, 1.4142135623730951, 1.42961333839197, 1.4451808069770467,
    1.460917794180647, 1.4768261459394993, 1.4929077282912648, 1.5091644275934228, 1.5255981507445384,
    1.5422108254079407, 1.559004400237837, 1.5759808451078865, 1.593142151342267, 1.6104903319492543,
    1.6280274218573478, 1.645755478153965, 1.6636765803267364, 1.681792830507429, 1.7001063537185235,
    1.718619298122478, 1.7373338352737062, 1.7562521603732995, 1.7753764925265212, 1.7947090750031072,
    1.8142521755003989, 1.8340080864093424, 1.8539791250833855, 1.8741676341103, 1.8945759815869656,
    1.9152065613971474, 1.9360617934922943, 1.9571441241754002, 1.978456026387951};

// pref * exp(-E u) for float32 rows in the expansion-only kernel, with the
// channel's exponent folded into the reduction: s = -E * T / ln 2 (per lane,
// once), so u s = (T m + j) + r' directly, r' = fma(u, s, -(T m + j)) in
// units of ln2 / T (|r'| <= 1/2), and exp(r' ln2 / T) - 1 by its Taylor series
// in r' (coefficients (ln2/T)^i / i!).  T = 64: `table` is kExp2Table64 and the
// series runs through i = 4 (truncation < 4e-14); T = 32: kExp2Table and i = 5
// (< 3e-15).  The rounding of s (relative 1.1e-16) moves r' by at most
// |u s| 1.1e-16 <= 3.5e-12 (|E u| <= 700), i.e. the result by a relative
// 7.6e-14 at the far end of the range, where the factor is below e^-300 of
// the near edges': float32 rows do not see it.  Same plan-side range check as
// scaled_exp (pref exp(-E u) a normal double).
template <int T>
__device__ __forceinline__ double scaled_exp_folded(double u, double s, double pref, const double* __restrict__ table) {
    static_assert(T == 32 || T == 64, "table of 32 or 64 entries");
    constexpr double kShift = 6755399441055744.0;  // 1.5 * 2^52
    const double t = fma(u, s, kShift);
    const int k = __double2loint(t);
    const double kd = t - kShift;
    const double r = fma(u, s, -kd);
    double q;
    if constexpr (T == 64) {
        q = fma(r, 5.732851688640402e-10, 2.1173137155464776e-07);
        q = fma(r, q, 5.86490495505617e-05);
        q = fma(r, q, 0.010830424696249145);
    } else {
        q = fma(r, 3.973709984549416e-11, 9.172562701824643e-09);
        q = fma(r, q, 1.693850972437182e-06);
        q = fma(r, q, 0.0002345961982022468);
        q = fma(r, q, 0.02166084939249829);
    }
    const double p = r * q;
    const double tj = pref * table[k & (T - 1)];
    const double v = fma(tj, p, tj);
    constexpr int kShiftBits = T == 64 ? 6 : 5;
    return __hiloint2double(__double2hiint(v) + (k >> kShiftBits) * (1 << 20), __double2loint(v));
}

// T / ln 2 for scaled_exp_folded's s.
__host__ __device__ constexpr double folded_scale(int T) { return T == 64 ? 92.33248261689366 : 46.16624130844683; }

}  // namespace mdsoap
