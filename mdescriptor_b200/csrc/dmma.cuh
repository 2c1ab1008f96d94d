// fp64 tensor-core (DMMA) building blocks shared by the centre kernels:
// coefficient-block layout, mma.sync wrappers, the in-place beta transform and
// the power spectrum (cpp/src/standalone/soap.cpp:915-926, :997-1012).
//
// Coefficient block of one centre: rows r = t n_max + n (species t, radial
// n), fp64; degree l occupies columns [col_off(l), col_off(l) + kpad(l)),
// 2l+1 values in the reference's within-l order, zero padded to a multiple of
// 4 (one mma K step).  The row stride is = 4 (mod 16) doubles, so the
// fragment reads below -- 4 rows x 4 columns per half warp -- hit 16
// distinct 8-byte bank pairs.
#pragma once

#include "common.cuh"

namespace mdsoap {

namespace mma {


__host__ __device__ constexpr int kpad(int l) { return (2 * l + 1 + 3) & ~3; }     // columns of degree l
__host__ __device__ constexpr int blocks8(int l) { return (2 * l + 1 + 7) / 8; }    // 8-row blocks of degree l
__host__ __device__ constexpr int col_off(int l) {                                  // first column of degree l
    int o = 0;
    for (int i = 0; i < l; ++i) o += kpad(i);
    return o;
}
__host__ __device__ constexpr int acc_off(int l) {                                  // first accumulator of degree l
    int o = 0;
    for (int i = 0; i < l; ++i) o += 2 * blocks8(i);
    return o;
}
__host__ __device__ constexpr int stride4(int x) { return x + ((4 - x % 16) + 16) % 16; }  // next >= x, = 4 mod 16

// Coefficient-block row stride (doubles) for l_max = L.
__host__ __device__ constexpr int row_stride(int L) { return stride4(col_off(L + 1)); }
// Harmonic row stride: block l at l*l, fragment reads reach l*l + 8*blocks8(l) - 1.
__host__ __device__ constexpr int y_stride(int L) {
    int need = (L + 1) * (L + 1);
    for (int l = 0; l <= L; ++l) need = need > l * l + 8 * blocks8(l) ? need : l * l + 8 * blocks8(l);
    return stride4(need);
}

// The warp-collective mma.sync is volatile asm: a plain asm statement is a
// pure function of its operands to the compiler, which may then move it into a
// branch taken by only some lanes (a consumer of its result under a
// lane-dependent condition), where the instruction's all-lanes requirement
// fails and the products come out wrong.
__device__ __forceinline__ void dmma8(double& c0, double& c1, double a0, double b0) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
        : "+d"(c0), "+d"(c1)
        : "d"(a0), "d"(b0));
}
__device__ __forceinline__ void dmma16(double& c0, double& c1, double& c2, double& c3, double a0, double a1,
                                       double b0) {
    asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+d"(c0), "+d"(c1), "+d"(c2), "+d"(c3)
        : "d"(a0), "d"(a1), "d"(b0));
}

// In-place beta transform of every species' block (soap.cpp:915-926).
template <int LMAX>
__device__ __forceinline__ void beta_mma(const double* __restrict__ bt, double* __restrict__ reg, int rs, int L,
                                         int S, int n, int g, int q) {
    static_for<0, LMAX + 1>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        if (l <= L) {
            const double a0 = bt[(l * 8 + g) * 8 + q];
            const double a1 = bt[(l * 8 + g) * 8 + 4 + q];
            for (int s = 0; s < S; ++s) {
                double* blk = reg + s * n * rs + col_off(l);
#pragma unroll
                for (int mb = 0; mb < (kpad(l) + 7) / 8; ++mb) {
                    const int m = 8 * mb + g;
                    const bool mok = m < kpad(l);
                    const double b0 = (mok && q < n) ? blk[q * rs + m] : 0.0;
                    const double b1 = (mok && q + 4 < n) ? blk[(q + 4) * rs + m] : 0.0;
                    double c0 = 0.0, c1 = 0.0;
                    dmma8(c0, c1, a0, b0);
                    dmma8(c0, c1, a1, b1);
                    __syncwarp();
                    const int mo = 8 * mb + 2 * q;
                    if (g < n) {
                        if (mo < kpad(l)) blk[g * rs + mo] = c0;
                        if (mo + 1 < kpad(l)) blk[g * rs + mo + 1] = c1;
                    }
                    __syncwarp();
                }
            }
        }
    });
}

// Output placement of the power spectrum (compression off: t1 <= t2, then
// l, then n1, then n2 with n2 >= n1 when t1 == t2), soap.cpp:997-1012.
struct FeatureMap {
    int S, n, L, R;
    unsigned n_magic;  // floor(2^32 / n) + 1 (0 for n = 1): r / n == umulhi(r, n_magic) for r < 2^16, n <= 32
    __device__ __forceinline__ int div_n(int r) const {
        return n_magic ? (int)__umulhi((unsigned)r, n_magic) : r;
    }
    // Offset of (r1, r2, l = 0) and the l stride, r1 <= r2.
    __device__ __forceinline__ int64_t base(int r1, int r2, int& bs) const {
        const int t1 = div_n(r1), n1 = r1 - t1 * n;
        const int t2 = div_n(r2), n2 = r2 - t2 * n;
        bs = t1 == t2 ? n * (n + 1) / 2 : n * n;
        return pair_base(S, n, L, t1, t2) +
               (t1 == t2 ? (int64_t)n1 * n - (int64_t)n1 * (n1 - 1) / 2 + (n2 - n1) : (int64_t)n1 * n + n2);
    }
};

__device__ __forceinline__ void store_pair(float* p, double a, double b) {
    *reinterpret_cast<float2*>(p) = make_float2((float)a, (float)b);
}
__device__ __forceinline__ void store_pair(double* p, double a, double b) {
    *reinterpret_cast<double2*>(p) = make_double2(a, b);
}

// Power spectrum of one centre from its coefficient block: P_l = C_l C_l^T
// over the rows, in 16 x 8 tiles on or above the diagonal.  Lane (g, q) holds
// rows r1 = 16i + g (+8) and columns r2 = 8j + 2q (+1); with n_max even the
// two columns are consecutive features of one pair block, written as one
// 8-byte (float) or 16-byte (double) store when aligned.  `out` is the
// centre's feature row; `pref` the factors pi sqrt(8 / (2l + 1)).
template <int LMAX, class OutT>
__device__ __forceinline__ void power_mma(const FeatureMap& fm, const double* __restrict__ pref,
                                          const double* __restrict__ reg, int rs, OutT* __restrict__ out, int g,
                                          int q) {
    const int L = fm.L, R = fm.R;
    const int RB = (R + 15) / 16, CB = (R + 7) / 8;
    const bool even = (fm.n & 1) == 0;
    const bool row_aligned = (reinterpret_cast<uintptr_t>(out) % (2 * sizeof(OutT))) == 0;
    for (int i = 0; i < RB; ++i) {
        for (int j = 2 * i; j < CB; ++j) {
            const int r2a = 8 * j + 2 * q, r2b = r2a + 1;
            const int rb = 8 * j + g;
            const double* rc = reg + rb * rs + q;
            const bool okc = rb < R;
            int64_t f[2][2];
            int s[2][2];
            bool v[2][2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r1 = 16 * i + g + 8 * h;
                v[h][0] = r1 <= r2a && r2a < R;
                v[h][1] = r1 <= r2b && r2b < R;
                f[h][0] = f[h][1] = 0;
                s[h][0] = s[h][1] = 0;
                if (even) {
                    // r2a even, so r2a and r2b share species; when both are
                    // stored the second feature follows the first.
                    if (v[h][0]) {
                        f[h][0] = fm.base(r1, r2a, s[h][0]);
                        f[h][1] = f[h][0] + 1;
                        s[h][1] = s[h][0];
                    } else if (v[h][1]) {
                        f[h][1] = fm.base(r1, r2b, s[h][1]);
                    }
                } else {
                    if (v[h][0]) f[h][0] = fm.base(r1, r2a, s[h][0]);
                    if (v[h][1]) f[h][1] = fm.base(r1, r2b, s[h][1]);
                }
            }
            const int r1a = 16 * i + g, r1b = r1a + 8;
            const double* ra = reg + r1a * rs + q;
            const double* rbp = reg + r1b * rs + q;
            const bool oka = r1a < R, okb = r1b < R;
            double c[LMAX + 1][4];
            static_for<0, LMAX + 1>([&](auto lc) {
                constexpr int l = decltype(lc)::value;
                c[l][0] = c[l][1] = c[l][2] = c[l][3] = 0.0;
                if (l <= L) {
#pragma unroll
                    for (int kb = 0; kb < kpad(l); kb += 4) {
                        const int o = col_off(l) + kb;
                        const double a0 = oka ? ra[o] : 0.0;
                        const double a1 = okb ? rbp[o] : 0.0;
                        const double b0 = okc ? rc[o] : 0.0;
                        dmma16(c[l][0], c[l][1], c[l][2], c[l][3], a0, a1, b0);
                    }
                }
            });
#pragma unroll
            for (int l = 0; l <= LMAX; ++l) {
                if (l <= L) {
                    const double p = pref[l];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const double x = p * c[l][2 * h], y = p * c[l][2 * h + 1];
                        const int64_t fa = f[h][0] + (int64_t)l * s[h][0];
                        const int64_t fb = f[h][1] + (int64_t)l * s[h][1];
                        if (even && row_aligned && v[h][0] && (fa & 1) == 0) {
                            store_pair(out + fa, x, y);
                        } else {
                            if (v[h][0]) out[fa] = (OutT)x;
                            if (v[h][1]) out[fb] = (OutT)y;
                        }
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// n_max == 8 tail: one species is exactly one 8-row block of the coefficient
// block, so every product tile is one species pair.

// In-place beta transform, two species per batch: all loads of a batch, then
// its tensor-core products, then its stores (soap.cpp:915-926).
template <int L>
__device__ __forceinline__ void beta_n8(const double* __restrict__ bt, double* __restrict__ reg, int rs, int S, int g,
                                        int q) {
    static_for<0, L + 1>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        constexpr int KP = kpad(l), MB = (KP + 7) / 8, C0 = col_off(l);
        const double a0 = bt[(l * 8 + g) * 8 + q];
        const double a1 = bt[(l * 8 + g) * 8 + 4 + q];
        for (int s = 0; s < S; s += 2) {
            double b[2][MB][2], c[2][MB][2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const double* blk = reg + (s + u) * 8 * rs + C0;
#pragma unroll
                for (int mb = 0; mb < MB; ++mb) {
                    const int m = 8 * mb + g;
                    const bool ok = s + u < S && m < KP;
                    b[u][mb][0] = ok ? blk[q * rs + m] : 0.0;
                    b[u][mb][1] = ok ? blk[(q + 4) * rs + m] : 0.0;
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int mb = 0; mb < MB; ++mb) {
                    c[u][mb][0] = c[u][mb][1] = 0.0;
                    dmma8(c[u][mb][0], c[u][mb][1], a0, b[u][mb][0]);
                    dmma8(c[u][mb][0], c[u][mb][1], a1, b[u][mb][1]);
                }
            __syncwarp();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                double* blk = reg + (s + u) * 8 * rs + C0;
#pragma unroll
                for (int mb = 0; mb < MB; ++mb) {
                    const int mo = 8 * mb + 2 * q;
                    if (s + u < S) {
                        if (mo < KP) blk[g * rs + mo] = c[u][mb][0];
                        if (mo + 1 < KP) blk[g * rs + mo + 1] = c[u][mb][1];
                    }
                }
            }
            __syncwarp();
        }
    });
}

// Power spectrum with n_max == 8 (compression off, soap.cpp:997-1012): for
// each species pair t1 <= t2 in feature order and each l, the 8 x 8 product
// C_{t1,l} C_{t2,l}^T on the tensor cores.  Lane (g, q) holds rows n1 = g,
// columns n2 = 2q, 2q+1: in an off-diagonal block those are features
// base + 8 g + 2q (+1), so a warp stores 64 consecutive features per l; in a
// diagonal block (n2 >= n1 kept) the offset is g*8 - g(g-1)/2 + (n2 - g).
// Feature offsets fit in 32 bits (F < 2^31 for any plan).
template <int L, class OutT>
__device__ __forceinline__ void power_n8(const double* __restrict__ pref, const double* __restrict__ reg, int rs,
                                         int S, OutT* __restrict__ out, int g, int q) {
    const int od = 8 * g + 2 * q;
    const int n2a = 2 * q, n2b = 2 * q + 1;
    const bool va = n2a >= g, vb = n2b >= g;
    const int dd = 8 * g - g * (g - 1) / 2 - g;  // diagonal offset of (g, n2) is dd + n2
    const bool row_aligned = (reinterpret_cast<uintptr_t>(out) % (2 * sizeof(OutT))) == 0;
    int base = 0;
    for (int t1 = 0; t1 < S; ++t1) {
        const double* A = reg + (t1 * 8 + g) * rs + q;
        for (int t2 = t1; t2 < S; ++t2) {
            const double* B = reg + (t2 * 8 + g) * rs + q;
            double c[L + 1][2];
            static_for<0, L + 1>([&](auto lc) {
                constexpr int l = decltype(lc)::value;
                c[l][0] = c[l][1] = 0.0;
#pragma unroll
                for (int kb = 0; kb < kpad(l); kb += 4) dmma8(c[l][0], c[l][1], A[col_off(l) + kb], B[col_off(l) + kb]);
            });
            if (t1 != t2) {
#pragma unroll
                for (int l = 0; l <= L; ++l) {
                    OutT* dst = out + base + 64 * l + od;
                    const double x = pref[l] * c[l][0], y = pref[l] * c[l][1];
                    if (row_aligned) {
                        store_pair(dst, x, y);
                    } else {
                        dst[0] = (OutT)x;
                        dst[1] = (OutT)y;
                    }
                }
                base += 64 * (L + 1);
            } else {
#pragma unroll
                for (int l = 0; l <= L; ++l) {
                    OutT* dst = out + base + 36 * l + dd;
                    const double x = pref[l] * c[l][0], y = pref[l] * c[l][1];
                    if (va && row_aligned && ((base + 36 * l + dd + n2a) & 1) == 0) {
                        store_pair(dst + n2a, x, y);
                    } else {
                        if (va) dst[n2a] = (OutT)x;
                        if (vb) dst[n2b] = (OutT)y;
                    }
                }
                base += 36 * (L + 1);
            }
        }
    }
}

// Beta transform and power spectrum with the coefficients held in registers
// (n_max == 8, at most MAXS species, compression off; soap.cpp:915-926 and
// :997-1012).  Per degree l:
//   1. C_t = beta_l R_t for every species t on the tensor cores: A = beta_l
//      (n x k, pi^{3/2} folded in), B = the raw sums of the coefficient block
//      (k x m, 8 columns per tile).  The accumulator tile (lane (g, q) holds
//      C[g][8mb + 2q] and C[g][8mb + 2q + 1]) is moved into the operand layout
//      of the power products (lane (g, q) holds C[g][4kb + q]) by shuffles,
//      and columns m >= 2l + 1 -- the block's padding, never cleared -- are
//      set to 0 there, so the padding may hold anything.
//   2. P = pi sqrt(8 / (2l + 1)) C_t1 C_t2^T for every pair t1 <= t2, each
//      lane storing its two features (see power_n8 for the offsets); with
//      compression crossover only t1 == t2 (species t's block at
//      t (L+1) n(n+1)/2), with mu1nu1 C_t (sum_t' C_t')^T in full n x n
//      blocks (species t's block at t (L+1) n^2).  mu2 arrives as one pooled
//      species in the compression-off layout.
// The coefficients of one degree are loaded once and shared by all pairs,
// and every pair's product chain is independent of the others.
// Degrees [l_lo, l_hi] are done, plus l_extra when it is >= 0 (several warps
// can then share one centre's block, each with its own degrees).
template <int L, int MAXS, class OutT>
__device__ __forceinline__ void tail_regs_n8(const double* __restrict__ bt, const double* __restrict__ reg, int rs,
                                             int S, int compression, const double* __restrict__ pref,
                                             OutT* __restrict__ out, int lane, int l_lo = 0, int l_hi = L,
                                             int l_extra = -1) {
    const int g = lane >> 2, q = lane & 3;
    const int od = 8 * g + 2 * q;
    const int n2a = 2 * q, n2b = 2 * q + 1;
    const bool va = n2a >= g, vb = n2b >= g;
    const int dd = 8 * g - g * (g - 1) / 2 - g;  // diagonal block: offset of (g, n2) is dd + n2
    const bool row_aligned = (reinterpret_cast<uintptr_t>(out) % (2 * sizeof(OutT))) == 0;
    const int src_lo = (lane & ~3) | (q >> 1), src_hi = src_lo + 2;
    const bool odd = (q & 1) != 0;
    constexpr int NKMAX = kpad(L) / 4;          // k steps of the largest degree
    constexpr int MBMAX = (kpad(L) + 7) / 8;    // 8-column tiles of the largest degree
    int pb[MAXS][MAXS];
#pragma unroll
    for (int t1 = 0; t1 < MAXS; ++t1)
#pragma unroll
        for (int t2 = t1; t2 < MAXS; ++t2) pb[t1][t2] = (int)pair_base(S, 8, L, t1, t2);
    // A runtime loop over l (one copy of the code); trip counts inside are
    // warp-uniform, the register arrays sized for the largest degree.
#pragma unroll 1
    for (int li = l_lo; li <= l_hi + (l_extra >= 0 ? 1 : 0); ++li) {
        const int l = li <= l_hi ? li : l_extra;
        const int KP = (2 * l + 1 + 3) & ~3, NK = KP / 4, MB = (KP + 7) / 8;
        int C0 = 0;
        for (int i = 0; i < l; ++i) C0 += (2 * i + 1 + 3) & ~3;
        const double a0 = bt[(l * 8 + g) * 8 + q];
        const double a1 = bt[(l * 8 + g) * 8 + 4 + q];
        double f[MAXS][NKMAX];
#pragma unroll
        for (int t = 0; t < MAXS; ++t) {
#pragma unroll
            for (int kb = 0; kb < NKMAX; ++kb) f[t][kb] = 0.0;
            if (t < S) {
                const double* blk = reg + t * 8 * rs + C0;
#pragma unroll
                for (int mb = 0; mb < MBMAX; ++mb) {
                    if (mb < MB) {
                        const int m = 8 * mb + g;
                        const double b0 = blk[q * rs + m], b1 = blk[(q + 4) * rs + m];
                        double c0 = 0.0, c1 = 0.0;
                        dmma8(c0, c1, a0, b0);
                        dmma8(c0, c1, a1, b1);
                        const double x0 = __shfl_sync(0xffffffffu, c0, src_lo);
                        const double x1 = __shfl_sync(0xffffffffu, c1, src_lo);
                        const double y0 = __shfl_sync(0xffffffffu, c0, src_hi);
                        const double y1 = __shfl_sync(0xffffffffu, c1, src_hi);
                        if (2 * mb < NKMAX) f[t][2 * mb] = (8 * mb + q < 2 * l + 1) ? (odd ? x1 : x0) : 0.0;
                        if (2 * mb + 1 < NKMAX)
                            f[t][2 * mb + 1] = (8 * mb + 4 + q < 2 * l + 1) ? (odd ? y1 : y0) : 0.0;
                    }
                }
            }
        }
        const double pl = pref[l];
        if (compression == 2) {
            double fs[NKMAX];
#pragma unroll
            for (int kb = 0; kb < NKMAX; ++kb) {
                fs[kb] = 0.0;
#pragma unroll
                for (int t = 0; t < MAXS; ++t) fs[kb] += f[t][kb];
            }
#pragma unroll
            for (int t = 0; t < MAXS; ++t) {
                if (t < S) {
                    double c0 = 0.0, c1 = 0.0;
#pragma unroll
                    for (int kb = 0; kb < NKMAX; ++kb)
                        if (kb < NK) dmma8(c0, c1, f[t][kb], fs[kb]);
                    OutT* dst = out + t * 64 * (L + 1) + 64 * l + od;
                    if (row_aligned) {
                        store_pair(dst, pl * c0, pl * c1);
                    } else {
                        dst[0] = (OutT)(pl * c0);
                        dst[1] = (OutT)(pl * c1);
                    }
                }
            }
            continue;
        }
#pragma unroll
        for (int t1 = 0; t1 < MAXS; ++t1) {
#pragma unroll
            for (int t2 = t1; t2 < MAXS; ++t2) {
                if (t2 < S && (compression != 3 || t1 == t2)) {
                    double c0 = 0.0, c1 = 0.0;
#pragma unroll
                    for (int kb = 0; kb < NKMAX; ++kb)
                        if (kb < NK) dmma8(c0, c1, f[t1][kb], f[t2][kb]);
                    const double x = pl * c0, y = pl * c1;
                    if (t1 != t2) {
                        OutT* dst = out + pb[t1][t2] + 64 * l + od;
                        if (row_aligned) {
                            store_pair(dst, x, y);
                        } else {
                            dst[0] = (OutT)x;
                            dst[1] = (OutT)y;
                        }
                    } else {
                        const int o = (compression == 3 ? t1 * 36 * (L + 1) : pb[t1][t2]) + 36 * l + dd;
                        OutT* dst = out + o;
                        if (va && row_aligned && ((o + n2a) & 1) == 0) {
                            store_pair(dst + n2a, x, y);
                        } else {
                            if (va) dst[n2a] = (OutT)x;
                            if (vb) dst[n2b] = (OutT)y;
                        }
                    }
                }
            }
        }
    }
}

}  // namespace mma

}  // namespace mdsoap
