// SOAP expansion + power spectrum, fused per centre (sm_100a, IEEE fp64).
//
// Reference arithmetic (cpp/src/standalone/soap.cpp):
//   g_{lk}(r)   = P_{lk} exp(-E_{lk} r^2)                      prepare_soap :507-572
//   Y_{lm}(d)   = real regular solid harmonics (r^l included)   solid_harmonics :101-216
//   S[t][l][k][m] = sum_{j in species t} g_{lk}(r_j) Y_{lm}(d_j) w_t       :881-914
//   c[t][n][lm] = pi^{3/2} sum_k beta[l][n][k] S[t][l][k][m]                :915-926
//   p(t1,t2,l,n1,n2) = pi sqrt(8/(2l+1)) sum_m c[t1][n1][lm] c[t2][n2][lm]  :997-1012
//
// Work decomposition (one warp per centre):
//   * the centre's bin neighbourhood is flattened into one candidate list
//     (32 (row, x-image) entries per round, prefix-summed across the warp), so
//     every candidate chunk fills all 32 lanes; candidates are accepted with
//     the reference's exact geometry and appended (ballot + popc) to a
//     per-warp edge queue in shared memory;
//   * per chunk of up to 32 queued edges, lane e evaluates Y_{lm} of edge e by
//     the Cartesian recurrence into a shared-memory row;
//   * every lane owns up to three radial channels (l, k) (channels sorted by
//     l descending, 32 per slot), evaluates its own table-driven exp() per
//     edge and keeps S[t][l][k][0..2l] in registers, reading Y rows as
//     shared-memory broadcasts; species live in register banks picked by a
//     warp-uniform branch (species beyond the banks take another pass);
//   * raw sums go to a shared coefficient block (rows padded to even length
//     so that the power spectrum reads them with 16-byte broadcasts), beta is
//     applied in place, and the power spectrum is written straight to the
//     output row: lane = column r2, broadcast row r1, so each warp store
//     covers runs of consecutive features.
#pragma once

#include "dmma.cuh"
#include "expneg.cuh"
#include "neighbors.cuh"

namespace mdsoap {

struct RadialItem {
    double prefactor;  // eta^l (alpha + eta)^(-l-3/2)
    double exponent;   // alpha eta / (alpha + eta)
    int32_t l;
    int32_t k;
};

// Plan constants passed by value (constant bank; uniform reads broadcast).
struct SoapTables {
    int32_t n_species, n_max, l_max, H;
    int32_t items;        // n_max * (l_max + 1) radial channels
    int32_t rows;         // n_species * n_max
    int64_t features;
    int32_t chunk;        // edges per harmonic chunk (<= 32)
    int32_t average;      // 0 off, 1 inner, 2 outer
    int32_t out_f64;      // output element: 1 double, 0 float
    int32_t beta_in_smem;
    int32_t warp_bytes;   // shared memory per warp
    int32_t r_offset;     // byte offset of the coefficient block inside a warp's region
    int32_t type_groups;  // passes over species groups
    int32_t slot_groups;  // passes over channel-slot groups
    int32_t r_global;     // 1: coefficient blocks live in global scratch
    int32_t csize;        // coefficient block length in doubles: S n (L+1)(L+2)
    int32_t hp;           // padded harmonic row length: (L+1)(L+2)
    int32_t rs;           // tensor-core tail: coefficient-block row stride (0: scalar tail)
    int32_t rsize;        // doubles of one centre's coefficient block
    uint32_t n_magic;     // floor(2^32 / n_max) + 1
    int32_t compression;  // 0 off, 1 mu2, 2 mu1nu1, 3 crossover (paired kernel only when not 0)
    int32_t coef_species; // species of the coefficient block: n_species, or 1 for mu2
    int32_t weighted;     // 1: per-edge weights (weighting function, w0, or mu2 pooling); paired kernel only
    int32_t split_tail;   // the paired kernel stops after the flush; 1: soap_tail_kernel, 2: soap_tail_generic_kernel finishes the centres
    int32_t grid_size;    // polynomial basis: quadrature nodes (0 for the GTO basis)
    int32_t ksplit;       // paired kernel: partial sums per species neighbour sum (2 in its float64 instantiations)
    int32_t edge_cap;     // edge-list split of the SPLIT path: accepted edges per centre slot (0: not used)
    int32_t parity_group; // expansion-only kernel: species per pass of the fused kernel, whose accepted-edge
                          // order sets the partial sum (of ksplit) each edge goes to
    double eta;           // 1 / (2 sigma^2)
    int32_t weight_fn;    // 0 none, 1 polynomial, 2 power, 3 exponential (soap.cpp:389-420)
    int32_t has_w0;       // the exact self pair takes weight w0
    double w_r0, w_c, w_d, w_m, w_0;
    double cutoff2;
    double soap_scale;    // pi^{3/2}
    double ynorm[kTri];   // N_lm (times sqrt 2 for m > 0), index l(l+1)/2 + m
    double yra[kTri];     // (2l-1)/(l-m)
    double yrb[kTri];     // (l+m-1)/(l-m)
    double power_pref[kMaxL + 1];
    double species_weight[kMaxSpecies];
};

struct SoapPointers {
    const double* positions;
    BinView bins;
    const RadialItem* items;  // channels sorted by l descending
    const double* betas;      // [(l_max+1)][n_max][n_max]
    void* out;                // average off: feature rows of centres
    double* cbuf;             // average inner: per-centre coefficient blocks (block-local rows)
    double* pbuf;             // average outer: per-centre power spectra (block-local rows)
    double* rbuf;             // r_global: per-centre coefficient scratch (block-local rows)
    int64_t out_row_begin;    // average off: output row of centre c is c - out_row_begin
    int64_t center_begin;     // first centre of the block (rows of cbuf / pbuf are relative to it)
    int64_t center_end;
    int64_t grid_begin;       // paired / tail kernels: centres [grid_begin, grid_end) of this launch,
    int64_t grid_end;         // rbuf rows relative to grid_begin
    const double* poly;       // polynomial basis: nodes [Q], then weighted values wv [Q][n_max]
    // Edge-list split (tab.edge_cap > 0): slot c = centre grid_begin + c.
    double4* edges;           // [slots][edge_cap] accepted edges (dx, dy, dz, r^2) in walk order
    int32_t* edge_info;       // [slots][edge_cap] species | exact-self flag << 16
    int32_t* edge_count;      // [slots] accepted edges (above edge_cap: slot overflowed)
};

// Radial weight of one edge (soap_weight, cpp/src/standalone/soap.cpp:389-420,
// without its species factor, which the kernels apply per species): the
// weighting function of the distance, replaced by w0 for the exact self pair.
__device__ __forceinline__ double soap_edge_weight(const SoapTables& tab, double d2, bool exact_self) {
    double value = 1.0;
    if (tab.weight_fn != 0) {
        const double distance = sqrt(d2);
        const double ratio = distance / tab.w_r0;
        if (tab.weight_fn == 1) {
            value = distance > tab.w_r0 ? 0.0
                                        : tab.w_c * pow(__dsub_rn(__dadd_rn(1.0, __dmul_rn(__dmul_rn(__dmul_rn(2.0, ratio), ratio), ratio)),
                                                                  __dmul_rn(__dmul_rn(3.0, ratio), ratio)),
                                                        tab.w_m);
        } else if (tab.weight_fn == 2) {
            value = tab.w_c / (tab.w_d + pow(ratio, tab.w_m));
        } else {
            value = tab.w_c / (tab.w_d + exp(-ratio));
        }
    }
    if (exact_self && tab.has_w0) value = tab.w_0;
    return value;
}

// Real regular solid harmonics of one displacement into a padded row: the
// block of degree l starts at l (l + 1) (even, so 16-byte aligned) and holds
// j = l - m (cos part), j = l (m = 0), j = l + m (sin part) at offset j, the
// reference's within-l order (soap.cpp:101-216 generic Cartesian recurrence,
// all l); offset 2l+1 is padding.
__device__ __forceinline__ void solid_harmonics(const SoapTables& tab, double x, double y, double z, double r2,
                                                double* __restrict__ out) {
    const int L = tab.l_max;
    double dr = 1.0, di = 0.0;  // diagonal P_mm (real, imaginary)
    for (int m = 0; m <= L; ++m) {
        if (m > 0) {
            const double f = -(2.0 * m - 1.0);
            const double nr = f * fma(x, dr, -__dmul_rn(y, di));
            const double ni = f * fma(x, di, __dmul_rn(y, dr));
            dr = nr;
            di = ni;
        }
        double pr2 = dr, pi2 = di;
        {
            const double nrm = tab.ynorm[tri(m, m)];
            if (m == 0) {
                out[0] = nrm * pr2;
            } else {
                out[m * (m + 1)] = nrm * pr2;
                out[m * (m + 1) + 2 * m] = nrm * pi2;
            }
        }
        if (m < L) {
            const double c = (2.0 * m + 1.0) * z;
            double pr1 = c * dr, pi1 = c * di;
            {
                const int l = m + 1;
                const double nrm = tab.ynorm[tri(l, m)];
                out[l * (l + 1) + l - m] = nrm * pr1;
                if (m > 0) out[l * (l + 1) + l + m] = nrm * pi1;
            }
            for (int l = m + 2; l <= L; ++l) {
                const double a = tab.yra[tri(l, m)] * z;
                const double b = tab.yrb[tri(l, m)] * r2;
                const double nr = fma(a, pr1, -b * pr2);
                const double ni = fma(a, pi1, -b * pi2);
                pr2 = pr1;
                pi2 = pi1;
                pr1 = nr;
                pi1 = ni;
                const double nrm = tab.ynorm[tri(l, m)];
                out[l * (l + 1) + l - m] = nrm * nr;
                if (m > 0) out[l * (l + 1) + l + m] = nrm * ni;
            }
        }
    }
}

// Same recurrence with a compile-time l_max: every index and coefficient
// offset is a constant, so the constant-bank coefficients feed the FP64
// instructions directly.
template <int L>
__device__ __forceinline__ void solid_harmonics_fixed(const SoapTables& tab, double x, double y, double z, double r2,
                                                      double* __restrict__ out) {
    double dr = 1.0, di = 0.0;
#pragma unroll
    for (int m = 0; m <= L; ++m) {
        if (m > 0) {
            const double f = -(2.0 * m - 1.0);
            const double nr = f * fma(x, dr, -__dmul_rn(y, di));
            const double ni = f * fma(x, di, __dmul_rn(y, dr));
            dr = nr;
            di = ni;
        }
        double pr2 = dr, pi2 = di;
        if (m == 0) {
            out[0] = tab.ynorm[0] * pr2;
        } else {
            out[m * (m + 1)] = tab.ynorm[m * (m + 1) / 2 + m] * pr2;
            out[m * (m + 1) + 2 * m] = tab.ynorm[m * (m + 1) / 2 + m] * pi2;
        }
        if (m < L) {
            const double c = (2.0 * m + 1.0) * z;
            double pr1 = c * dr, pi1 = c * di;
            {
                const int l = m + 1;
                out[l * (l + 1) + l - m] = tab.ynorm[l * (l + 1) / 2 + m] * pr1;
                if (m > 0) out[l * (l + 1) + l + m] = tab.ynorm[l * (l + 1) / 2 + m] * pi1;
            }
#pragma unroll
            for (int l = m + 2; l <= L; ++l) {
                const int i = l * (l + 1) / 2 + m;
                const double a = tab.yra[i] * z;
                const double b = tab.yrb[i] * r2;
                const double nr = fma(a, pr1, -b * pr2);
                const double ni = fma(a, pi1, -b * pi2);
                pr2 = pr1;
                pi2 = pi1;
                pr1 = nr;
                pi1 = ni;
                out[l * (l + 1) + l - m] = tab.ynorm[i] * nr;
                if (m > 0) out[l * (l + 1) + l + m] = tab.ynorm[i] * ni;
            }
        }
    }
}

template <int LMAX>
__device__ __forceinline__ void harmonics_any(const SoapTables& tab, double x, double y, double z, double r2,
                                              double* __restrict__ out) {
    if (tab.l_max == LMAX)
        solid_harmonics_fixed<LMAX>(tab, x, y, z, r2, out);
    else
        solid_harmonics(tab, x, y, z, r2, out);
}

// Power spectrum for l in [LA, LB]: lane = column r2, whose rows of every l
// in the group sit in registers; the loop over rows r1 <= r2 reads each row
// r1 once per l as 16-byte shared-memory broadcasts, and one feature index
// per (r1, r2) serves all l of the group.
template <int LA, int LB, class OutT>
__device__ __forceinline__ void power_group(const SoapTables& tab, const double* __restrict__ c,
                                            OutT* __restrict__ out, int lane, int r1_first, int r1_step) {
    constexpr int NOWN = (LB + 1) * (LB + 1) - LA * LA;
    constexpr int NL = LB - LA + 1;
    const int S = tab.coef_species, n = tab.n_max, L = tab.l_max, R = tab.rows;
    if (LA > L) return;
    const int64_t T = (int64_t)n * (n + 1) / 2, nn = (int64_t)n * n;
    const int sn = S * n;
    for (int r2base = 0; r2base < R; r2base += 32) {
        const int r2 = r2base + lane;
        const bool active = r2 < R;
        const int t2 = active ? r2 / n : 0;
        const int n2 = active ? r2 - t2 * n : 0;
        double own[NOWN];
#pragma unroll
        for (int l = LA; l <= LB; ++l) {
            const double* cl = c + sn * l * (l + 1) + r2 * (2 * l + 2);
#pragma unroll
            for (int m = 0; m < 2 * l + 1; ++m) own[l * l - LA * LA + m] = (active && l <= L) ? cl[m] : 0.0;
        }
        const int r1_end = min(R - 1, r2base + 31);
        int t1 = r1_first / n, n1 = r1_first - (r1_first / n) * n;
        int64_t base = pair_base(S, n, L, t1, t2);
        int64_t bs = t1 == t2 ? T : nn;
        for (int r1 = r1_first; r1 <= r1_end; r1 += r1_step) {
            double v[NL];
#pragma unroll
            for (int l = LA; l <= LB; ++l) {
                double acc = 0.0;
                if (l <= L) {
                    const double2* o = reinterpret_cast<const double2*>(c + sn * l * (l + 1) + r1 * (2 * l + 2));
#pragma unroll
                    for (int m = 0; m < 2 * l + 1; m += 2) {
                        const double2 q = o[m / 2];
                        acc = fma(q.x, own[l * l - LA * LA + m], acc);
                        if (m + 1 < 2 * l + 1) acc = fma(q.y, own[l * l - LA * LA + m + 1], acc);
                    }
                }
                v[l - LA] = acc;
            }
            if (active && r2 >= r1) {
                const int64_t inner = t1 == t2 ? (int64_t)n1 * n - (int64_t)n1 * (n1 - 1) / 2 + (n2 - n1)
                                               : (int64_t)n1 * n + n2;
                OutT* dst = out + base + inner;
#pragma unroll
                for (int l = LA; l <= LB; ++l)
                    if (l <= L) dst[l * bs] = (OutT)(tab.power_pref[l] * v[l - LA]);
            }
            n1 += r1_step;
            if (n1 >= n) {
                while (n1 >= n) {
                    n1 -= n;
                    ++t1;
                }
                if (t1 <= t2) {
                    base = pair_base(S, n, L, t1, t2);
                    bs = t1 == t2 ? T : nn;
                }
            }
        }
    }
}

// Power spectrum in any compression layout (soap.cpp:933-1012), one feature
// per lane and a warp-uniform walk over the layout; coef(t, k, l, m) reads
// coefficient (species t, radial k, degree l, component m) -- the species sum
// of mu1nu1 is formed on the fly.  Used where the tensor-core tails do not
// cover a layout.
template <class Coef, class OutT>
__device__ __forceinline__ void power_generic(const Coef& coef, const double* __restrict__ pref, int S, int n, int L,
                                              int compression, OutT* __restrict__ out, int lane) {
    int64_t f = 0;
    auto dot = [&](int t1, int n1, int t2, int n2, int l) {
        double acc = 0.0;
        for (int m = 0; m < 2 * l + 1; ++m) {
            double b;
            if (t2 < 0) {  // species sum (mu1nu1)
                b = 0.0;
                for (int t = 0; t < S; ++t) b += coef(t, n2, l, m);
            } else {
                b = coef(t2, n2, l, m);
            }
            acc = fma(coef(t1, n1, l, m), b, acc);
        }
        return pref[l] * acc;
    };
    if (compression == 2) {  // mu1nu1: species -> l -> n1 -> n2 (all)
        for (int t = 0; t < S; ++t)
            for (int l = 0; l <= L; ++l)
                for (int n1 = 0; n1 < n; ++n1) {
                    for (int n2 = lane; n2 < n; n2 += 32) out[f + n2] = (OutT)dot(t, n1, -1, n2, l);
                    f += n;
                }
    } else if (compression == 3) {  // crossover: species -> l -> n1 -> n2 >= n1
        for (int t = 0; t < S; ++t)
            for (int l = 0; l <= L; ++l)
                for (int n1 = 0; n1 < n; ++n1) {
                    for (int n2 = n1 + lane; n2 < n; n2 += 32) out[f + n2 - n1] = (OutT)dot(t, n1, t, n2, l);
                    f += n - n1;
                }
    } else {  // off (and mu2, one pooled species): t1 <= t2 -> l -> n1 -> n2 (>= n1 when t1 == t2)
        for (int t1 = 0; t1 < S; ++t1)
            for (int t2 = t1; t2 < S; ++t2)
                for (int l = 0; l <= L; ++l)
                    for (int n1 = 0; n1 < n; ++n1) {
                        const int lo = t1 == t2 ? n1 : 0;
                        for (int n2 = lo + lane; n2 < n; n2 += 32) out[f + n2 - lo] = (OutT)dot(t1, n1, t2, n2, l);
                        f += n - lo;
                    }
    }
}

// l groups sized so that a lane's register rows stay near 50 doubles.
// Rows r1 = r1_first, r1_first + r1_step, ... (several warps split a centre).
template <int LMAX, class OutT>
__device__ __forceinline__ void power_spectrum_warp(const SoapTables& tab, const double* __restrict__ c,
                                                    OutT* __restrict__ out, int lane, int r1_first = 0,
                                                    int r1_step = 1) {
    if constexpr (LMAX <= 6) {
        power_group<0, LMAX, OutT>(tab, c, out, lane, r1_first, r1_step);
    } else if constexpr (LMAX <= 8) {
        power_group<0, 5, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<6, LMAX, OutT>(tab, c, out, lane, r1_first, r1_step);
    } else {
        power_group<0, 6, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<7, 9, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<10, 11, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<12, 13, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<14, 15, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<16, 17, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<18, 19, OutT>(tab, c, out, lane, r1_first, r1_step);
        power_group<20, 20, OutT>(tab, c, out, lane, r1_first, r1_step);
    }
}

// In-place beta transform of the raw sums R[l][t][k][m] -> c[l][t][n][m]
// (padded rows), soap.cpp:915-926.  For n_max <= 8 the n x n block beta_l
// sits in registers while the warp sweeps the (t, m) columns of that l.
template <int NMAX>
__device__ __forceinline__ void beta_transform_warp(const SoapTables& tab, const double* __restrict__ beta,
                                                    double* __restrict__ R, int lane, int nthreads = 32) {
    const int S = tab.coef_species, n = tab.n_max, L = tab.l_max;
    for (int l = 0; l <= L; ++l) {
        const int len = 2 * l + 1, pad = 2 * l + 2;
        const int cols = S * len;
        double* rl = R + cblock(S, n, l);
        const double* bl = beta + (int64_t)l * n * n;
        if constexpr (NMAX <= 8) {
            double b[NMAX][NMAX];
#pragma unroll
            for (int i = 0; i < NMAX; ++i)
#pragma unroll
                for (int k = 0; k < NMAX; ++k) b[i][k] = (i < n && k < n) ? tab.soap_scale * bl[i * n + k] : 0.0;
            for (int col = lane; col < cols; col += nthreads) {
                const int t = col / len;
                const int m = col - t * len;
                double* base = rl + t * n * pad + m;
                double r[NMAX];
#pragma unroll
                for (int k = 0; k < NMAX; ++k) r[k] = k < n ? base[k * pad] : 0.0;
#pragma unroll
                for (int i = 0; i < NMAX; ++i) {
                    double acc = 0.0;
#pragma unroll
                    for (int k = 0; k < NMAX; ++k) acc = fma(b[i][k], r[k], acc);
                    if (i < n) base[i * pad] = acc;
                }
            }
        } else {
            for (int col = lane; col < cols; col += nthreads) {
                const int t = col / len;
                const int m = col - t * len;
                double* base = rl + t * n * pad + m;
                double r[NMAX];
#pragma unroll
                for (int k = 0; k < NMAX; ++k) r[k] = k < n ? base[k * pad] : 0.0;
                for (int nn = 0; nn < n; ++nn) {
                    double acc = 0.0;
#pragma unroll
                    for (int k = 0; k < NMAX; ++k) {
                        if (k < n) acc = fma(bl[nn * n + k], r[k], acc);
                    }
                    base[nn * pad] = tab.soap_scale * acc;
                }
            }
        }
    }
}

// Flattened candidate walk of one centre (warp-cooperative).  The bin
// neighbourhood of the centre is a set of (row, x-image) entries, each a
// contiguous run of sorted atoms; 32 entries per round are prefix-summed and
// each candidate chunk then gives every lane one candidate.  visit(valid, j,
// tx, ty, tz) is called by all lanes the same number of times.
template <class Visit>
__device__ __forceinline__ void for_each_candidate_flat(const StructInfo& si, const BinView& v, int64_t center,
                                                        int lane, int* __restrict__ seg_prefix,
                                                        int* __restrict__ seg_start, int* __restrict__ seg_t,
                                                        Visit&& visit) {
    const int Mx = si.M[0], My = si.M[1], Mz = si.M[2];
    const int Kx = si.K[0], Ky = si.K[1], Kz = si.K[2];
    const int cb = v.bin_of[center];
    const int cx = cb % Mx, cy = (cb / Mx) % My, cz = cb / (Mx * My);
    const int64_t bb = si.bin_base;
    const int64_t ab = si.atom_begin;
    const int lo = cx - Kx, hi = cx + Kx;
    const int tx0 = si.periodic ? floor_div(lo, Mx) : 0;
    const int nxs = si.periodic ? floor_div(hi, Mx) - tx0 + 1 : 1;
    const int wy = 2 * Ky + 1;
    const int entries = wy * (2 * Kz + 1) * nxs;
    for (int round = 0; round < entries; round += 32) {
        const int e = round + lane;
        bool valid = e < entries;
        int start = 0, len = 0, tpack = 0;
        if (valid) {
            const int row = e / nxs;
            const int xs = e - row * nxs;
            const int dz = row / wy - Kz;
            const int dy = row - (row / wy) * wy - Ky;
            const int ey = cy + dy, ez = cz + dz;
            int ty = 0, tz = 0, tx = 0, b0, b1;
            if (si.periodic) {
                ty = floor_div(ey, My);
                tz = floor_div(ez, Mz);
                tx = tx0 + xs;
                b0 = max(lo, tx * Mx) - tx * Mx;
                b1 = min(hi, tx * Mx + Mx - 1) - tx * Mx;
            } else {
                valid = ey >= 0 && ey < My && ez >= 0 && ez < Mz;
                b0 = max(lo, 0);
                b1 = min(hi, Mx - 1);
            }
            valid = valid && b0 <= b1;
            if (valid) {
                const int64_t rowbase = bb + Mx * ((ey - ty * My) + My * (ez - tz * Mz));
                start = v.bin_start[rowbase + b0];
                len = v.bin_start[rowbase + b1 + 1] - start;
                tpack = (tx + 512) | ((ty + 512) << 10) | ((tz + 512) << 20);
            }
        }
        int incl = len;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int up = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += up;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        __syncwarp();
        seg_prefix[lane] = incl - len;
        seg_start[lane] = start;
        seg_t[lane] = tpack;
        __syncwarp();
        for (int q0 = 0; q0 < total; q0 += 32) {
            const int q = q0 + lane;
            const bool cvalid = q < total;
            int i = 0;
#pragma unroll
            for (int step = 16; step > 0; step >>= 1)
                if (seg_prefix[i + step] <= q) i += step;
            const int a = seg_start[i] + (q - seg_prefix[i]);
            const int tp = seg_t[i];
            const int j = cvalid ? v.sorted[ab + a] : 0;
            visit(cvalid, j, (tp & 1023) - 512, ((tp >> 10) & 1023) - 512, ((tp >> 20) & 1023) - 512);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// Centre kernel.  Template parameters: MAXT species register banks per pass;
// L0..L2 the padded lengths (2l+1 maxima) of the three channel slots a lane
// owns per pass (0 = slot unused); NMAX >= n_max; LMAX >= l_max; MINB the
// minimum resident CTAs per SM the register allocation must allow.
template <int MAXT, int L0, int L1, int L2, int NMAX, int LMAX, int MINB>
__global__ void __launch_bounds__(kWarps * 32, MINB)
soap_center_kernel(const __grid_constant__ SoapTables tab, const SoapPointers p) {
    constexpr int NS = (L0 > 0) + (L1 > 0) + (L2 > 0);
    // n_max <= 8: the beta transform and power spectrum run on the fp64 tensor
    // cores (dmma.cuh) from a row-strided coefficient block; otherwise scalar.
    constexpr bool kMmaTail = NMAX <= 8;
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // S: species of the coefficient block (1 when mu2 pools them all into one
    // density, soap.cpp:613-615); per-edge weights when a weighting function,
    // w0 or the mu2 pooling asks for them (soap_weight, soap.cpp:389-420).
    const int S = tab.coef_species, n = tab.n_max, H = tab.hp;
    const bool pooled = tab.compression == 1;
    const bool weighted = tab.weighted != 0;
    const int beta_count = (tab.l_max + 1) * n * n;
    // CTA-shared: exp table (32 doubles), then beta (optional).
    double* etab = reinterpret_cast<double*>(smem);
    if (threadIdx.x < 32) etab[threadIdx.x] = kExp2Table[threadIdx.x];
    int shared_bytes = 256;
    const double* beta = p.betas;
    if constexpr (kMmaTail) {
        // [l][n][k] scaled by pi^{3/2}, zero padded to 8 x 8.
        double* bt = reinterpret_cast<double*>(smem + 256);
        for (int i = threadIdx.x; i < (tab.l_max + 1) * 64; i += blockDim.x) {
            const int l = i / 64, nn = (i / 8) % 8, k = i % 8;
            bt[i] = (nn < n && k < n) ? tab.soap_scale * p.betas[((int64_t)l * n + nn) * n + k] : 0.0;
        }
        beta = bt;
        shared_bytes += (tab.l_max + 1) * 64 * 8;
    } else if (tab.beta_in_smem) {
        double* sbeta = reinterpret_cast<double*>(smem + 256);
        for (int i = threadIdx.x; i < beta_count; i += blockDim.x) sbeta[i] = p.betas[i];
        beta = sbeta;
        shared_bytes += (beta_count * 8 + 15) & ~15;
    }
    __syncthreads();
    // Centres [grid_begin, grid_end) of this launch (the block's, or a chunk of it).
    const int64_t center = p.grid_begin + (int64_t)blockIdx.x * kWarps + warp;
    if (center >= p.grid_end) return;

    unsigned char* region = smem + shared_bytes + (size_t)warp * tab.warp_bytes;
    int* seg_prefix = reinterpret_cast<int*>(region);          // 40 ints
    int* seg_start = seg_prefix + 40;                           // 32 ints
    int* seg_t = seg_start + 32;                                // 32 ints
    int* perm = seg_t + 32;                                     // 32 ints: chunk order by species
    double* pdx = reinterpret_cast<double*>(region + kRegionHeader);
    double* pdy = pdx + kPending;
    double* pdz = pdy + kPending;
    double* pr2 = pdz + kPending;
    int32_t* ptype = reinterpret_cast<int32_t*>(pr2 + kPending);
    double* pw = reinterpret_cast<double*>(region + kRegionHeader + kPending * 36);
    double* ybuf = reinterpret_cast<double*>(region + kRegionHeader + kPending * 44);
    const int64_t local = center - p.center_begin;
    double* R = tab.r_global ? p.rbuf + local * tab.rsize : reinterpret_cast<double*>(region + tab.r_offset);

    const BinView& bv = p.bins;
    const StructInfo si = bv.info[bv.struct_of[center]];
    const int wi[3] = {bv.wrap[3 * center], bv.wrap[3 * center + 1], bv.wrap[3 * center + 2]};
    const int chunk = tab.chunk;

    for (int tg = 0; tg < tab.type_groups; ++tg) {
        const int tb = tg * MAXT;
        const int te = min(S, tb + MAXT);
        for (int sg = 0; sg < tab.slot_groups; ++sg) {
            double pref[3], expo[3];
            int il[3], ik[3];
            bool ivalid[3];
#pragma unroll
            for (int s = 0; s < 3; ++s) {
                const int idx = 32 * (NS * sg + s) + lane;
                ivalid[s] = s < NS && idx < tab.items;
                const RadialItem it = ivalid[s] ? p.items[idx] : RadialItem{0.0, 0.0, 0, 0};
                pref[s] = it.prefactor;
                expo[s] = -it.exponent;
                il[s] = it.l;
                ik[s] = it.k;
            }
            const double* ybase0 = ybuf + il[0] * (il[0] + 1);
            const double* ybase1 = ybuf + il[1] * (il[1] + 1);
            const double* ybase2 = ybuf + il[2] * (il[2] + 1);
            double a0[MAXT][L0 > 0 ? L0 : 1];
            double a1[MAXT][L1 > 0 ? L1 : 1];
            double a2[MAXT][L2 > 0 ? L2 : 1];
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
#pragma unroll
                for (int m = 0; m < (L0 > 0 ? L0 : 1); ++m) a0[t][m] = 0.0;
#pragma unroll
                for (int m = 0; m < (L1 > 0 ? L1 : 1); ++m) a1[t][m] = 0.0;
#pragma unroll
                for (int m = 0; m < (L2 > 0 ? L2 : 1); ++m) a2[t][m] = 0.0;
            }

            // One edge into species bank TT: 16-byte broadcast reads of the
            // harmonic row (padding only feeds accumulators that are never stored).
            auto accumulate = [&](auto bank, double g0, double g1, double g2, int eo) {
                constexpr int TT = decltype(bank)::value;
#pragma unroll
                for (int m = 0; m < L0; m += 2) {
                    const double2 y = *reinterpret_cast<const double2*>(ybase0 + eo + m);
                    a0[TT][m] = fma(g0, y.x, a0[TT][m]);
                    if (m + 1 < L0) a0[TT][m + 1] = fma(g0, y.y, a0[TT][m + 1]);
                }
#pragma unroll
                for (int m = 0; m < L1; m += 2) {
                    const double2 y = *reinterpret_cast<const double2*>(ybase1 + eo + m);
                    a1[TT][m] = fma(g1, y.x, a1[TT][m]);
                    if (m + 1 < L1) a1[TT][m + 1] = fma(g1, y.y, a1[TT][m + 1]);
                }
#pragma unroll
                for (int m = 0; m < L2; m += 2) {
                    const double2 y = *reinterpret_cast<const double2*>(ybase2 + eo + m);
                    a2[TT][m] = fma(g2, y.x, a2[TT][m]);
                    if (m + 1 < L2) a2[TT][m + 1] = fma(g2, y.y, a2[TT][m + 1]);
                }
            };
            auto radial = [&](int e, double w, double& g0, double& g1, double& g2) {
                const double r2e = pr2[e];
                g0 = L0 > 0 ? w * pref[0] * exp_nonpositive(expo[0] * r2e, etab) : 0.0;
                g1 = L1 > 0 ? w * pref[1] * exp_nonpositive(expo[1] * r2e, etab) : 0.0;
                g2 = L2 > 0 ? w * pref[2] * exp_nonpositive(expo[2] * r2e, etab) : 0.0;
            };
            auto process = [&](int count) {
                if (lane < count)
                    harmonics_any<LMAX>(tab, pdx[lane], pdy[lane], pdz[lane], pr2[lane], ybuf + lane * H);
                // Stable counting sort of the chunk by species bank: each bank
                // then runs over a contiguous range with a static register bank.
                const int mine = lane < count ? ptype[lane] : MAXT;
                const unsigned lt = (1u << lane) - 1u;
                int run_start[MAXT + 1];
                run_start[0] = 0;
                int rank = 0;
#pragma unroll
                for (int tt = 0; tt < MAXT; ++tt) {
                    const unsigned m = __ballot_sync(0xffffffffu, mine == tt);
                    if (mine == tt) rank = run_start[tt] + __popc(m & lt);
                    run_start[tt + 1] = run_start[tt] + __popc(m);
                }
                if (lane < count) perm[rank] = lane;
                __syncwarp();
                static_for<0, MAXT>([&](auto bank) {
                    constexpr int TT = decltype(bank)::value;
                    const int end = run_start[TT + 1];
                    if (run_start[TT] == end) return;
                    // The pooled density carries each edge's species weight.
                    const double w = pooled ? 1.0 : tab.species_weight[tb + TT];
                    int i = run_start[TT];
                    // Two edges per step: more independent exp() chains in flight.
                    for (; i + 1 < end; i += 2) {
                        const int ea = perm[i], eb = perm[i + 1];
                        double ga0, ga1, ga2, gb0, gb1, gb2;
                        radial(ea, weighted ? w * pw[ea] : w, ga0, ga1, ga2);
                        radial(eb, weighted ? w * pw[eb] : w, gb0, gb1, gb2);
                        accumulate(bank, ga0, ga1, ga2, ea * H);
                        accumulate(bank, gb0, gb1, gb2, eb * H);
                    }
                    if (i < end) {
                        const int ea = perm[i];
                        double ga0, ga1, ga2;
                        radial(ea, weighted ? w * pw[ea] : w, ga0, ga1, ga2);
                        accumulate(bank, ga0, ga1, ga2, ea * H);
                    }
                });
                __syncwarp();
            };

            int pcount = 0;
            // One batch of up to 32 accepted edges (lanes with ok) into the
            // queue in lane order, whole chunks drained.
            auto enqueue = [&](bool ok, double dx, double dy, double dz, double d2, double ew, int t) {
                const unsigned mask = __ballot_sync(0xffffffffu, ok);
                if (ok) {
                    const int q = pcount + __popc(mask & ((1u << lane) - 1u));
                    pdx[q] = dx;
                    pdy[q] = dy;
                    pdz[q] = dz;
                    pr2[q] = d2;
                    pw[q] = ew;
                    ptype[q] = pooled ? 0 : t - tb;
                }
                pcount += __popc(mask);
                // Drain whole chunks; the queue holds < chunk entries between
                // candidate batches, so it never exceeds chunk + 31 <= 63 < kPending.
                while (pcount >= chunk) {
                    __syncwarp();
                    process(chunk);
                    const int rem = pcount - chunk;
                    double sx = 0.0, sy = 0.0, sz = 0.0, sr = 0.0, sw = 1.0;
                    int st = 0;
                    if (lane < rem) {
                        sx = pdx[chunk + lane];
                        sy = pdy[chunk + lane];
                        sz = pdz[chunk + lane];
                        sr = pr2[chunk + lane];
                        sw = pw[chunk + lane];
                        st = ptype[chunk + lane];
                    }
                    __syncwarp();
                    if (lane < rem) {
                        pdx[lane] = sx;
                        pdy[lane] = sy;
                        pdz[lane] = sz;
                        pr2[lane] = sr;
                        pw[lane] = sw;
                        ptype[lane] = st;
                    }
                    __syncwarp();
                    pcount = rem;
                }
            };
            // Edge lists (p.edge_count set): the centre's accepted edges from
            // the walk kernel's slot, unless it overflowed.  The walk visits
            // the same bin rows in the same order and only drops candidates
            // beyond the prefilter sphere, so for float64 rows (every edge
            // through the exact test) the edges arrive in this kernel's own
            // walk order and the rows are the same bit for bit.
            const int64_t slot = center - p.grid_begin;
            const int nedges = p.edge_count ? p.edge_count[slot] : -1;
            if (nedges >= 0 && nedges <= tab.edge_cap) {
                for (int f = 0; f < nedges; f += 32) {
                    const int e = f + lane;
                    bool ok = false;
                    double4 d = make_double4(0.0, 0.0, 0.0, 0.0);
                    double ew = 1.0;
                    int t = -1;
                    if (e < nedges) {
                        d = p.edges[slot * tab.edge_cap + e];
                        const int info = p.edge_info[slot * tab.edge_cap + e];
                        t = info & 0xffff;
                        ok = pooled || (t >= tb && t < te);
                        if (ok && weighted) {
                            ew = soap_edge_weight(tab, d.w, (info >> 16) != 0);
                            if (pooled) ew *= tab.species_weight[t];
                        }
                    }
                    enqueue(ok, d.x, d.y, d.z, d.w, ew, t);
                }
            } else {
                for_each_candidate_flat(si, bv, center, lane, seg_prefix, seg_start, seg_t,
                                        [&](bool valid, int j, int tx, int ty, int tz) {
                    int nimg[3];
                    double dx = 0.0, dy = 0.0, dz = 0.0, d2 = 0.0, ew = 1.0;
                    int t = -1;
                    bool ok = false;
                    if (valid) {
                        t = bv.type[si.atom_begin + j];
                        if (pooled || (t >= tb && t < te))
                            ok = accept_candidate(si, bv, p.positions, center, wi, j, tx, ty, tz, tab.cutoff2, nimg,
                                                  dx, dy, dz, d2);
                        if (ok && weighted) {
                            ew = soap_edge_weight(tab, d2, si.atom_begin + j == center && nimg[0] == 0 &&
                                                               nimg[1] == 0 && nimg[2] == 0);
                            if (pooled) ew *= tab.species_weight[t];
                        }
                    }
                    enqueue(ok, dx, dy, dz, d2, ew, t);
                });
            }
            __syncwarp();
            if (pcount > 0) process(pcount);

            // Flush the raw sums.  Tensor-core tail: row (t, k), columns
            // col_off(l) .. + kpad(l), padding written as 0; scalar tail:
            // R[l][t][k][m], rows padded to 2l+2.
            auto flush_slot = [&](auto len_c, auto& a, int sl, int tt) {
                constexpr int LS = decltype(len_c)::value;
                const int t = tb + tt;
                const int len = 2 * il[sl] + 1;
                if constexpr (kMmaTail) {
                    double* dst = R + (t * n + ik[sl]) * tab.rs + mma::col_off(il[sl]);
                    const int kp = mma::kpad(il[sl]);
#pragma unroll
                    for (int m = 0; m < LS; ++m)
                        if (m < kp) dst[m] = m < len ? a[tt][m] : 0.0;
#pragma unroll
                    for (int m = LS; m < ((LS + 3) & ~3); ++m)
                        if (m < kp) dst[m] = 0.0;
                } else {
                    double* dst = R + cblock(S, n, il[sl]) + (t * n + ik[sl]) * (len + 1);
#pragma unroll
                    for (int m = 0; m < LS; ++m)
                        if (m < len) dst[m] = a[tt][m];
                }
            };
#pragma unroll
            for (int tt = 0; tt < MAXT; ++tt) {
                if (tb + tt < te) {
                    if (L0 > 0 && ivalid[0]) flush_slot(std::integral_constant<int, L0>{}, a0, 0, tt);
                    if (L1 > 0 && ivalid[1]) flush_slot(std::integral_constant<int, L1>{}, a1, 1, tt);
                    if (L2 > 0 && ivalid[2]) flush_slot(std::integral_constant<int, L2>{}, a2, 2, tt);
                }
            }
            __syncwarp();
        }
    }

    // mu1nu1 and crossover rows (soap.cpp:933-996): one feature per lane over
    // the layout, from the transformed coefficients.
    auto compressed_rows = [&](auto coef) {
        if (tab.average == 0) {
            const int64_t row = center - p.out_row_begin;
            if (tab.out_f64)
                power_generic(coef, tab.power_pref, S, n, tab.l_max, tab.compression,
                              static_cast<double*>(p.out) + row * tab.features, lane);
            else
                power_generic(coef, tab.power_pref, S, n, tab.l_max, tab.compression,
                              static_cast<float*>(p.out) + row * tab.features, lane);
        } else {
            power_generic(coef, tab.power_pref, S, n, tab.l_max, tab.compression, p.pbuf + local * tab.features,
                          lane);
        }
    };
    const bool compressed = tab.average != 1 && (tab.compression == 2 || tab.compression == 3);
    if constexpr (kMmaTail) {
        const int g = lane >> 2, q = lane & 3, L = tab.l_max, R_rows = tab.rows;
        mma::beta_mma<LMAX>(beta, R, tab.rs, L, S, n, g, q);
        __syncwarp();
        const mma::FeatureMap fm{S, n, L, R_rows, tab.n_magic};
        if (compressed) {
            const int rs = tab.rs;
            compressed_rows([&](int t, int k, int l, int m) { return R[(t * n + k) * rs + mma::col_off(l) + m]; });
        } else if (tab.average == 0) {
            const int64_t row = center - p.out_row_begin;
            if (tab.out_f64)
                mma::power_mma<LMAX>(fm, tab.power_pref, R, tab.rs, static_cast<double*>(p.out) + row * tab.features,
                                     g, q);
            else
                mma::power_mma<LMAX>(fm, tab.power_pref, R, tab.rs, static_cast<float*>(p.out) + row * tab.features,
                                     g, q);
        } else if (tab.average == 1) {
            // The structure kernel's layout: [l][r][m], rows padded to 2l+2.
            double* dst = p.cbuf + local * tab.csize;
            for (int l = 0; l <= L; ++l) {
                const int pad = 2 * l + 2;
                double* dl = dst + cblock(S, n, l);
                const double* src = R + mma::col_off(l);
                for (int i = lane; i < R_rows * pad; i += 32) {
                    const int r = i / pad, m = i - r * pad;
                    dl[i] = m < 2 * l + 1 ? src[r * tab.rs + m] : 0.0;
                }
            }
        } else {
            mma::power_mma<LMAX>(fm, tab.power_pref, R, tab.rs, p.pbuf + local * tab.features, g, q);
        }
        return;
    } else {
    beta_transform_warp<NMAX>(tab, beta, R, lane);
    __syncwarp();
    if (compressed) {
        compressed_rows([&](int t, int k, int l, int m) { return R[cblock(S, n, l) + (t * n + k) * (2 * l + 2) + m]; });
    } else if (tab.average == 0) {
        const int64_t row = center - p.out_row_begin;
        if (tab.out_f64)
            power_spectrum_warp<LMAX>(tab, R, static_cast<double*>(p.out) + row * tab.features, lane);
        else
            power_spectrum_warp<LMAX>(tab, R, static_cast<float*>(p.out) + row * tab.features, lane);
    } else if (tab.average == 1) {
        double* dst = p.cbuf + local * tab.csize;
        for (int i = lane; i < tab.csize; i += 32) dst[i] = R[i];
    } else {
        power_spectrum_warp<LMAX>(tab, R, p.pbuf + local * tab.features, lane);
    }
    }
}

// ---------------------------------------------------------------------------
// Structure-level averages (one CTA per structure of the block).
//   inner: c averaged over the structure's atoms, then the power spectrum
//          (soap.cpp:1019-1067);
//   outer: power spectra averaged over the atoms (soap.cpp:1068-1120).
template <int LMAX>
__global__ void __launch_bounds__(kWarps * 32)
soap_structure_kernel(const __grid_constant__ SoapTables tab, const int64_t* __restrict__ offsets,
                      int64_t structure_begin, int64_t structure_end, const double* __restrict__ cbuf,
                      const double* __restrict__ pbuf, void* out, int64_t out_row_begin) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int64_t s = structure_begin + blockIdx.x;
    if (s >= structure_end) return;
    const int64_t block_first_atom = offsets[structure_begin];
    const int64_t a0 = offsets[s] - block_first_atom;
    const int64_t count = offsets[s + 1] - offsets[s];
    const double scale = count > 0 ? 1.0 / (double)count : 0.0;
    const int64_t F = tab.features;
    if (tab.average == 1) {
        const int csize = tab.csize;
        double* c = reinterpret_cast<double*>(smem);
        for (int i = threadIdx.x; i < csize; i += blockDim.x) {
            double sum = 0.0;
            for (int64_t a = 0; a < count; ++a) sum += cbuf[(a0 + a) * csize + i];
            c[i] = sum * scale;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            if (tab.compression == 2 || tab.compression == 3) {
                // c layout: [l][t n + k][m], rows padded to 2l + 2.
                const int S = tab.coef_species, n = tab.n_max;
                auto coef = [&](int t, int k, int l, int m) { return c[cblock(S, n, l) + (t * n + k) * (2 * l + 2) + m]; };
                if (tab.out_f64)
                    power_generic(coef, tab.power_pref, S, n, tab.l_max, tab.compression,
                                  static_cast<double*>(out) + (s - out_row_begin) * F, (int)threadIdx.x);
                else
                    power_generic(coef, tab.power_pref, S, n, tab.l_max, tab.compression,
                                  static_cast<float*>(out) + (s - out_row_begin) * F, (int)threadIdx.x);
            } else if (tab.out_f64) {
                power_spectrum_warp<LMAX>(tab, c, static_cast<double*>(out) + (s - out_row_begin) * F, threadIdx.x);
            } else {
                power_spectrum_warp<LMAX>(tab, c, static_cast<float*>(out) + (s - out_row_begin) * F, threadIdx.x);
            }
        }
    } else {
        for (int64_t i = threadIdx.x; i < F; i += blockDim.x) {
            double sum = 0.0;
            for (int64_t a = 0; a < count; ++a) sum += pbuf[(a0 + a) * F + i];
            const double v = sum * scale;
            if (tab.out_f64)
                static_cast<double*>(out)[(s - out_row_begin) * F + i] = v;
            else
                static_cast<float*>(out)[(s - out_row_begin) * F + i] = (float)v;
        }
    }
}

}  // namespace mdsoap
