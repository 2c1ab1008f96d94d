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
//   * candidates from the bin walk are accepted with the reference's exact
//     geometry and appended (ballot + popc) to a per-warp queue in shared
//     memory;
//   * per chunk of up to 32 queued edges, lane e evaluates Y_{lm} of edge e by
//     the Cartesian recurrence and stores the row in shared memory;
//   * every lane owns up to three radial channels (l, k) (channels sorted by
//     l descending, 32 per slot), evaluates its own exp() per edge and keeps
//     S[t][l][k][0..2l] in registers, reading Y_{lm} rows as shared-memory
//     broadcasts; species live in separate register banks picked by a
//     warp-uniform branch;
//   * the raw sums go to shared memory, beta is applied in place, and the
//     power spectrum is written straight to the output row (lane = column r2,
//     broadcast row r1), so no feature staging buffer is needed.
#pragma once

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
    int32_t r_global;     // 1: coefficient blocks live in global scratch (too big for shared memory)
    int32_t pad_;
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
    void* out;                // average off: rows of centres; else unused
    double* cbuf;             // average inner: per-centre coefficients (block-local rows)
    double* pbuf;             // average outer: per-centre power spectra (block-local rows)
    double* rbuf;             // r_global: per-centre coefficient scratch (block-local rows)
    int64_t out_row_begin;    // average off: output row of centre c is c - out_row_begin
    int64_t center_begin;
    int64_t center_end;
};

__device__ __forceinline__ int tri(int l, int m) { return l * (l + 1) / 2 + m; }

// Real regular solid harmonics of one displacement into out[0..H), layout
// l^2 + (l - m) = cos part, l^2 + l = m0, l^2 + (l + m) = sin part
// (soap.cpp:101-216 generic Cartesian recurrence, all l).
__device__ __forceinline__ void solid_harmonics(const SoapTables& tab, double x, double y, double z, double r2,
                                                double* __restrict__ out) {
    const int L = tab.l_max;
    double dr = 1.0, di = 0.0;  // diagonal P_mm (real, imaginary)
    for (int m = 0; m <= L; ++m) {
        if (m > 0) {
            const double f = -(2.0 * m - 1.0);
            const double nr = f * (x * dr - y * di);
            const double ni = f * (x * di + y * dr);
            dr = nr;
            di = ni;
        }
        double pr2 = dr, pi2 = di;
        {
            const double nrm = tab.ynorm[tri(m, m)];
            if (m == 0) {
                out[0] = nrm * pr2;
            } else {
                out[m * m] = nrm * pr2;              // l = m: l^2 + l - m
                out[m * m + 2 * m] = nrm * pi2;      // l^2 + l + m
            }
        }
        if (m < L) {
            const double c = (2.0 * m + 1.0) * z;
            double pr1 = c * dr, pi1 = c * di;
            {
                const int l = m + 1;
                const double nrm = tab.ynorm[tri(l, m)];
                out[l * l + l - m] = nrm * pr1;
                if (m > 0) out[l * l + l + m] = nrm * pi1;
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
                out[l * l + l - m] = nrm * nr;
                if (m > 0) out[l * l + l + m] = nrm * ni;
            }
        }
    }
}

__device__ __forceinline__ int64_t feature_index(int S, int n, int L, int t1, int n1, int t2, int n2, int l) {
    const int64_t T = (int64_t)n * (n + 1) / 2;
    const int64_t nn = (int64_t)n * n;
    int64_t base = (int64_t)(L + 1) * (t1 * T + nn * ((int64_t)t1 * (S - 1) - (int64_t)t1 * (t1 - 1) / 2));
    if (t2 > t1) {
        base += (int64_t)(L + 1) * (T + (int64_t)(t2 - t1 - 1) * nn);
        return base + l * nn + (int64_t)n1 * n + n2;
    }
    return base + l * T + (int64_t)n1 * n - (int64_t)n1 * (n1 - 1) / 2 + (n2 - n1);
}

// Power spectrum of one coefficient block c (layout [l][t][n][m], S n H
// doubles in shared memory) into the feature row `out` (global memory).
template <int LMAX, class OutT>
__device__ __forceinline__ void power_spectrum_warp(const SoapTables& tab, const double* __restrict__ c,
                                                    OutT* __restrict__ out, int lane) {
    const int S = tab.n_species, n = tab.n_max, L = tab.l_max, R = tab.rows;
    for (int r2base = 0; r2base < R; r2base += 32) {
        const int r2 = r2base + lane;
        const bool active = r2 < R;
        const int t2 = active ? r2 / n : 0;
        const int n2 = active ? r2 - t2 * n : 0;
        const int r1_end = min(R - 1, r2base + 31);
        for (int l = 0; l <= L; ++l) {
            const int len = 2 * l + 1;
            const double* cl = c + (int64_t)S * n * l * l;
            double own[2 * LMAX + 1];
#pragma unroll
            for (int m = 0; m < 2 * LMAX + 1; ++m) own[m] = (m < len && active) ? cl[r2 * len + m] : 0.0;
            const double pref = tab.power_pref[l];
            int t1 = 0, n1 = 0;
            for (int r1 = 0; r1 <= r1_end; ++r1) {
                const double* o = cl + r1 * len;
                double v = 0.0;
#pragma unroll
                for (int m = 0; m < 2 * LMAX + 1; ++m) {
                    if (m < len) v = fma(o[m], own[m], v);
                }
                if (active && r2 >= r1) out[feature_index(S, n, L, t1, n1, t2, n2, l)] = (OutT)(pref * v);
                if (++n1 == n) {
                    n1 = 0;
                    ++t1;
                }
            }
        }
    }
}

// In-place beta transform of the raw sums R[l][t][k][m] -> c[l][t][n][m].
template <int NMAX>
__device__ __forceinline__ void beta_transform_warp(const SoapTables& tab, const double* __restrict__ beta,
                                                    double* __restrict__ R, int lane) {
    const int S = tab.n_species, n = tab.n_max, L = tab.l_max;
    for (int l = 0; l <= L; ++l) {
        const int len = 2 * l + 1;
        const int cols = S * len;
        double* rl = R + (int64_t)S * n * l * l;
        const double* bl = beta + (int64_t)l * n * n;
        for (int col = lane; col < cols; col += 32) {
            const int t = col / len;
            const int m = col - t * len;
            double* base = rl + t * n * len + m;
            double r[NMAX];
#pragma unroll
            for (int k = 0; k < NMAX; ++k) r[k] = k < n ? base[k * len] : 0.0;
            for (int nn = 0; nn < n; ++nn) {
                double acc = 0.0;
#pragma unroll
                for (int k = 0; k < NMAX; ++k) {
                    if (k < n) acc = fma(bl[nn * n + k], r[k], acc);
                }
                base[nn * len] = tab.soap_scale * acc;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Centre kernel.  Template parameters: MAXT species register banks per pass;
// L0..L2 the padded lengths (2l+1 maxima) of the three channel slots a lane
// owns per pass (0 = slot unused); NMAX >= n_max; LMAX >= l_max.
template <int MAXT, int L0, int L1, int L2, int NMAX, int LMAX>
__global__ void __launch_bounds__(kWarps * 32)
soap_center_kernel(const __grid_constant__ SoapTables tab, const SoapPointers p) {
    constexpr int NS = (L0 > 0) + (L1 > 0) + (L2 > 0);
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int S = tab.n_species, n = tab.n_max, H = tab.H;
    const int beta_count = (tab.l_max + 1) * n * n;
    int beta_bytes = 0;
    const double* beta = p.betas;
    if (tab.beta_in_smem) {
        double* sbeta = reinterpret_cast<double*>(smem);
        for (int i = threadIdx.x; i < beta_count; i += blockDim.x) sbeta[i] = p.betas[i];
        beta = sbeta;
        beta_bytes = (beta_count * 8 + 15) & ~15;
    }
    __syncthreads();
    const int64_t center = p.center_begin + (int64_t)blockIdx.x * kWarps + warp;
    if (center >= p.center_end) return;

    unsigned char* region = smem + beta_bytes + (size_t)warp * tab.warp_bytes;
    double* pdx = reinterpret_cast<double*>(region);
    double* pdy = pdx + kPending;
    double* pdz = pdy + kPending;
    double* pr2 = pdz + kPending;
    int32_t* ptype = reinterpret_cast<int32_t*>(pr2 + kPending);
    double* ybuf = reinterpret_cast<double*>(region + kPending * 36);
    const int64_t local = center - p.center_begin;
    double* R = tab.r_global ? p.rbuf + local * ((int64_t)S * n * H)
                             : reinterpret_cast<double*>(region + tab.r_offset);

    const BinView& bv = p.bins;
    const StructInfo* si_ptr = bv.info + bv.struct_of[center];
    const StructInfo si = *si_ptr;
    const int wi[3] = {bv.wrap[3 * center], bv.wrap[3 * center + 1], bv.wrap[3 * center + 2]};
    const int chunk = tab.chunk;

    for (int tg = 0; tg < tab.type_groups; ++tg) {
        const int tb = tg * MAXT;
        const int te = min(S, tb + MAXT);
        for (int sg = 0; sg < tab.slot_groups; ++sg) {
            double pref[3], expo[3];
            int yoff[3], il[3], ik[3];
            bool ivalid[3];
#pragma unroll
            for (int s = 0; s < 3; ++s) {
                const int idx = 32 * (NS * sg + s) + lane;
                ivalid[s] = s < NS && idx < tab.items;
                const RadialItem it = ivalid[s] ? p.items[idx] : RadialItem{0.0, 0.0, 0, 0};
                pref[s] = it.prefactor;
                expo[s] = it.exponent;
                il[s] = it.l;
                ik[s] = it.k;
                yoff[s] = it.l * it.l;
            }
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

            auto process = [&](int count) {
                if (lane < count) solid_harmonics(tab, pdx[lane], pdy[lane], pdz[lane], pr2[lane], ybuf + lane * H);
                __syncwarp();
                for (int e = 0; e < count; ++e) {
                    const double r2 = pr2[e];
                    const int t = ptype[e];
                    const double w = tab.species_weight[tb + t];
                    const double g0 = L0 > 0 ? w * pref[0] * exp(-expo[0] * r2) : 0.0;
                    const double g1 = L1 > 0 ? w * pref[1] * exp(-expo[1] * r2) : 0.0;
                    const double g2 = L2 > 0 ? w * pref[2] * exp(-expo[2] * r2) : 0.0;
                    const double* yr = ybuf + e * H;
#pragma unroll
                    for (int tt = 0; tt < MAXT; ++tt) {
                        if (tt == t) {
#pragma unroll
                            for (int m = 0; m < L0; ++m) a0[tt][m] = fma(g0, yr[yoff[0] + m], a0[tt][m]);
#pragma unroll
                            for (int m = 0; m < L1; ++m) a1[tt][m] = fma(g1, yr[yoff[1] + m], a1[tt][m]);
#pragma unroll
                            for (int m = 0; m < L2; ++m) a2[tt][m] = fma(g2, yr[yoff[2] + m], a2[tt][m]);
                        }
                    }
                }
                __syncwarp();
            };

            int pcount = 0;
            for_each_candidate(si, bv, center, lane, [&](bool valid, int j, int tx, int ty, int tz) {
                int nimg[3];
                double dx = 0.0, dy = 0.0, dz = 0.0, d2 = 0.0;
                int t = -1;
                bool ok = false;
                if (valid) {
                    t = bv.type[si.atom_begin + j];
                    if (t >= tb && t < te)
                        ok = accept_candidate(si, bv, p.positions, center, wi, j, tx, ty, tz, tab.cutoff2, nimg,
                                              dx, dy, dz, d2);
                }
                const unsigned mask = __ballot_sync(0xffffffffu, ok);
                if (ok) {
                    const int q = pcount + __popc(mask & ((1u << lane) - 1u));
                    pdx[q] = dx;
                    pdy[q] = dy;
                    pdz[q] = dz;
                    pr2[q] = d2;
                    ptype[q] = t - tb;
                }
                pcount += __popc(mask);
                if (pcount >= chunk) {
                    __syncwarp();
                    process(chunk);
                    const int rem = pcount - chunk;
                    double sx = 0.0, sy = 0.0, sz = 0.0, sr = 0.0;
                    int st = 0;
                    if (lane < rem) {
                        sx = pdx[chunk + lane];
                        sy = pdy[chunk + lane];
                        sz = pdz[chunk + lane];
                        sr = pr2[chunk + lane];
                        st = ptype[chunk + lane];
                    }
                    __syncwarp();
                    if (lane < rem) {
                        pdx[lane] = sx;
                        pdy[lane] = sy;
                        pdz[lane] = sz;
                        pr2[lane] = sr;
                        ptype[lane] = st;
                    }
                    __syncwarp();
                    pcount = rem;
                }
            });
            __syncwarp();
            if (pcount > 0) process(pcount);

            // Flush the raw sums: R[l][t][k][m] at S n l^2 + (t n + k)(2l+1) + m.
#pragma unroll
            for (int tt = 0; tt < MAXT; ++tt) {
                const int t = tb + tt;
                if (t < te) {
                    if (L0 > 0 && ivalid[0]) {
                        const int len = 2 * il[0] + 1;
                        double* dst = R + (int64_t)S * n * il[0] * il[0] + (t * n + ik[0]) * len;
#pragma unroll
                        for (int m = 0; m < L0; ++m)
                            if (m < len) dst[m] = a0[tt][m];
                    }
                    if (L1 > 0 && ivalid[1]) {
                        const int len = 2 * il[1] + 1;
                        double* dst = R + (int64_t)S * n * il[1] * il[1] + (t * n + ik[1]) * len;
#pragma unroll
                        for (int m = 0; m < L1; ++m)
                            if (m < len) dst[m] = a1[tt][m];
                    }
                    if (L2 > 0 && ivalid[2]) {
                        const int len = 2 * il[2] + 1;
                        double* dst = R + (int64_t)S * n * il[2] * il[2] + (t * n + ik[2]) * len;
#pragma unroll
                        for (int m = 0; m < L2; ++m)
                            if (m < len) dst[m] = a2[tt][m];
                    }
                }
            }
            __syncwarp();
        }
    }

    beta_transform_warp<NMAX>(tab, beta, R, lane);
    __syncwarp();
    if (tab.average == 0) {
        const int64_t row = center - p.out_row_begin;
        if (tab.out_f64)
            power_spectrum_warp<LMAX>(tab, R, static_cast<double*>(p.out) + row * tab.features, lane);
        else
            power_spectrum_warp<LMAX>(tab, R, static_cast<float*>(p.out) + row * tab.features, lane);
    } else if (tab.average == 1) {
        const int64_t csize = (int64_t)S * n * H;
        double* dst = p.cbuf + local * csize;
        for (int64_t i = lane; i < csize; i += 32) dst[i] = R[i];
    } else {
        power_spectrum_warp<LMAX>(tab, R, p.pbuf + local * tab.features, lane);
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
        const int64_t csize = (int64_t)tab.n_species * tab.n_max * tab.H;
        double* c = reinterpret_cast<double*>(smem);
        for (int64_t i = threadIdx.x; i < csize; i += blockDim.x) {
            double sum = 0.0;
            for (int64_t a = 0; a < count; ++a) sum += cbuf[(a0 + a) * csize + i];
            c[i] = sum * scale;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            if (tab.out_f64)
                power_spectrum_warp<LMAX>(tab, c, static_cast<double*>(out) + (s - out_row_begin) * F, threadIdx.x);
            else
                power_spectrum_warp<LMAX>(tab, c, static_cast<float*>(out) + (s - out_row_begin) * F, threadIdx.x);
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
