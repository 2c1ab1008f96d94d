// SOAP expansion + power spectrum on the fp64 tensor-core path (sm_100a DMMA).
//
// Same arithmetic as soap.cuh (cpp/src/standalone/soap.cpp:507-572 radial
// factors, :101-216 solid harmonics, :881-926 expansion and beta, :997-1012
// power spectrum); the three contractions run as fp64 mma.sync tiles instead
// of scalar FMAs, which on B200 issue 8-16x fewer warp instructions for the
// same flops:
//
//   expansion   S[t][l][k][m] += sum_e g_{lk}(r_e) Y_{lm}(d_e)     per 4 edges of
//               one species: A = Y^T (m x e), B = g (e x k), C = S^T (m x k)
//   beta        c[t][l][n][m] = pi^{3/2} sum_k beta_l[n][k] S[k][m]:  A = beta_l,
//               B = S (k x m), in place
//   power       P_l = C_l C_l^T over the rows r = t n_max + n (upper triangle,
//               16 x 8 tiles), K = m
//
// One warp per centre.  Accepted edges (exact reference geometry) are queued
// in shared memory; a flush sorts the queue by species (ballots) and walks
// each species' run in 4-edge groups: lanes (g, q) = (lane / 4, lane % 4)
// evaluate the exp() of channel (l, k = g) for edge q of the group -- the B
// fragment -- and read the A fragment from an 8-edge harmonic buffer filled
// by 4 lanes per edge (columns m = h, h+4, ... of phase h).  The species'
// accumulator fragments live in registers for the run and in the centre's
// coefficient block (fp64, rows r, stride RS = 4 mod 16 doubles so that every
// fragment read is bank-conflict free) in between.
#pragma once

#include "soap.cuh"

namespace mdsoap {

namespace mma {

constexpr int kQueue = 96;  // edge queue per warp (flush at 64; a candidate round adds <= 32)
constexpr int kFlush = 64;

// Shared-memory layout of one CTA (host and device agree through these).
struct Layout {
    int tri;          // (L+1)(L+2)/2 harmonic coefficients
    int coef_off;     // bytes: yra, yrb, ynorm (3 * tri doubles)
    int radial_off;   // (L+1) * 8 * {prefactor, -exponent}
    int beta_off;     // (L+1) * 8 * 8 scaled beta, zero padded
    int shared;       // bytes before the first warp region
    int rs, ys;       // row strides (doubles)
    int y_off, reg_off, warp_bytes;
};

__host__ __device__ inline Layout layout(int L, int rows) {
    Layout o{};
    auto al = [](int x) { return (x + 15) & ~15; };
    o.tri = (L + 1) * (L + 2) / 2;
    o.coef_off = 256;
    o.radial_off = al(o.coef_off + 3 * o.tri * 8);
    o.beta_off = al(o.radial_off + (L + 1) * 16 * 8);
    o.shared = al(o.beta_off + (L + 1) * 64 * 8);
    o.rs = row_stride(L);
    o.ys = y_stride(L);
    o.y_off = 512 + kQueue * 40;  // walk tables (512 B), then dx dy dz r2 (doubles), type, perm
    o.reg_off = al(o.y_off + 8 * o.ys * 8);
    o.warp_bytes = al(o.reg_off + rows * o.rs * 8);
    return o;
}

// Real solid harmonics of one displacement, columns |m| = h, h+4, h+8, ... of
// phase h (0..3), into a compact row: degree l at l*l, within-l index l - m
// (cos part), l (m = 0), l + m (sin part) -- the reference's order
// (soap.cpp:101-216 generic Cartesian recurrence).  The diagonal advances
// four orders at a time: P_mm = (2m-1)(2m-3)(2m-5)(2m-7) (x+iy)^4 P_{m-4,m-4}.
// `ca`, `cb`, `cn` are the recurrence and normalisation coefficients indexed
// l(l+1)/2 + m.
__device__ __forceinline__ void harmonics_phase(int L, int h, double x, double y, double z, double r2,
                                                const double* __restrict__ ca, const double* __restrict__ cb,
                                                const double* __restrict__ cn, double* __restrict__ out) {
    double dr = 1.0, di = 0.0;
#pragma unroll
    for (int s = 1; s <= 3; ++s) {
        if (s <= h) {
            const double f = -(2.0 * s - 1.0);
            const double nr = f * (x * dr - y * di);
            const double ni = f * (x * di + y * dr);
            dr = nr;
            di = ni;
        }
    }
    const double wr = x * x - y * y, wi = 2.0 * x * y;
    const double ur = wr * wr - wi * wi, ui = 2.0 * wr * wi;
    for (int m = h; m <= L; m += 4) {
        if (m > h) {
            const double f = (2.0 * m - 1.0) * (2.0 * m - 3.0) * (2.0 * m - 5.0) * (2.0 * m - 7.0);
            const double nr = f * (ur * dr - ui * di);
            const double ni = f * (ur * di + ui * dr);
            dr = nr;
            di = ni;
        }
        double pr2 = dr, pi2 = di;
        {
            const double nrm = cn[m * (m + 1) / 2 + m];
            out[m * m] = nrm * pr2;                       // j = l - m = 0 (or m = 0)
            if (m > 0) out[m * m + 2 * m] = nrm * pi2;    // j = l + m
        }
        if (m < L) {
            const double c = (2.0 * m + 1.0) * z;
            double pr1 = c * dr, pi1 = c * di;
            {
                const int l = m + 1;
                const double nrm = cn[l * (l + 1) / 2 + m];
                out[l * l + 1] = nrm * pr1;
                if (m > 0) out[l * l + l + m] = nrm * pi1;
            }
            for (int l = m + 2; l <= L; ++l) {
                const int i = l * (l + 1) / 2 + m;
                const double a = ca[i] * z;
                const double b = cb[i] * r2;
                const double nr = fma(a, pr1, -b * pr2);
                const double ni = fma(a, pi1, -b * pi2);
                pr2 = pr1;
                pi2 = pi1;
                pr1 = nr;
                pi1 = ni;
                const double nrm = cn[i];
                out[l * l + l - m] = nrm * nr;
                if (m > 0) out[l * l + l + m] = nrm * ni;
            }
        }
    }
}

// Accumulator fragments of one species <-> its coefficient rows.  Element
// acc[acc_off(l) + 2b + e] of lane (g, q) is S[k = 2q + e][m = 8b + g].
template <int LMAX, bool STORE>
__device__ __forceinline__ void move_acc(double* acc, double* __restrict__ reg, int rs, int L, int n, int species,
                                         int g, int q) {
    static_for<0, LMAX + 1>([&](auto lc) {
        constexpr int l = decltype(lc)::value;
        if (l <= L) {
#pragma unroll
            for (int b = 0; b < blocks8(l); ++b) {
                const int m = 8 * b + g;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int k = 2 * q + e;
                    double* slot = reg + (species * n + k) * rs + col_off(l) + m;
                    const bool ok = m < kpad(l) && k < n;
                    if constexpr (STORE) {
                        if (ok) *slot = acc[acc_off(l) + 2 * b + e];
                    } else {
                        acc[acc_off(l) + 2 * b + e] = ok ? *slot : 0.0;
                    }
                }
            }
        }
    });
}

}  // namespace mma

// ---------------------------------------------------------------------------
// Centre kernel, fp64 tensor-core path: n_max <= 8, l_max <= LMAX.
template <int LMAX, int MINB>
__global__ void __launch_bounds__(kWarps * 32, MINB)
soap_mma_kernel(const __grid_constant__ SoapTables tab, const SoapPointers p) {
    using namespace mma;
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int S = tab.n_species, n = tab.n_max, L = tab.l_max, R = tab.rows;
    const Layout lay = layout(L, R);
    const int rs = lay.rs, ys = lay.ys;

    // CTA-shared tables.
    double* etab = reinterpret_cast<double*>(smem);
    double* ca = reinterpret_cast<double*>(smem + lay.coef_off);
    double* cb = ca + lay.tri;
    double* cn = cb + lay.tri;
    double* radial = reinterpret_cast<double*>(smem + lay.radial_off);  // [l][k][2]
    double* bt = reinterpret_cast<double*>(smem + lay.beta_off);        // [l][n][k]
    if (threadIdx.x < 32) etab[threadIdx.x] = kExp2Table[threadIdx.x];
    for (int i = threadIdx.x; i < lay.tri; i += blockDim.x) {
        ca[i] = tab.yra[i];
        cb[i] = tab.yrb[i];
        cn[i] = tab.ynorm[i];
    }
    for (int i = threadIdx.x; i < (L + 1) * 16; i += blockDim.x) radial[i] = 0.0;
    for (int i = threadIdx.x; i < (L + 1) * 64; i += blockDim.x) {
        const int l = i / 64, nn = (i / 8) % 8, k = i % 8;
        bt[i] = (nn < n && k < n) ? tab.soap_scale * p.betas[((int64_t)l * n + nn) * n + k] : 0.0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tab.items; i += blockDim.x) {
        const RadialItem it = p.items[i];
        radial[(it.l * 8 + it.k) * 2] = it.prefactor;
        radial[(it.l * 8 + it.k) * 2 + 1] = -it.exponent;
    }
    __syncthreads();
    const int64_t center = p.center_begin + (int64_t)blockIdx.x * kWarps + warp;
    if (center >= p.center_end) return;

    unsigned char* region = smem + lay.shared + (size_t)warp * lay.warp_bytes;
    int* seg_prefix = reinterpret_cast<int*>(region);
    int* seg_start = seg_prefix + 40;
    int* seg_t = seg_start + 32;
    double* qdx = reinterpret_cast<double*>(region + 512);
    double* qdy = qdx + kQueue;
    double* qdz = qdy + kQueue;
    double* qr2 = qdz + kQueue;
    int* qtype = reinterpret_cast<int*>(qr2 + kQueue);
    int* perm = qtype + kQueue;
    double* ybuf = reinterpret_cast<double*>(region + lay.y_off);
    double* reg = reinterpret_cast<double*>(region + lay.reg_off);
    const int64_t local = center - p.center_begin;

    {
        double2* z2 = reinterpret_cast<double2*>(reg);
        const int count = R * rs / 2;
        for (int i = lane; i < count; i += 32) z2[i] = make_double2(0.0, 0.0);
    }
    // Radial constants of channel (l, k = g) for every l.
    double pref[LMAX + 1], expo[LMAX + 1];
#pragma unroll
    for (int l = 0; l <= LMAX; ++l) {
        pref[l] = l <= L ? radial[(l * 8 + g) * 2] : 0.0;
        expo[l] = l <= L ? radial[(l * 8 + g) * 2 + 1] : 0.0;
    }
    constexpr int NACC = acc_off(LMAX + 1);
    double acc[NACC];

    // One species' run of `cnt` queued edges (perm[0..cnt)).
    uint64_t seen = 0;  // species whose coefficient rows already hold sums
    auto run_species = [&](int s, int cnt) {
        if ((seen >> s) & 1ull) {
            move_acc<LMAX, false>(acc, reg, rs, L, n, s, g, q);
        } else {
#pragma unroll
            for (int i = 0; i < NACC; ++i) acc[i] = 0.0;
            seen |= 1ull << s;
        }
        const double w = tab.species_weight[s];
        for (int c0 = 0; c0 < cnt; c0 += 8) {
            const int hs = c0 + (lane >> 2);
            if (hs < cnt) {
                const int e = perm[hs];
                harmonics_phase(L, lane & 3, qdx[e], qdy[e], qdz[e], qr2[e], ca, cb, cn, ybuf + (lane >> 2) * ys);
            }
            // Radial factors of both 4-edge groups first: 2 (LMAX+1)
            // independent exp() chains, no branch (padding slots weigh 0).
            double gv[2][LMAX + 1];
            bool valid[2];
#pragma unroll
            for (int grp = 0; grp < 2; ++grp) {
                const int slot = c0 + 4 * grp + q;
                valid[grp] = slot < cnt;
                const double r2 = valid[grp] ? qr2[perm[slot]] : 0.0;
                const double wv = valid[grp] ? w : 0.0;
#pragma unroll
                for (int l = 0; l <= LMAX; ++l) gv[grp][l] = wv * pref[l] * exp_nonpositive(expo[l] * r2, etab);
            }
            __syncwarp();
#pragma unroll
            for (int grp = 0; grp < 2; ++grp) {
                if (c0 + 4 * grp < cnt) {
                    const double* yrow = ybuf + (4 * grp + q) * ys;
                    static_for<0, LMAX + 1>([&](auto lc) {
                        constexpr int l = decltype(lc)::value;
                        if (l <= L) {
#pragma unroll
                            for (int b = 0; b < blocks8(l); b += 2) {
                                const int m0 = 8 * b + g;
                                const double a0 = (valid[grp] && m0 < 2 * l + 1) ? yrow[l * l + m0] : 0.0;
                                double* c = acc + acc_off(l) + 2 * b;
                                if (b + 1 < blocks8(l)) {
                                    const double a1 =
                                        (valid[grp] && m0 + 8 < 2 * l + 1) ? yrow[l * l + m0 + 8] : 0.0;
                                    dmma16(c[0], c[1], c[2], c[3], a0, a1, gv[grp][l]);
                                } else {
                                    dmma8(c[0], c[1], a0, gv[grp][l]);
                                }
                            }
                        }
                    });
                }
            }
            __syncwarp();
        }
        move_acc<LMAX, true>(acc, reg, rs, L, n, s, g, q);
        __syncwarp();
    };

    // Sort the queue by species (ballots, stable) and run each species.
    auto flush = [&](int count) {
        __syncwarp();
        int ty[3];
#pragma unroll
        for (int w = 0; w < 3; ++w) {
            const int e = 32 * w + lane;
            ty[w] = e < count ? qtype[e] : -1;
        }
        const unsigned lt = (1u << lane) - 1u;
        for (int s = 0; s < S; ++s) {
            int cnt = 0;
            int rank[3];
#pragma unroll
            for (int w = 0; w < 3; ++w) {
                const unsigned m = __ballot_sync(0xffffffffu, ty[w] == s);
                rank[w] = cnt + __popc(m & lt);
                cnt += __popc(m);
            }
            if (cnt == 0) continue;
#pragma unroll
            for (int w = 0; w < 3; ++w)
                if (ty[w] == s) perm[rank[w]] = 32 * w + lane;
            __syncwarp();
            run_species(s, cnt);
        }
        __syncwarp();
    };

    const BinView& bv = p.bins;
    const StructInfo si = bv.info[bv.struct_of[center]];
    const int wi[3] = {bv.wrap[3 * center], bv.wrap[3 * center + 1], bv.wrap[3 * center + 2]};
    int pcount = 0;
    for_each_candidate_flat(si, bv, center, lane, seg_prefix, seg_start, seg_t,
                            [&](bool valid, int j, int tx, int ty, int tz) {
        int nimg[3];
        double dx = 0.0, dy = 0.0, dz = 0.0, d2 = 0.0;
        int t = -1;
        bool ok = false;
        if (valid) {
            t = bv.type[si.atom_begin + j];
            if (t >= 0)
                ok = accept_candidate(si, bv, p.positions, center, wi, j, tx, ty, tz, tab.cutoff2, nimg, dx, dy, dz,
                                      d2);
        }
        const unsigned mask = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            const int slot = pcount + __popc(mask & ((1u << lane) - 1u));
            qdx[slot] = dx;
            qdy[slot] = dy;
            qdz[slot] = dz;
            qr2[slot] = d2;
            qtype[slot] = t;
        }
        pcount += __popc(mask);
        // The queue holds < kFlush entries between candidate rounds, so it
        // never exceeds kFlush + 31 < kQueue.
        if (pcount >= kFlush) {
            flush(pcount);
            pcount = 0;
        }
    });
    __syncwarp();
    if (pcount > 0) flush(pcount);

    beta_mma<LMAX>(bt, reg, rs, L, S, n, g, q);
    __syncwarp();
    const FeatureMap fm{S, n, L, R, tab.n_magic};
    if (tab.average == 0) {
        const int64_t row = center - p.out_row_begin;
        if (tab.out_f64)
            power_mma<LMAX>(fm, tab.power_pref, reg, rs, static_cast<double*>(p.out) + row * tab.features, g, q);
        else
            power_mma<LMAX>(fm, tab.power_pref, reg, rs, static_cast<float*>(p.out) + row * tab.features, g, q);
    } else if (tab.average == 1) {
        // Coefficient blocks in the layout the structure kernel reads:
        // [l][r][m], rows padded to 2l+2 (padding written as 0).
        double* dst = p.cbuf + local * tab.csize;
        for (int l = 0; l <= L; ++l) {
            const int pad = 2 * l + 2;
            double* dl = dst + cblock(S, n, l);
            for (int i = lane; i < R * pad; i += 32) {
                const int r = i / pad, m = i - r * pad;
                dl[i] = m < 2 * l + 1 ? reg[r * rs + col_off(l) + m] : 0.0;
            }
        }
    } else {
        power_mma<LMAX>(fm, tab.power_pref, reg, rs, p.pbuf + local * tab.features, g, q);
    }
}

}  // namespace mdsoap
