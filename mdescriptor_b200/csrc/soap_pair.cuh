// SOAP centre kernel with two warps per centre (large radial/angular bases).
//
// Same arithmetic as soap_center_kernel (soap.cuh); the difference is the
// division of labour.  A CTA of 64 threads owns one centre:
//   * the radial channels (l, k) are split between the warps: warp A owns
//     channel slot A (32 channels), warp B slots B1 and B2, so each warp keeps
//     only its own species banks in registers (about half of the one-warp
//     kernel's), which doubles the warps an SM can hold;
//   * both warps walk the candidate list (64 candidates per step) and append
//     accepted edges, warp A's then warp B's, to one shared queue;
//   * one harmonic chunk in shared memory serves both warps;
//   * the beta transform runs on 64 threads and the power spectrum splits the
//     broadcast rows r1 between the warps by parity.
// Barriers are named (id 1, 64 threads) because the two warps execute
// different template instantiations of the edge phase; every barrier is
// reached the same number of times by both, since all loop trip counts derive
// from values both warps read from shared memory.
#pragma once

#include "soap.cuh"

namespace mdsoap {

constexpr int kPairPending = 96;      // >= chunk - 1 + 64
constexpr int kPairHeader = 640;      // candidate tables, permutation, counters (bytes)

__device__ __forceinline__ void pair_barrier() { asm volatile("bar.sync 1, 64;" ::: "memory"); }

struct PairShared {
    double* etab;
    int* seg_prefix;  // 40
    int* seg_start;   // 32
    int* seg_t;       // 32
    int* perm;        // 32
    int* misc;        // [0..1] per-warp accept counts, [2] round total, [4..4+MAXT] run starts
    double *pdx, *pdy, *pdz, *pr2;
    int32_t* ptype;
    double* ybuf;
};

// Edge phase of one warp: channel slots S0 (length L0) and S1 (length L1, 0 =
// none), items[32 * slot + lane].  Fills this warp's channels of R for every
// species.
template <int MAXT, int L0, int L1, int LMAX>
__device__ __forceinline__ void pair_edge_phase(const SoapTables& tab, const SoapPointers& p, const PairShared& sh,
                                                const StructInfo& si, int64_t center, const int* wi, double* R,
                                                int warp, int lane, int slot0, int slot1) {
    const int S = tab.n_species, n = tab.n_max, H = tab.hp;
    const int chunk = tab.chunk;
    const BinView& bv = p.bins;
    const int tid = warp * 32 + lane;
    // Candidate walk geometry (identical in both warps).
    const int Mx = si.M[0], My = si.M[1], Mz = si.M[2];
    const int Kx = si.K[0], Ky = si.K[1], Kz = si.K[2];
    const int cb = bv.bin_of[center];
    const int cx = cb % Mx, cy = (cb / Mx) % My, cz = cb / (Mx * My);
    const int64_t bb = si.bin_base;
    const int64_t ab = si.atom_begin;
    const int lo = cx - Kx, hi = cx + Kx;
    const int tx0 = si.periodic ? floor_div(lo, Mx) : 0;
    const int nxs = si.periodic ? floor_div(hi, Mx) - tx0 + 1 : 1;
    const int wy = 2 * Ky + 1;
    const int entries = wy * (2 * Kz + 1) * nxs;

    for (int tb = 0; tb < S; tb += MAXT) {
        const int te = min(S, tb + MAXT);
        double pref0 = 0.0, expo0 = 0.0, pref1 = 0.0, expo1 = 0.0;
        int il0 = 0, ik0 = 0, il1 = 0, ik1 = 0;
        bool v0 = false, v1 = false;
        {
            // Slots are padded to 32 entries; padding has l = -1.
            const int i0 = 32 * slot0 + lane;
            v0 = i0 < tab.items && p.items[i0].l >= 0;
            if (v0) {
                const RadialItem it = p.items[i0];
                pref0 = it.prefactor;
                expo0 = -it.exponent;
                il0 = it.l;
                ik0 = it.k;
            }
            if (L1 > 0) {
                const int i1 = 32 * slot1 + lane;
                v1 = i1 < tab.items && p.items[i1].l >= 0;
                if (v1) {
                    const RadialItem it = p.items[i1];
                    pref1 = it.prefactor;
                    expo1 = -it.exponent;
                    il1 = it.l;
                    ik1 = it.k;
                }
            }
        }
        const double* ybase0 = sh.ybuf + il0 * (il0 + 1);
        const double* ybase1 = sh.ybuf + il1 * (il1 + 1);
        double a0[MAXT][L0];
        double a1[MAXT][L1 > 0 ? L1 : 1];
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
#pragma unroll
            for (int m = 0; m < L0; ++m) a0[t][m] = 0.0;
#pragma unroll
            for (int m = 0; m < (L1 > 0 ? L1 : 1); ++m) a1[t][m] = 0.0;
        }

        auto accumulate = [&](auto bank, double g0, double g1, int eo) {
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
        };
        auto radial = [&](int e, double w, double& g0, double& g1) {
            const double r2e = sh.pr2[e];
            g0 = w * pref0 * exp_nonpositive(expo0 * r2e, sh.etab);
            g1 = L1 > 0 ? w * pref1 * exp_nonpositive(expo1 * r2e, sh.etab) : 0.0;
        };
        // Both warps: harmonics for the chunk, species sort, then each warp
        // accumulates its own channels.
        auto process = [&](int count) {
            if (tid < count)
                harmonics_any<LMAX>(tab, sh.pdx[tid], sh.pdy[tid], sh.pdz[tid], sh.pr2[tid], sh.ybuf + tid * H);
            if (warp == 0) {
                const int mine = lane < count ? sh.ptype[lane] : MAXT;
                const unsigned lt = (1u << lane) - 1u;
                int start = 0, rank = 0;
#pragma unroll
                for (int tt = 0; tt < MAXT; ++tt) {
                    const unsigned m = __ballot_sync(0xffffffffu, mine == tt);
                    if (mine == tt) rank = start + __popc(m & lt);
                    if (lane == 0) sh.misc[4 + tt] = start;
                    start += __popc(m);
                }
                if (lane == 0) sh.misc[4 + MAXT] = start;
                if (lane < count) sh.perm[rank] = lane;
            }
            pair_barrier();
            static_for<0, MAXT>([&](auto bank) {
                constexpr int TT = decltype(bank)::value;
                const int begin = sh.misc[4 + TT], end = sh.misc[5 + TT];
                if (begin == end) return;
                const double w = tab.species_weight[tb + TT];
                int i = begin;
                for (; i + 1 < end; i += 2) {
                    const int ea = sh.perm[i], eb = sh.perm[i + 1];
                    double ga0, ga1, gb0, gb1;
                    radial(ea, w, ga0, ga1);
                    radial(eb, w, gb0, gb1);
                    accumulate(bank, ga0, ga1, ea * H);
                    accumulate(bank, gb0, gb1, eb * H);
                }
                if (i < end) {
                    const int ea = sh.perm[i];
                    double ga0, ga1;
                    radial(ea, w, ga0, ga1);
                    accumulate(bank, ga0, ga1, ea * H);
                }
            });
            pair_barrier();
        };

        int pcount = 0;
        for (int round = 0; round < entries; round += 32) {
            if (warp == 0) {
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
                        start = bv.bin_start[rowbase + b0];
                        len = bv.bin_start[rowbase + b1 + 1] - start;
                        tpack = (tx + 512) | ((ty + 512) << 10) | ((tz + 512) << 20);
                    }
                }
                int incl = len;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int up = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += up;
                }
                sh.seg_prefix[lane] = incl - len;
                sh.seg_start[lane] = start;
                sh.seg_t[lane] = tpack;
                if (lane == 31) sh.misc[2] = incl;
            }
            pair_barrier();
            const int total = sh.misc[2];
            for (int q0 = 0; q0 < total; q0 += 64) {
                const int q = q0 + tid;
                const bool cvalid = q < total;
                int i = 0;
#pragma unroll
                for (int step = 16; step > 0; step >>= 1)
                    if (sh.seg_prefix[i + step] <= q) i += step;
                const int a = sh.seg_start[i] + (q - sh.seg_prefix[i]);
                const int tp = sh.seg_t[i];
                const int j = cvalid ? bv.sorted[ab + a] : 0;
                int nimg[3];
                double dx = 0.0, dy = 0.0, dz = 0.0, d2 = 0.0;
                int t = -1;
                bool ok = false;
                if (cvalid) {
                    t = bv.type[ab + j];
                    if (t >= tb && t < te)
                        ok = accept_candidate(si, bv, p.positions, center, wi, j, (tp & 1023) - 512,
                                              ((tp >> 10) & 1023) - 512, ((tp >> 20) & 1023) - 512, tab.cutoff2,
                                              nimg, dx, dy, dz, d2);
                }
                const unsigned mask = __ballot_sync(0xffffffffu, ok);
                if (lane == 0) sh.misc[warp] = __popc(mask);
                pair_barrier();
                const int c0 = sh.misc[0], c1 = sh.misc[1];
                if (ok) {
                    const int slot = pcount + (warp == 1 ? c0 : 0) + __popc(mask & ((1u << lane) - 1u));
                    sh.pdx[slot] = dx;
                    sh.pdy[slot] = dy;
                    sh.pdz[slot] = dz;
                    sh.pr2[slot] = d2;
                    sh.ptype[slot] = t - tb;
                }
                pcount += c0 + c1;
                pair_barrier();
                // Drain whole chunks; the queue holds < chunk entries between
                // steps, so it never exceeds chunk + 63 <= kPairPending - 1.
                while (pcount >= chunk) {
                    process(chunk);
                    const int rem = pcount - chunk;
                    double sx = 0.0, sy = 0.0, sz = 0.0, sr = 0.0;
                    int st = 0;
                    if (tid < rem) {
                        sx = sh.pdx[chunk + tid];
                        sy = sh.pdy[chunk + tid];
                        sz = sh.pdz[chunk + tid];
                        sr = sh.pr2[chunk + tid];
                        st = sh.ptype[chunk + tid];
                    }
                    pair_barrier();
                    if (tid < rem) {
                        sh.pdx[tid] = sx;
                        sh.pdy[tid] = sy;
                        sh.pdz[tid] = sz;
                        sh.pr2[tid] = sr;
                        sh.ptype[tid] = st;
                    }
                    pair_barrier();
                    pcount = rem;
                }
            }
            pair_barrier();
        }
        if (pcount > 0) process(pcount);

        // Flush this warp's channels: R[l][t][k][m], rows padded to 2l+2.
#pragma unroll
        for (int tt = 0; tt < MAXT; ++tt) {
            const int t = tb + tt;
            if (t < te) {
                if (v0) {
                    const int len = 2 * il0 + 1;
                    double* dst = R + cblock(S, n, il0) + (t * n + ik0) * (len + 1);
#pragma unroll
                    for (int m = 0; m < L0; ++m)
                        if (m < len) dst[m] = a0[tt][m];
                }
                if (L1 > 0 && v1) {
                    const int len = 2 * il1 + 1;
                    double* dst = R + cblock(S, n, il1) + (t * n + ik1) * (len + 1);
#pragma unroll
                    for (int m = 0; m < (L1 > 0 ? L1 : 1); ++m)
                        if (m < len) dst[m] = a1[tt][m];
                }
            }
        }
        pair_barrier();
    }
}

// Template parameters: MAXT species banks per pass; LA = slot A length (warp
// A); LB1, LB2 = slot lengths of warp B (LB2 may be 0); NMAX >= n_max; LMAX
// >= l_max; MINB resident CTAs per SM for the register budget.
template <int MAXT, int LA, int LB1, int LB2, int NMAX, int LMAX, int MINB>
__global__ void __launch_bounds__(64, MINB)
soap_pair_kernel(const __grid_constant__ SoapTables tab, const SoapPointers p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t center = p.center_begin + blockIdx.x;
    if (center >= p.center_end) return;  // uniform for the CTA
    PairShared sh;
    sh.etab = reinterpret_cast<double*>(smem);
    if (threadIdx.x < 32) sh.etab[threadIdx.x] = kExp2Table[threadIdx.x];
    int* header = reinterpret_cast<int*>(smem + 256);
    sh.seg_prefix = header;
    sh.seg_start = header + 40;
    sh.seg_t = header + 72;
    sh.perm = header + 104;
    sh.misc = header + 136;
    unsigned char* queue = smem + 256 + kPairHeader;
    sh.pdx = reinterpret_cast<double*>(queue);
    sh.pdy = sh.pdx + kPairPending;
    sh.pdz = sh.pdy + kPairPending;
    sh.pr2 = sh.pdz + kPairPending;
    sh.ptype = reinterpret_cast<int32_t*>(sh.pr2 + kPairPending);
    sh.ybuf = reinterpret_cast<double*>(queue + kPairPending * 36);
    const int64_t local = center - p.center_begin;
    double* R = tab.r_global ? p.rbuf + local * tab.csize : reinterpret_cast<double*>(queue + tab.r_offset);
    const BinView& bv = p.bins;
    const StructInfo si = bv.info[bv.struct_of[center]];
    const int wi[3] = {bv.wrap[3 * center], bv.wrap[3 * center + 1], bv.wrap[3 * center + 2]};
    pair_barrier();
    if (warp == 0)
        pair_edge_phase<MAXT, LA, 0, LMAX>(tab, p, sh, si, center, wi, R, warp, lane, 0, 0);
    else
        pair_edge_phase<MAXT, LB1, LB2, LMAX>(tab, p, sh, si, center, wi, R, warp, lane, 1, 2);
    // R complete (the edge phase ends with a barrier).
    beta_transform_warp<NMAX>(tab, p.betas, R, threadIdx.x, 64);
    pair_barrier();
    if (tab.average == 0) {
        const int64_t row = center - p.out_row_begin;
        if (tab.out_f64)
            power_spectrum_warp<LMAX>(tab, R, static_cast<double*>(p.out) + row * tab.features, lane, warp, 2);
        else
            power_spectrum_warp<LMAX>(tab, R, static_cast<float*>(p.out) + row * tab.features, lane, warp, 2);
    } else if (tab.average == 1) {
        double* dst = p.cbuf + local * tab.csize;
        for (int i = threadIdx.x; i < tab.csize; i += 64) dst[i] = R[i];
    } else {
        power_spectrum_warp<LMAX>(tab, R, p.pbuf + local * tab.features, lane, warp, 2);
    }
}

}  // namespace mdsoap
