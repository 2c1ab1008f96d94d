// SOAP centre kernel with paired radial channels (sm_100a, IEEE fp64).
//
// Same arithmetic as soap_center_kernel (soap.cuh, reference
// cpp/src/standalone/soap.cpp:598-1017); three things differ:
//
//   * Channel pairs.  With l_max = L compile-time, the (L+1) degrees of one
//     radial index k are grouped as {L}, {L-1, 0}, {L-2, 1}, ...: every group
//     holds at most 2L+1 harmonic components, and lane (g, k) owns group g of
//     radial index k for every species.  A lane therefore keeps 2L+1
//     accumulators per species (13 for L = 6, against 13 + 5 when channels
//     are dealt out by degree) and evaluates two radial factors per edge.
//     The harmonic row of an edge is stored group by group ("views"), so a
//     lane reads its components as one contiguous run; the component m of a
//     lane belongs to the first channel below the split 2 l_A + 1 and to the
//     second above it, and since every split is odd, each pair of components
//     (2p+1, 2p+2) above the smallest split picks its radial factor with one
//     select per edge.
//   * Prefiltered walk.  The binning kernel stores every atom's wrapped
//     position and species in bin order (BinView::spos).  A candidate is
//     first tested on those (one coalesced 32-byte load, six fp64 operations,
//     against the structure's pre_cut2 = (cutoff + margin)^2, the margin four
//     orders above any rounding difference); survivors are compacted and
//     tested exactly by accept_candidate (the reference's own arithmetic) 32
//     at a time, so the pair set and the displacement bits stay those of the
//     reference graph.
//   * Radial factors by scaled_exp (prefactor folded, 2^m through the
//     exponent field); species weights multiply the raw sums once, at the
//     flush, instead of every edge.
//
// Plans whose tail runs as a kernel of its own (SPLIT) take the walk and the
// expansion as two instantiations (MODE 1 and 2 below) over per-centre edge
// lists in HBM: the walk needs no accumulators and the expansion no walk
// state, so each keeps more warps resident than the one-kernel form.
//
// The coefficient block layout, the beta transform and the power spectrum on
// the fp64 tensor cores are dmma.cuh's, as in soap_center_kernel.
#pragma once

#include "bulk_copy.cuh"
#include "soap.cuh"

namespace mdsoap {

namespace paired {

template <int L>
struct Layout {
    static constexpr int G = 1 + (L + 1) / 2;  // channel groups per radial index
    static constexpr int W = 2 * L + 1;        // accumulators per species per lane
    static constexpr int VS = W + 1;           // view stride (even: 16-byte loads)
    // Harmonic row of one edge (doubles): G views, padded to = 2 (mod 4) so
    // that the lane-per-edge row writes spread over 8 bank pairs.
    static constexpr int ROW = G * VS + ((2 - (G * VS) % 4) + 4) % 4;
    __host__ __device__ static constexpr int la(int g) { return g == 0 ? L : L - g; }
    __host__ __device__ static constexpr int lb(int g) { return (g == 0 || g - 1 >= L - g) ? -1 : g - 1; }
    static constexpr int LAMIN = la(G - 1);    // smallest first-channel degree
    static constexpr int NSEL = L - LAMIN;     // radial-factor selects per edge
    // Offset of harmonic component j of degree l in the row.
    __host__ __device__ static constexpr int pos(int l, int j) {
        for (int g = 0; g < G; ++g) {
            if (la(g) == l) return g * VS + j;
            if (lb(g) == l) return g * VS + 2 * la(g) + 1 + j;
        }
        return 0;
    }
};

// Per-warp shared-memory region (bytes); the harmonic rows follow.
constexpr int kSegBytes = 544;                     // seg_prefix[40] seg_start[32] seg_t[32], 128 B spare
constexpr int kSegOffBytes = 3 * 32 * 8;           // per-segment offset vectors
constexpr int kPreQueue = 96;                      // prefilter survivors awaiting the exact test
constexpr int kPreBytes = 3 * kPreQueue * 4;
// Accepted-edge queue: below chunk (<= 32) entries before a prefilter round,
// which may append 64 direct edges (float32 plans), or before an exact test
// (32 more).
constexpr int kPendingPaired = 96;
constexpr int kEdgeBytes = kPendingPaired * (5 * 8 + 4); // dx dy dz r2 weight + species
constexpr int kSortBytes = 32 * 2 * 8;             // r2 and weight of a chunk's edges in bank order
constexpr int kHeaderBytes = kSegBytes + kSegOffBytes + kPreBytes + kEdgeBytes + kSortBytes;
static_assert(kHeaderBytes % 16 == 0, "harmonic rows must start 16-byte aligned");
// The expansion-only kernel (MODE 2) has no walk: its region starts with an
// edge queue of 64 (below chunk <= 32 entries before a fetch of 32 more).
constexpr int kPendingExpand = 64;
constexpr int kHeaderBytesExpand = kPendingExpand * (5 * 8 + 4) + kSortBytes;
static_assert(kHeaderBytesExpand % 16 == 0, "harmonic rows must start 16-byte aligned");
__host__ __device__ constexpr int header_bytes(int mode) { return mode == 2 ? kHeaderBytesExpand : kHeaderBytes; }
// Exp table of the expansion-only kernel's float32 rows (scaled_exp_folded).
constexpr int kFoldT = 64;
// CTA shared memory the exp table takes (the kernel's first bytes).
__host__ __device__ constexpr int exp_table_bytes(int mode, bool precise) {
    return (mode == 2 && !precise && kFoldT == 64) ? 512 : 256;
}

// Real regular solid harmonics of one displacement into the paired row
// (soap.cpp:101-216, generic Cartesian recurrence; within a degree, j = l - m
// is the cos part, j = l (m = 0), j = l + m the sin part).
// Every loop index is a compile-time constant, so each row offset is one.
template <int L>
__device__ __forceinline__ void harmonics_row(const SoapTables& tab, double x, double y, double z, double r2,
                                              double* __restrict__ out) {
    using P = Layout<L>;
    double dr = 1.0, di = 0.0;
    static_for<0, L + 1>([&](auto mc) {
        constexpr int m = decltype(mc)::value;
        if constexpr (m > 0) {
            const double f = -(2.0 * m - 1.0);
            const double nr = f * fma(x, dr, -__dmul_rn(y, di));
            const double ni = f * fma(x, di, __dmul_rn(y, dr));
            dr = nr;
            di = ni;
        }
        double pr2 = dr, pi2 = di;
        constexpr int id = m * (m + 1) / 2 + m;
        if constexpr (m == 0) {
            out[P::pos(0, 0)] = tab.ynorm[0] * pr2;
        } else {
            constexpr int o1 = P::pos(m, 0), o2 = P::pos(m, 2 * m);
            out[o1] = tab.ynorm[id] * pr2;
            out[o2] = tab.ynorm[id] * pi2;
        }
        if constexpr (m < L) {
            const double c = (2.0 * m + 1.0) * z;
            double pr1 = c * dr, pi1 = c * di;
            {
                constexpr int l = m + 1;
                constexpr int i = l * (l + 1) / 2 + m;
                constexpr int o1 = P::pos(l, l - m), o2 = P::pos(l, l + m);
                out[o1] = tab.ynorm[i] * pr1;
                if constexpr (m > 0) out[o2] = tab.ynorm[i] * pi1;
            }
            static_for<m + 2, L + 1>([&](auto lc) {
                constexpr int l = decltype(lc)::value;
                constexpr int i = l * (l + 1) / 2 + m;
                constexpr int o1 = P::pos(l, l - m), o2 = P::pos(l, l + m);
                const double a = tab.yra[i] * z;
                const double b = tab.yrb[i] * r2;
                const double nr = fma(a, pr1, -b * pr2);
                const double ni = fma(a, pi1, -b * pi2);
                pr2 = pr1;
                pi2 = pi1;
                pr1 = nr;
                pi1 = ni;
                out[o1] = tab.ynorm[i] * nr;
                if constexpr (m > 0) out[o2] = tab.ynorm[i] * ni;
            });
        }
    });
}

}  // namespace paired

// Beta transform and power spectrum (or the inner-average block copy) of one
// centre from its raw-sum block R in shared memory, one warp: the tail for
// plans whose coefficients do not stay in registers (n_max < 8, more species
// than register banks, average inner, compression through power_generic).
// Used by the fused paired kernel and by soap_tail_generic_kernel.
template <int L>
__device__ __forceinline__ void tail_generic(const SoapTables& tab, const SoapPointers& p, double* R,
                                             const double* bt, int64_t center, int lane) {
    const int S = tab.coef_species, n = tab.n_max;
    const int gq = lane >> 2, qq = lane & 3, R_rows = tab.rows;
    const bool n8 = n == 8;
    const int64_t local = center - p.center_begin;
    if (n8)
        mma::beta_n8<L>(bt, R, tab.rs, S, gq, qq);
    else
        mma::beta_mma<L>(bt, R, tab.rs, L, S, n, gq, qq);
    __syncwarp();
    const mma::FeatureMap fm{S, n, L, R_rows, tab.n_magic};
    if (tab.average != 1 && (tab.compression == 2 || tab.compression == 3)) {
        const int rs = tab.rs;
        auto coef = [&](int t, int k, int l, int m) { return R[(t * n + k) * rs + mma::col_off(l) + m]; };
        if (tab.average == 0) {
            const int64_t row = center - p.out_row_begin;
            if (tab.out_f64)
                power_generic(coef, tab.power_pref, S, n, L, tab.compression,
                              static_cast<double*>(p.out) + row * tab.features, lane);
            else
                power_generic(coef, tab.power_pref, S, n, L, tab.compression,
                              static_cast<float*>(p.out) + row * tab.features, lane);
        } else {
            power_generic(coef, tab.power_pref, S, n, L, tab.compression, p.pbuf + local * tab.features, lane);
        }
        return;
    }
    if (tab.average == 0) {
        const int64_t row = center - p.out_row_begin;
        if (tab.out_f64) {
            double* dst = static_cast<double*>(p.out) + row * tab.features;
            if (n8)
                mma::power_n8<L>(tab.power_pref, R, tab.rs, S, dst, gq, qq);
            else
                mma::power_mma<L>(fm, tab.power_pref, R, tab.rs, dst, gq, qq);
        } else {
            float* dst = static_cast<float*>(p.out) + row * tab.features;
            if (n8)
                mma::power_n8<L>(tab.power_pref, R, tab.rs, S, dst, gq, qq);
            else
                mma::power_mma<L>(fm, tab.power_pref, R, tab.rs, dst, gq, qq);
        }
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
        if (n8)
            mma::power_n8<L>(tab.power_pref, R, tab.rs, S, p.pbuf + local * tab.features, gq, qq);
        else
            mma::power_mma<L>(fm, tab.power_pref, R, tab.rs, p.pbuf + local * tab.features, gq, qq);
    }
}

// One warp per centre.  MAXT species register banks per pass over the
// neighbourhood; L = l_max exactly; PRECISE selects the radial-factor
// accuracy (float64 rows need the full one); MINB resident CTAs per SM.
// SPLIT: the kernel ends after the flush, handing the raw sums to
// soap_tail_kernel (no tail code, so fewer registers).
// POLY: polynomial radial basis (soap.cpp:450-492, 805-857): per edge, the
// warp evaluates the modified-Bessel overlaps flir_l(r, q) on the quadrature
// nodes (lanes over nodes, the reference's recurrence and operation order,
// its clamp at 0), and each lane projects its two channels onto the weighted
// basis: g_ln = 4 pi r^-l sum_q flir_l(r, q) wv[q][n] (4 pi at l = 0 for the
// exact self pair).  The accumulation and the tail are the GTO path's, with
// beta = identity and no pi^{3/2} (the plan uploads those).
// MODE (edge-list split of the SPLIT path, for plans with tab.edge_cap > 0):
//   0  walk and expansion in one kernel; when p.edge_count is set, only the
//      centres whose accepted edges overflowed their slot (count > edge_cap);
//   1  walk only: each centre's accepted edges, in walk order, go to its
//      slot of p.edges / p.edge_info (species | exact-self flag << 16) and
//      their number to p.edge_count;
//   2  expansion only: the edges come from the slots MODE 1 filled (centres
//      with an overflowed slot are left to MODE 0).
// The edges reach the expansion in the same order either way, so the three
// give the same rows bit for bit.
template <int MAXT, int L, bool PRECISE, int MINB, bool SPLIT = false, bool POLY = false, int MODE = 0>
__global__ void __launch_bounds__(kWarps * 32, MINB)
soap_paired_kernel(const __grid_constant__ SoapTables tab, const SoapPointers p) {
    using P = paired::Layout<L>;
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // S: species of the coefficient block (1 when mu2 pools them all).
    const int S = tab.coef_species, n = tab.n_max;
    const bool pooled = tab.compression == 1;
    // CTA-shared: exp table (32 doubles), then beta as [l][n][k] scaled by
    // pi^{3/2} and zero padded to 8 x 8.
    // The expansion-only kernel's float32 rows use scaled_exp_folded<kFoldT>
    // (a table of kFoldT entries); everything else the 32-entry table.
    constexpr bool kFolded = MODE == 2 && !PRECISE && !POLY;
    double* etab = reinterpret_cast<double*>(smem);
    if constexpr (kFolded && paired::kFoldT == 64) {
        for (int i = threadIdx.x; i < 64; i += blockDim.x) etab[i] = kExp2Table64[i];
    } else {
        if (threadIdx.x < 32) etab[threadIdx.x] = kExp2Table[threadIdx.x];
    }
    double* bt = reinterpret_cast<double*>(smem + 256);
    if (!SPLIT)
        for (int i = threadIdx.x; i < (L + 1) * 64; i += blockDim.x) {
            const int l = i / 64, nn = (i / 8) % 8, k = i % 8;
            bt[i] = (nn < n && k < n) ? tab.soap_scale * p.betas[((int64_t)l * n + nn) * n + k] : 0.0;
        }
    // POLY: nodes [Q] and weighted values [Q][8] (zero beyond n_max) after beta.
    const int Q = POLY ? tab.grid_size : 0;
    double* qnodes = bt + (L + 1) * 64;
    double* qwv = qnodes + Q;
    if (POLY) {
        for (int i = threadIdx.x; i < Q; i += blockDim.x) qnodes[i] = p.poly[i];
        for (int i = threadIdx.x; i < Q * 8; i += blockDim.x) {
            const int qq = i / 8, nn = i % 8;
            qwv[i] = nn < n ? p.poly[Q + qq * n + nn] : 0.0;
        }
    }
    // The expansion-only kernel keeps no beta table (its tail runs as a kernel of its own).
    const int kShared = paired::exp_table_bytes(MODE, PRECISE) + (MODE == 2 ? 0 : (L + 1) * 64 * 8) +
                        (POLY ? ((Q * 9 * 8 + 15) & ~15) : 0);
    __syncthreads();

    unsigned char* region = smem + kShared + (size_t)warp * tab.warp_bytes;
    int* seg_prefix = reinterpret_cast<int*>(region);  // 40
    int* seg_start = seg_prefix + 40;                   // 32
    int* seg_t = seg_start + 32;                        // 32
    double* seg_off = reinterpret_cast<double*>(region + paired::kSegBytes);  // [3][32]
    int* qa = reinterpret_cast<int*>(region + paired::kSegBytes + paired::kSegOffBytes);
    int* qt = qa + paired::kPreQueue;
    int* qs = qt + paired::kPreQueue;
    constexpr int kPend = MODE == 2 ? paired::kPendingExpand : paired::kPendingPaired;
    constexpr int kHead = paired::header_bytes(MODE);
    double* pdx = reinterpret_cast<double*>(
        region + (MODE == 2 ? 0 : paired::kSegBytes + paired::kSegOffBytes + paired::kPreBytes));
    double* pdy = pdx + kPend;
    double* pdz = pdy + kPend;
    double* pr2 = pdz + kPend;
    double* pw = pr2 + kPend;
    int32_t* ptype = reinterpret_cast<int32_t*>(pw + kPend);
    double* sr2 = reinterpret_cast<double*>(region + kHead - paired::kSortBytes);
    double* sw = sr2 + 32;
    double* ybuf = reinterpret_cast<double*>(region + kHead);
    // POLY: flir_l(r, q) of the current edge, [L+1][Q], after the harmonic rows.
    double* flir = ybuf + tab.chunk * P::ROW;
    // Centres: CTA b owns the contiguous range [c_lo, c_hi) of this launch
    // and its warps stride through it, so the CTA's centres share a few
    // structures whose bins, positions and sorted positions stay in L1.  A
    // grid of resident CTAs makes the kernel persistent; a grid of one CTA
    // per kWarps centres gives every warp one centre.
    const int64_t total_centres = p.grid_end - p.grid_begin;
    const int64_t per_cta = (total_centres + gridDim.x - 1) / gridDim.x;
    const int64_t c_lo = p.grid_begin + (int64_t)blockIdx.x * per_cta;
    const int64_t c_hi = min(p.grid_end, c_lo + per_cta);
    auto run_centre = [&](const int64_t center) {
    __syncwarp();  // the previous centre's tail reads are done before the walk reuses the region
    const int64_t slot = center - p.grid_begin;  // edge-list slot of this centre
    int nedges = 0;                              // MODE 2: accepted edges in the slot
    if constexpr (MODE == 0) {
        if (p.edge_count && p.edge_count[slot] <= tab.edge_cap) return;
    } else if constexpr (MODE == 2) {
        nedges = p.edge_count[slot];
        if (nedges > tab.edge_cap) return;
    }
    const int64_t local = center - p.center_begin;
    double* R = tab.r_global ? p.rbuf + (center - p.grid_begin) * tab.rsize
                             : reinterpret_cast<double*>(region + tab.r_offset);

    const BinView& bv = p.bins;
    const StructInfo& si = bv.info[bv.struct_of[center]];
    const int wi[3] = {bv.wrap[3 * center], bv.wrap[3 * center + 1], bv.wrap[3 * center + 2]};
    double wpos[3];
    wrapped_position(si, p.positions + 3 * center, bv.wrap + 3 * center, wpos);
    const int chunk = MODE == 1 ? 32 : tab.chunk;
    // Beta transform and power spectrum in registers (n_max == 8, the whole
    // coefficient block in one pass of banks, per-centre rows).
    // Split sums (PRECISE instantiations, i.e. float64 rows): each species'
    // neighbour sum is kept as two partial sums over alternate accepted
    // edges, in two register banks, added at the flush -- half-length sums,
    // as the reference's two-lane SIMD reduction forms them
    // (soap.cpp:905-912); a pass then holds MAXT / 2 species.
    constexpr int ks = PRECISE ? 2 : 1;
    constexpr int spp = MAXT / ks;
    const bool regs_tail = n == 8 && S * ks <= MAXT && tab.average != 1;

    // This lane's channel pair: group g of radial index k.
    // kPair (expansion-only kernel, float32 rows, n_max even): the two half
    // warps take alternate edges of a run, and lane (g, kp) of a half owns
    // radial indices kp and kp + n/2 of group g -- each harmonic view it
    // loads serves two channels, half the shared-memory loads per edge.  The
    // halves' sums are added at the flush, where half h writes row kp + h n/2.
    constexpr bool kPair = MODE == 2 && !PRECISE && !POLY && MAXT == 1;
    const int nh = kPair ? max(n >> 1, 1) : n;
    const int g = kPair ? (lane & 15) / nh : lane / n;
    const int kp = kPair ? (lane & 15) - g * nh : lane - g * n;  // first radial index
    const int k = kPair ? kp + (lane >> 4) * nh : kp;            // radial index of the flushed row
    const bool lane_on = g < P::G;
    const int lA = lane_on ? (g == 0 ? L : L - g) : 0;
    const int lB = (lane_on && g > 0 && g - 1 < L - g) ? g - 1 : -1;
    const int split = 2 * lA + 1;
    double prefA = 0.0, nEA = 0.0, prefB = 0.0, nEB = 0.0;
    double prefA1 = 0.0, nEA1 = 0.0, prefB1 = 0.0, nEB1 = 0.0;  // kPair: radial index kp + n/2
    if (lane_on) {
        const RadialItem a = p.items[(L - lA) * n + kp];  // items are sorted by l descending
        prefA = a.prefactor;
        nEA = -a.exponent;
        if (lB >= 0) {
            const RadialItem b = p.items[(L - lB) * n + kp];
            prefB = b.prefactor;
            nEB = -b.exponent;
        }
        if (kPair) {
            const RadialItem a1 = p.items[(L - lA) * n + kp + nh];
            prefA1 = a1.prefactor;
            nEA1 = -a1.exponent;
            if (lB >= 0) {
                const RadialItem b1 = p.items[(L - lB) * n + kp + nh];
                prefB1 = b1.prefactor;
                nEB1 = -b1.exponent;
            }
        }
    }
    bool first_above[P::NSEL > 0 ? P::NSEL : 1];
#pragma unroll
    for (int q = 0; q < P::NSEL; ++q) first_above[q] = lA > P::LAMIN + q;
    const int view = lane_on ? g * P::VS : 0;

    // Candidate walk geometry.
    const int Mx = si.M[0], My = si.M[1], Mz = si.M[2];
    const int Kx = si.K[0], Ky = si.K[1], Kz = si.K[2];
    const int periodic = si.periodic;
    const int cb = bv.bin_of[center];
    const int cx = cb % Mx, cy = (cb / Mx) % My, cz = cb / (Mx * My);
    const int64_t bb = si.bin_base;
    const int64_t ab = si.atom_begin;
    const int xlo = cx - Kx, xhi = cx + Kx;
    const int tx0 = periodic ? floor_div(xlo, Mx) : 0;
    const int nxs = periodic ? floor_div(xhi, Mx) - tx0 + 1 : 1;
    const int wy = 2 * Ky + 1;
    const int entries = wy * (2 * Kz + 1) * nxs;
    const double pre2 = si.pre_cut2, in2 = si.in_cut2;

    // The walk-only kernel takes every species in one pass.
    const int pass_species = MODE == 1 ? max(S, 1) : spp;
    int written = 0;  // MODE 1: accepted edges of this centre so far
    for (int tb = 0; tb < S; tb += pass_species) {
        const int te = min(S, tb + pass_species);
        // kPair: acc[0] radial index kp, acc[1] kp + n/2.
        double acc[kPair ? 2 : MAXT][P::W];
#pragma unroll
        for (int t = 0; t < (kPair ? 2 : MAXT); ++t)
#pragma unroll
            for (int m = 0; m < P::W; ++m) acc[t][m] = 0.0;

        // One edge into bank TT.
        auto accumulate = [&](auto bank, double gA, double gB, int e) {
            constexpr int TT = decltype(bank)::value;
            double gs[P::NSEL > 0 ? P::NSEL : 1];
#pragma unroll
            for (int q = 0; q < P::NSEL; ++q) gs[q] = first_above[q] ? gA : gB;
            const double2* yv = reinterpret_cast<const double2*>(ybuf + e * P::ROW + view);
#pragma unroll
            for (int mm = 0; mm < (P::W + 1) / 2; ++mm) {
                const double2 y = yv[mm];
                const int m0 = 2 * mm, m1 = 2 * mm + 1;
                const double g0 = m0 < 2 * P::LAMIN + 1 ? gA : gs[(m0 - 1) / 2 - P::LAMIN];
                acc[TT][m0] = fma(g0, y.x, acc[TT][m0]);
                if (m1 < P::W) {
                    const double g1 = m1 < 2 * P::LAMIN + 1 ? gA : gs[(m1 - 1) / 2 - P::LAMIN];
                    acc[TT][m1] = fma(g1, y.y, acc[TT][m1]);
                }
            }
        };
        // POLY: radial factors of the lane's two channels for one edge (d2 = r^2).
        auto poly_radial = [&](double d2, double& gA, double& gB) {
            const double r = sqrt(d2);
            const double eta = tab.eta;
            __syncwarp();
            for (int q = lane; q < Q; q += 32) {
                const double x = qnodes[q];
                if (r <= 1e-14) {
                    flir[q] = exp_nonpositive(__dmul_rn(__dmul_rn(-eta, x), x), etab);
                    for (int l = 1; l <= L; ++l) flir[l * Q + q] = 0.0;
                    continue;
                }
                // polynomial_flir, soap.cpp:470-489 (operation order kept, no contraction).
                const double pre = __ddiv_rn(0.25, __dmul_rn(__dmul_rn(eta, r), x));
                const double dm = __dsub_rn(x, r), dp = __dadd_rn(x, r);
                const double minus = exp_nonpositive(__dmul_rn(__dmul_rn(-eta, dm), dm), etab);
                const double plus = exp_nonpositive(__dmul_rn(__dmul_rn(-eta, dp), dp), etab);
                double v2 = __dmul_rn(pre, __dsub_rn(minus, plus));
                flir[q] = v2;
                if (L >= 1) {
                    double v1 = __dmul_rn(pre, __dsub_rn(__dadd_rn(minus, plus), __dmul_rn(2.0, v2)));
                    flir[Q + q] = v1;
#pragma unroll
                    for (int l = 2; l <= L; ++l) {
                        const double v = fmax(0.0, __dsub_rn(v2, __dmul_rn(__dmul_rn(pre, 4.0 * l - 2.0), v1)));
                        flir[l * Q + q] = v;
                        v2 = v1;
                        v1 = v;
                    }
                }
            }
            __syncwarp();
            double sa = 0.0, sb = 0.0;
            const double* fa = flir + lA * Q;
            const double* fb = flir + (lB >= 0 ? lB : 0) * Q;
            for (int q = 0; q < Q; ++q) {
                const double w = qwv[q * 8 + k];
                sa = fma(fa[q], w, sa);
                sb = fma(fb[q], w, sb);
            }
            // scale 4 pi r^-l (soap.cpp:811-818): r^-l as the reference's running product.
            constexpr double kFourPi = 12.566370614359172953850573533118;
            const double inv = r <= 1e-14 ? 0.0 : 1.0 / r;
            double pa = 1.0, pb = 1.0;
            for (int l = 0; l < lA; ++l) pa *= inv;
            for (int l = 0; l < (lB >= 0 ? lB : 0); ++l) pb *= inv;
            const double scale_a = r <= 1e-14 ? (lA == 0 ? kFourPi : 0.0) : kFourPi * pa;
            const double scale_b = r <= 1e-14 ? (lB == 0 ? kFourPi : 0.0) : kFourPi * pb;
            gA = lane_on ? scale_a * sa : 0.0;
            gB = (lane_on && lB >= 0) ? scale_b * sb : 0.0;
        };

        auto process = [&](int count) {
            // (The walk-only kernel never queues: its accepted edges go
            // straight to the centre's slot, beyond edge_cap only counted.)
            // Stable counting sort of the chunk by species bank; each edge's
            // harmonic row, r^2 and weight go to its rank, so a bank's edges
            // are consecutive rows.
            const int mine = lane < count ? ptype[lane] : MAXT;
            const unsigned lt = (1u << lane) - 1u;
            int run_start[MAXT + 1];
            run_start[0] = 0;
            int rank = 0;
#pragma unroll
            for (int tt = 0; tt < MAXT; ++tt) {
                const unsigned msk = __ballot_sync(0xffffffffu, mine == tt);
                if (mine == tt) rank = run_start[tt] + __popc(msk & lt);
                run_start[tt + 1] = run_start[tt] + __popc(msk);
            }
            if (lane < count) {
                paired::harmonics_row<L>(tab, pdx[lane], pdy[lane], pdz[lane], pr2[lane], ybuf + rank * P::ROW);
                sr2[rank] = pr2[lane];
                sw[rank] = pw[lane];
            }
            __syncwarp();
            const bool weighted = tab.weighted != 0;
            if constexpr (kPair) {
                // Two edges per step, one per half warp (one species, one bank).
                const int half = lane >> 4;
                constexpr double fs = folded_scale(paired::kFoldT);
                const double sA0 = nEA * fs, sB0 = nEB * fs, sA1 = nEA1 * fs, sB1 = nEB1 * fs;
                for (int ea = 0; ea < count; ea += 2) {
                    const bool live = ea + half < count;
                    const int e = live ? ea + half : count - 1;
                    const double u = sr2[e];
                    double gA0 = scaled_exp_folded<paired::kFoldT>(u, sA0, prefA, etab);
                    double gB0 = scaled_exp_folded<paired::kFoldT>(u, sB0, prefB, etab);
                    double gA1 = scaled_exp_folded<paired::kFoldT>(u, sA1, prefA1, etab);
                    double gB1 = scaled_exp_folded<paired::kFoldT>(u, sB1, prefB1, etab);
                    if (weighted) {
                        const double w = sw[e];
                        gA0 *= w;
                        gB0 *= w;
                        gA1 *= w;
                        gB1 *= w;
                    }
                    if (!live) gA0 = gB0 = gA1 = gB1 = 0.0;
                    double gs0[P::NSEL > 0 ? P::NSEL : 1], gs1[P::NSEL > 0 ? P::NSEL : 1];
#pragma unroll
                    for (int q = 0; q < P::NSEL; ++q) {
                        gs0[q] = first_above[q] ? gA0 : gB0;
                        gs1[q] = first_above[q] ? gA1 : gB1;
                    }
                    const double2* yv = reinterpret_cast<const double2*>(ybuf + e * P::ROW + view);
#pragma unroll
                    for (int mm = 0; mm < (P::W + 1) / 2; ++mm) {
                        const double2 y = yv[mm];
                        const int m0 = 2 * mm, m1 = 2 * mm + 1;
                        const bool a0 = m0 < 2 * P::LAMIN + 1, a1 = m1 < 2 * P::LAMIN + 1;
                        acc[0][m0] = fma(a0 ? gA0 : gs0[(m0 - 1) / 2 - P::LAMIN], y.x, acc[0][m0]);
                        acc[1][m0] = fma(a0 ? gA1 : gs1[(m0 - 1) / 2 - P::LAMIN], y.x, acc[1][m0]);
                        if (m1 < P::W) {
                            acc[0][m1] = fma(a1 ? gA0 : gs0[(m1 - 1) / 2 - P::LAMIN], y.y, acc[0][m1]);
                            acc[1][m1] = fma(a1 ? gA1 : gs1[(m1 - 1) / 2 - P::LAMIN], y.y, acc[1][m1]);
                        }
                    }
                }
                __syncwarp();
                return;
            }
            // One edge per step: two independent exp chains per lane are
            // enough to cover their latency, and the shorter loop body (one
            // copy per species bank) stays in the instruction cache.
            static_for<0, MAXT>([&](auto bank) {
                constexpr int TT = decltype(bank)::value;
                const int end = run_start[TT + 1];
                for (int ea = run_start[TT]; ea < end; ++ea) {
                    const double ua = sr2[ea];
                    double gAa, gBa;
                    if constexpr (POLY) {
                        poly_radial(ua, gAa, gBa);
                    } else {
                        gAa = scaled_exp<PRECISE>(nEA * ua, prefA, etab);
                        gBa = scaled_exp<PRECISE>(nEB * ua, prefB, etab);
                    }
                    if (weighted) {
                        const double wa = sw[ea];
                        gAa *= wa;
                        gBa *= wa;
                    }
                    accumulate(bank, gAa, gBa, ea);
                }
            });
            __syncwarp();
        };

        // The walk runs as one flat loop in which each stage has a single
        // call site (the hot code is then inlined once, which keeps it in the
        // instruction cache).  Every step takes the first applicable action:
        //   1. a full chunk of accepted edges (or the last edges) -> process;
        //   2. 32 prefilter survivors (or the last ones) -> exact test;
        //   3. candidates left in this round -> prefilter 32 of them;
        //   4. segments left -> set up the next round of 32 segments;
        //   5. otherwise done.
        // Stage 1 runs whenever pcount >= chunk, so stage 2 starts with
        // pcount < chunk and the edge queue never exceeds chunk + 31 <= 63 <
        // kPending; likewise stage 2 runs whenever qn >= 32, so stage 3 (64
        // candidates, two per lane) leaves at most 95 < kPreQueue survivors.
        int qn = 0;      // prefilter survivors queued (warp-uniform)
        int pcount = 0;  // accepted edges queued (warp-uniform)
        int naccepted = 0;  // accepted edges of this pass so far (split sums: bank parity)
        int round = 0;   // next segment index
        int q0 = 0, total = 0;
        int fetched = 0;  // MODE 2: edges of the slot read so far
        int seg_first = 0x7fffffff;  // first candidate of non-empty segment `lane` of this round
        // MODE 2: the lane's edge of the next batch of 32, loaded one batch
        // ahead so that the load overlaps the processing of the current one.
        double4 next_d = make_double4(0.0, 0.0, 0.0, 0.0);
        int next_info = 0;
        if (MODE == 2 && lane < nedges) {
            next_d = p.edges[slot * tab.edge_cap + lane];
            next_info = p.edge_info[slot * tab.edge_cap + lane];
        }
        while (true) {
            const bool walk_done = MODE == 2 ? fetched >= nedges : (q0 >= total && round >= entries);
            if (pcount >= chunk || (walk_done && qn == 0 && pcount > 0)) {
                const int count = min(pcount, chunk);
                __syncwarp();
                process(count);
                // Move the rest (up to 63 edges) to the queue's front.
                const int rem = pcount - count;
                double sx[2], sy[2], sz[2], sr[2], swt[2];
                int st[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = lane + 32 * h;
                    if (i < rem) {
                        sx[h] = pdx[count + i];
                        sy[h] = pdy[count + i];
                        sz[h] = pdz[count + i];
                        sr[h] = pr2[count + i];
                        swt[h] = pw[count + i];
                        st[h] = ptype[count + i];
                    }
                }
                __syncwarp();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = lane + 32 * h;
                    if (i < rem) {
                        pdx[i] = sx[h];
                        pdy[i] = sy[h];
                        pdz[i] = sz[h];
                        pr2[i] = sr[h];
                        pw[i] = swt[h];
                        ptype[i] = st[h];
                    }
                }
                __syncwarp();
                pcount = rem;
            } else if (MODE == 2 && fetched < nedges) {
                // Next 32 edges of the slot, this pass's species, in order.
                const int e = fetched + lane;
                bool ok = false, in_group = false;
                const double4 d = next_d;
                const int info = next_info;
                const int t = info & 0xffff;
                const bool self = (info >> 16) != 0;
                if (e < nedges) {
                    ok = pooled || (t >= tb && t < te);
                    // The fused kernel's pass holding this species: its
                    // accepted edges, in order, alternate between the
                    // partial sums (float64 rows).
                    in_group = pooled || t / tab.parity_group == tb / tab.parity_group;
                }
                if (e + 32 < nedges) {
                    next_d = p.edges[slot * tab.edge_cap + e + 32];
                    next_info = p.edge_info[slot * tab.edge_cap + e + 32];
                }
                const unsigned mask = __ballot_sync(0xffffffffu, ok);
                const unsigned group = ks > 1 ? __ballot_sync(0xffffffffu, in_group) : 0u;
                if (ok) {
                    const int rank = __popc(mask & ((1u << lane) - 1u));
                    const int grank = __popc(group & ((1u << lane) - 1u));
                    const int q = pcount + rank;
                    double w = 1.0;
                    if (tab.weighted) {
                        w = soap_edge_weight(tab, d.w, self);
                        if (pooled) w *= tab.species_weight[t];
                    }
                    pdx[q] = d.x;
                    pdy[q] = d.y;
                    pdz[q] = d.z;
                    pr2[q] = d.w;
                    pw[q] = w;
                    ptype[q] = (pooled ? 0 : t - tb) * ks + ((naccepted + grank) & (ks - 1));
                }
                pcount += __popc(mask);
                naccepted += __popc(group);
                fetched += 32;
                __syncwarp();
            } else if (MODE != 2 && (qn >= 32 || (walk_done && qn > 0))) {
                // Exact test of queued survivors [0, count): the reference's geometry.
                const int count = min(qn, 32);
                __syncwarp();
                bool ok = false;
                double dx = 0.0, dy = 0.0, dz = 0.0, d2 = 0.0, w = 1.0;
                int t = 0;
                if (lane < count) {
                    const int j = qa[lane], tp = qt[lane];
                    t = qs[lane];
                    int nimg[3];
                    ok = accept_candidate(si, bv, p.positions, center, wi, j, (tp & 1023) - 512,
                                          ((tp >> 10) & 1023) - 512, ((tp >> 20) & 1023) - 512, tab.cutoff2, nimg,
                                          dx, dy, dz, d2);
                    if (MODE == 1) {
                        // Species and the exact-self flag; the expansion forms the weight.
                        if (ok && tab.weighted && ab + j == center && nimg[0] == 0 && nimg[1] == 0 && nimg[2] == 0)
                            t |= 1 << 16;
                    } else if (ok && tab.weighted) {
                        w = soap_edge_weight(tab, d2,
                                             ab + j == center && nimg[0] == 0 && nimg[1] == 0 && nimg[2] == 0);
                        // The pooled density carries each neighbour's species weight.
                        if (pooled) w *= tab.species_weight[t];
                    }
                }
                const unsigned mask = __ballot_sync(0xffffffffu, ok);
                if (MODE == 1 && ok) {
                    // Walk only: straight to the centre's slot.
                    const int e = written + __popc(mask & ((1u << lane) - 1u));
                    if (e < tab.edge_cap) {
                        p.edges[slot * tab.edge_cap + e] = make_double4(dx, dy, dz, d2);
                        p.edge_info[slot * tab.edge_cap + e] = t;
                    }
                } else if (ok) {
                    const int rank = __popc(mask & ((1u << lane) - 1u));
                    const int q = pcount + rank;
                    pdx[q] = dx;
                    pdy[q] = dy;
                    pdz[q] = dz;
                    pr2[q] = d2;
                    pw[q] = w;
                    ptype[q] = (pooled ? 0 : t - tb) * ks + ((naccepted + rank) & (ks - 1));
                }
                if (MODE == 1)
                    written += __popc(mask);
                else
                    pcount += __popc(mask);
                naccepted += __popc(mask);
                // Move the remaining survivors (up to 63) to the queue's front.
                const int rem = qn - count;
                int sa0 = 0, st0 = 0, ss0 = 0, sa1 = 0, st1 = 0, ss1 = 0;
                if (lane < rem) {
                    sa0 = qa[count + lane];
                    st0 = qt[count + lane];
                    ss0 = qs[count + lane];
                }
                if (lane + 32 < rem) {
                    sa1 = qa[count + 32 + lane];
                    st1 = qt[count + 32 + lane];
                    ss1 = qs[count + 32 + lane];
                }
                __syncwarp();
                if (lane < rem) {
                    qa[lane] = sa0;
                    qt[lane] = st0;
                    qs[lane] = ss0;
                }
                if (lane + 32 < rem) {
                    qa[32 + lane] = sa1;
                    qt[32 + lane] = st1;
                    qs[32 + lane] = ss1;
                }
                __syncwarp();
                qn = rem;
            } else if (MODE != 2 && q0 < total) {
                // Prefilter candidates q0 .. q0 + 63 of this round, two per
                // lane (q0 + lane and q0 + 32 + lane): the two searches and
                // the two position loads are independent, so their latencies
                // overlap.  Survivors are queued in candidate order.
                const int qA = q0 + lane, qB = q0 + 32 + lane;
                bool passA = false, passB = false;
                int aA = 0, tyA = 0, iA = 0, aB = 0, tyB = 0, iB = 0;  // a: local atom id
                // Float32 plans take candidates whose prefilter d^2 lies below
                // the inner radius straight into the edge queue, with the
                // prefilter's displacement (a few 1e-16 relative from the
                // reference's): their membership in the pair set is certain,
                // and float32 rows do not see the displacement's last bits.
                // The rest go through the exact test.
                constexpr bool kDirect = !PRECISE && !POLY;
                bool dirA = false, dirB = false;
                double xA = 0.0, yA = 0.0, zA = 0.0, rA = 0.0, xB = 0.0, yB = 0.0, zB = 0.0, rB = 0.0;
                {
                    // Segment of each candidate: the non-empty segments have
                    // strictly increasing starts, so candidate q belongs to
                    // segment #{starts <= q} - 1.  Bit d of (hi:lo) marks a
                    // segment starting at q0 + d; lane i holds segment i's start.
                    const int d = seg_first - q0;
                    const unsigned lo = __reduce_or_sync(0xffffffffu, (d >= 0 && d < 32) ? 1u << d : 0u);
                    const unsigned hi = __reduce_or_sync(0xffffffffu, (d >= 32 && d < 64) ? 1u << (d - 32) : 0u);
                    const int before = __popc(__ballot_sync(0xffffffffu, d < 0)) - 1;
                    const unsigned upto = 0xffffffffu >> (31 - lane);
                    iA = before + __popc(lo & upto);
                    iB = before + __popc(lo) + __popc(hi & upto);
                }
                if (qA < total) {
                    const double4 sp = bv.spos[ab + seg_start[iA] + (qA - seg_prefix[iA])];
                    const long long code = __double_as_longlong(sp.w);
                    tyA = (int)(code & 127) - 1;
                    aA = (int)(code >> 7);
                    xA = sp.x + seg_off[iA];
                    yA = sp.y + seg_off[32 + iA];
                    zA = sp.z + seg_off[64 + iA];
                    rA = fma(zA, zA, fma(yA, yA, xA * xA));
                    passA = (pooled || (tyA >= tb && tyA < te)) && rA <= pre2;
                    dirA = kDirect && passA && rA <= in2;
                }
                if (qB < total) {
                    const double4 sp = bv.spos[ab + seg_start[iB] + (qB - seg_prefix[iB])];
                    const long long code = __double_as_longlong(sp.w);
                    tyB = (int)(code & 127) - 1;
                    aB = (int)(code >> 7);
                    xB = sp.x + seg_off[iB];
                    yB = sp.y + seg_off[32 + iB];
                    zB = sp.z + seg_off[64 + iB];
                    rB = fma(zB, zB, fma(yB, yB, xB * xB));
                    passB = (pooled || (tyB >= tb && tyB < te)) && rB <= pre2;
                    dirB = kDirect && passB && rB <= in2;
                }
                const unsigned lt = (1u << lane) - 1u;
                if constexpr (kDirect) {
                    // Direct edges, in candidate order, after the queued ones.
                    const unsigned dA = __ballot_sync(0xffffffffu, dirA);
                    const unsigned dB = __ballot_sync(0xffffffffu, dirB);
                    auto push = [&](int at, int a, int ty, int seg, double x, double y, double z, double r) {
                        double w = 1.0;
                        int info = ty;
                        if (tab.weighted) {
                            const bool self = ab + a == center && seg_t[seg] == (512 | (512 << 10) | (512 << 20));
                            if (MODE == 1) {
                                info |= self ? 1 << 16 : 0;
                            } else {
                                w = soap_edge_weight(tab, r, self);
                                if (pooled) w *= tab.species_weight[ty];
                            }
                        }
                        if constexpr (MODE == 1) {
                            // Walk only: straight to the centre's slot (the queue
                            // stays empty, so `at` is the edge's rank among the
                            // centre's accepted edges after `written`).
                            const int e = written + at;
                            if (e < tab.edge_cap) {
                                p.edges[slot * tab.edge_cap + e] = make_double4(x, y, z, r);
                                p.edge_info[slot * tab.edge_cap + e] = info;
                            }
                            return;
                        }
                        pdx[at] = x;
                        pdy[at] = y;
                        pdz[at] = z;
                        pr2[at] = r;
                        pw[at] = w;
                        ptype[at] = pooled ? 0 : ty - tb;
                    };
                    if (dirA) push(pcount + __popc(dA & lt), aA, tyA, iA, xA, yA, zA, rA);
                    if (dirB) push(pcount + __popc(dA) + __popc(dB & lt), aB, tyB, iB, xB, yB, zB, rB);
                    if (MODE == 1)
                        written += __popc(dA) + __popc(dB);
                    else
                        pcount += __popc(dA) + __popc(dB);
                    naccepted += __popc(dA) + __popc(dB);
                    passA = passA && !dirA;
                    passB = passB && !dirB;
                }
                const unsigned maskA = __ballot_sync(0xffffffffu, passA);
                const unsigned maskB = __ballot_sync(0xffffffffu, passB);
                if (passA) {
                    const int at = qn + __popc(maskA & lt);
                    qa[at] = aA;
                    qt[at] = seg_t[iA];
                    qs[at] = tyA;
                }
                if (passB) {
                    const int at = qn + __popc(maskA) + __popc(maskB & lt);
                    qa[at] = aB;
                    qt[at] = seg_t[iB];
                    qs[at] = tyB;
                }
                qn += __popc(maskA) + __popc(maskB);
                q0 += 64;
                __syncwarp();
            } else if (MODE != 2 && round < entries) {
                // Segments round .. round + 31: one (y, z) bin row at one x image each.
                const int e = round + lane;
                bool valid = e < entries;
                int start = 0, len = 0, tpack = 0;
                double ox = 0.0, oy = 0.0, oz = 0.0;
                if (valid) {
                    const int row = e / nxs;
                    const int xs = e - row * nxs;
                    const int dz = row / wy - Kz;
                    const int dy = row - (row / wy) * wy - Ky;
                    const int ey = cy + dy, ez = cz + dz;
                    int ty = 0, tz = 0, tx = 0, b0, b1;
                    // Axis-aligned bins: drop rows whose box lies beyond the
                    // prefilter sphere and trim the x range to the bins the
                    // sphere reaches (the dropped candidates would all fail
                    // the prefilter, so the survivors and their order are
                    // unchanged).
                    int rxlo = xlo, rxhi = xhi;
                    if (si.aligned) {
                        const double hx = si.extent[0] / Mx, hy = si.extent[1] / My, hz = si.extent[2] / Mz;
                        const double cx_ = wpos[0] - si.origin[0], cy_ = wpos[1] - si.origin[1],
                                     cz_ = wpos[2] - si.origin[2];
                        const double eps = 1e-8 * (1.0 + si.extent[0] + si.extent[1] + si.extent[2] + fabs(cx_) +
                                                   fabs(cy_) + fabs(cz_) + sqrt(pre2));
                        auto gap = [&](double c, int e, double h) {
                            const double lo = e * h, hi = (e + 1) * h;
                            return fmax(0.0, (c < lo ? lo - c : (c > hi ? c - hi : 0.0)) - eps);
                        };
                        const double ry = gap(cy_, ey, hy), rz = gap(cz_, ez, hz);
                        const double rem = pre2 - ry * ry - rz * rz;
                        if (rem < 0.0) {
                            valid = false;
                        } else if (hx > 0.0) {
                            const double reach = sqrt(rem) + eps;
                            rxlo = max(xlo, (int)fmax(floor((cx_ - reach) / hx), (double)xlo - 1.0));
                            rxhi = min(xhi, (int)fmin(floor((cx_ + reach) / hx), (double)xhi + 1.0));
                        }
                    }
                    if (periodic) {
                        ty = floor_div(ey, My);
                        tz = floor_div(ez, Mz);
                        tx = tx0 + xs;
                        b0 = max(rxlo, tx * Mx) - tx * Mx;
                        b1 = min(rxhi, tx * Mx + Mx - 1) - tx * Mx;
                    } else {
                        valid = valid && ey >= 0 && ey < My && ez >= 0 && ez < Mz;
                        b0 = max(rxlo, 0);
                        b1 = min(rxhi, Mx - 1);
                    }
                    valid = valid && b0 <= b1;
                    if (valid) {
                        const int64_t rowbase = bb + Mx * ((ey - ty * My) + My * (ez - tz * Mz));
                        start = bv.bin_start[rowbase + b0];
                        len = bv.bin_start[rowbase + b1 + 1] - start;
                        tpack = (tx + 512) | ((ty + 512) << 10) | ((tz + 512) << 20);
                        // Approximate displacement = wrapped neighbour + t.A - wrapped centre.
                        const double fx = (double)tx, fy = (double)ty, fz = (double)tz;
                        ox = fma(fz, si.cell[6], fma(fy, si.cell[3], fx * si.cell[0])) - wpos[0];
                        oy = fma(fz, si.cell[7], fma(fy, si.cell[4], fx * si.cell[1])) - wpos[1];
                        oz = fma(fz, si.cell[8], fma(fy, si.cell[5], fx * si.cell[2])) - wpos[2];
                    }
                }
                int incl = len;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int up = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += up;
                }
                total = __shfl_sync(0xffffffffu, incl, 31);
                q0 = 0;
                round += 32;
                // Only the non-empty segments are kept, in order.
                const unsigned nonempty = __ballot_sync(0xffffffffu, len > 0);
                const int at = __popc(nonempty & ((1u << lane) - 1u));
                __syncwarp();
                if (len > 0) {
                    seg_prefix[at] = incl - len;
                    seg_start[at] = start;
                    seg_t[at] = tpack;
                    seg_off[at] = ox;
                    seg_off[32 + at] = oy;
                    seg_off[64 + at] = oz;
                }
                __syncwarp();
                seg_first = lane < __popc(nonempty) ? seg_prefix[lane] : 0x7fffffff;
            } else {
                break;
            }
        }

        if constexpr (kPair) {
            // Both halves' sums of both radial indices; half h keeps index kp + h n/2.
#pragma unroll
            for (int m = 0; m < P::W; ++m) {
                const double v0 = acc[0][m] + __shfl_xor_sync(0xffffffffu, acc[0][m], 16);
                const double v1 = acc[1][m] + __shfl_xor_sync(0xffffffffu, acc[1][m], 16);
                acc[0][m] = (lane >> 4) ? v1 : v0;
            }
        }
        // Flush the raw sums times the species weight: row (t, k), degree l
        // at columns col_off(l) .. + kpad(l), padding written as 0 where the
        // tail reads it.
        if (MODE != 1 && lane_on) {
            const int colA = mma::col_off(lA);
            const int colB = lB >= 0 ? mma::col_off(lB) - split : 0;
            const int padA = mma::kpad(lA), padB = lB >= 0 ? mma::kpad(lB) : 0;
            static_for<0, MAXT>([&](auto bank) {
                constexpr int tt = decltype(bank)::value;
                // Bank tt holds species tb + tt / ks (partial sum tt % ks).
                const int t = tb + tt / ks;
                if (tt % ks == 0 && t < te) {
                    const double w = pooled ? 1.0 : tab.species_weight[t];
                    double* row = R + (t * n + k) * tab.rs;
#pragma unroll
                    for (int m = 0; m < P::W; ++m) {
                        double v = acc[tt][m];
                        if constexpr (ks == 2 && tt + 1 < MAXT) v += acc[tt + 1][m];
                        if (m < split)
                            row[colA + m] = w * v;
                        else if (lB >= 0)
                            row[colB + m] = w * v;
                    }
                    // The register tails (tail_regs_n8, soap_tail_kernel) never read the padding.
                    if (!regs_tail && !(MODE == 2 && tab.split_tail == 1)) {
                        for (int m = split; m < padA; ++m) row[colA + m] = 0.0;
                        if (lB >= 0)
                            for (int m = 2 * lB + 1; m < padB; ++m) row[colB + split + m] = 0.0;
                    }
                }
            });
        }
        __syncwarp();
    }

    if constexpr (MODE == 1) {
        if (lane == 0) p.edge_count[slot] = written;
        return;
    }
    if (SPLIT || tab.split_tail) {
        // The tail runs as its own kernel (soap_tail_kernel): hand the raw
        // sums over through global scratch, one contiguous block per centre
        // (already there when the flush wrote them to global memory).
        if (tab.r_global) return;
        const double2* src = reinterpret_cast<const double2*>(R);
        double2* dst = reinterpret_cast<double2*>(p.rbuf + (center - p.grid_begin) * tab.rsize);
        for (int i = lane; i < tab.rsize / 2; i += 32) dst[i] = src[i];
        return;
    }

    if (regs_tail) {
        // Coefficients stay in registers from the beta transform to the power spectrum.
        if (tab.average == 0) {
            const int64_t row = center - p.out_row_begin;
            if (tab.out_f64)
                mma::tail_regs_n8<L, MAXT>(bt, R, tab.rs, S, tab.compression, tab.power_pref,
                                           static_cast<double*>(p.out) + row * tab.features, lane);
            else
                mma::tail_regs_n8<L, MAXT>(bt, R, tab.rs, S, tab.compression, tab.power_pref,
                                           static_cast<float*>(p.out) + row * tab.features, lane);
        } else {
            mma::tail_regs_n8<L, MAXT>(bt, R, tab.rs, S, tab.compression, tab.power_pref,
                                       p.pbuf + local * tab.features, lane);
        }
        return;
    }
    tail_generic<L>(tab, p, R, bt, center, lane);
    };
    for (int64_t center = c_lo + warp; center < c_hi; center += kWarps) run_centre(center);
}

// Tail of the paired kernel as a kernel of its own (n_max == 8, average off
// or outer, at most MAXS species).  Persistent: CTA b takes centres b,
// b + gridDim.x, ...; each centre's raw-sum block arrives in shared memory by
// one bulk (TMA) copy, double buffered, so the next centre's block is in
// flight while the four warps work on this one.  Warp w runs the register
// tail (beta transform + power spectrum on the fp64 tensor cores) for the
// degrees of channel group w -- {L}, {L-1, 0}, {L-2, 1}, ..., four groups of
// about equal tensor-core work for L = 5, 6.  A copy that does not complete
// within a second sets kErrTailTimeout and ends the CTA.
template <int L, int MAXS>
__global__ void __launch_bounds__(kWarps * 32)
soap_tail_kernel(const __grid_constant__ SoapTables tab, const SoapPointers p) {
    using P = paired::Layout<L>;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int S = tab.coef_species, n = tab.n_max;
    double* bt = reinterpret_cast<double*>(smem);
    for (int i = threadIdx.x; i < (L + 1) * 64; i += blockDim.x) {
        const int l = i / 64, nn = (i / 8) % 8, k = i % 8;
        bt[i] = (nn < n && k < n) ? tab.soap_scale * p.betas[((int64_t)l * n + nn) * n + k] : 0.0;
    }
    constexpr int kShared = (L + 1) * 64 * 8;
    double* const rbuf = reinterpret_cast<double*>(smem + kShared);  // two blocks of rsize doubles
    const uint32_t bytes = (uint32_t)tab.rsize * 8u;  // a multiple of 256 (row_stride)
    const int64_t count = p.grid_end - p.grid_begin;
    if (threadIdx.x == 0) {
        bulk::barrier_init(&bars[0], 1);
        bulk::barrier_init(&bars[1], 1);
        bulk::barrier_init_fence();
    }
    __syncthreads();
    int64_t c = blockIdx.x;
    if (threadIdx.x == 0 && c < count) {
        bulk::arrive_expect(&bars[0], bytes);
        bulk::load(rbuf, p.rbuf + c * tab.rsize, bytes, &bars[0]);
    }
    const int la = warp < P::G ? P::la(warp) : 0, lb = warp < P::G ? P::lb(warp) : -1;
    for (int it = 0; c < count; ++it, c += gridDim.x) {
        const int b = it & 1;
        const int64_t next = c + gridDim.x;
        // Buffer b^1 was last read in iteration it - 1, which ended in a barrier.
        if (threadIdx.x == 0 && next < count) {
            bulk::proxy_fence();
            bulk::arrive_expect(&bars[b ^ 1], bytes);
            bulk::load(rbuf + (b ^ 1) * tab.rsize, p.rbuf + next * tab.rsize, bytes, &bars[b ^ 1]);
        }
        const bool ok = bulk::wait(&bars[b], (uint32_t)(it >> 1) & 1u);
        if (__syncthreads_or(!ok)) {
            // Before the CTA hands its shared memory back, give each copy it
            // issued one more bounded wait: the one that timed out and the one
            // for the next centre.  A copy still outstanding after both waits
            // (two further seconds) is left in flight; the error word already
            // tells the host that this launch's rows are invalid.
            if (threadIdx.x == 0) {
                atomicOr(p.bins.error, kErrTailTimeout);
                bulk::wait(&bars[b], (uint32_t)(it >> 1) & 1u);
                if (next < count) bulk::wait(&bars[b ^ 1], (uint32_t)((it + 1) >> 1) & 1u);
            }
            __syncthreads();
            return;
        }
        const double* R = rbuf + b * tab.rsize;
        const int64_t center = p.grid_begin + c;
        if (warp < P::G) {
            if (tab.average == 0) {
                const int64_t row = center - p.out_row_begin;
                if (tab.out_f64)
                    mma::tail_regs_n8<L, MAXS>(bt, R, tab.rs, S, tab.compression, tab.power_pref,
                                               static_cast<double*>(p.out) + row * tab.features, lane, la, la, lb);
                else
                    mma::tail_regs_n8<L, MAXS>(bt, R, tab.rs, S, tab.compression, tab.power_pref,
                                               static_cast<float*>(p.out) + row * tab.features, lane, la, la, lb);
            } else {
                mma::tail_regs_n8<L, MAXS>(bt, R, tab.rs, S, tab.compression, tab.power_pref,
                                           p.pbuf + (center - p.center_begin) * tab.features, lane, la, la, lb);
            }
        }
        __syncthreads();
    }
}

// Tail of the paired kernel as a kernel of its own for plans whose
// coefficients do not stay in registers (tail_generic): n_max < 8, more
// species than register banks, compression layouts through power_generic.
// Without tail code the expansion kernel keeps a small instruction-cache
// footprint.  Persistent: warp w of CTA b takes centres (b * kWarps + w) +
// i * gridDim.x * kWarps, copying each raw-sum block into its own slice of
// shared memory (coalesced 16-byte loads) before the tail.
template <int L>
__global__ void __launch_bounds__(kWarps * 32)
soap_tail_generic_kernel(const __grid_constant__ SoapTables tab, const SoapPointers p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n = tab.n_max;
    double* bt = reinterpret_cast<double*>(smem);
    for (int i = threadIdx.x; i < (L + 1) * 64; i += blockDim.x) {
        const int l = i / 64, nn = (i / 8) % 8, k = i % 8;
        bt[i] = (nn < n && k < n) ? tab.soap_scale * p.betas[((int64_t)l * n + nn) * n + k] : 0.0;
    }
    __syncthreads();
    constexpr int kShared = (L + 1) * 64 * 8;
    double* R = reinterpret_cast<double*>(smem + kShared) + (int64_t)warp * tab.rsize;
    const int64_t count = p.grid_end - p.grid_begin;
    for (int64_t c = (int64_t)blockIdx.x * kWarps + warp; c < count; c += (int64_t)gridDim.x * kWarps) {
        const double2* src = reinterpret_cast<const double2*>(p.rbuf + c * tab.rsize);
        double2* dst = reinterpret_cast<double2*>(R);
        __syncwarp();
        for (int i = lane; i < tab.rsize / 2; i += 32) dst[i] = src[i];
        __syncwarp();
        tail_generic<L>(tab, p, R, bt, p.grid_begin + c, lane);
    }
}

}  // namespace mdsoap
