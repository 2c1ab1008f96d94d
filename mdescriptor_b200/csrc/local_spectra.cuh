// Local spherical spectra on the GPU: SphericalExpansion, SoapRadialSpectrum
// and SoapPowerSpectrum (featomic-style GTO radial integrals of a Gaussian
// density).
//
// Reference: cpp/src/standalone/spherical_expansion.cpp:124-206 (driver and
// row assembly :15-113), cpp/src/common/local_spherical_common.hpp
// (hyp1f1_series :33-47, regularized_hyp1f1_positive :148-156, GtoRadialBasis
// :181-299, real_spherical_harmonics_into :376-443, cutoff_value :445-454,
// compute_coefficients_into :489-540), feature layout local_layout.hpp:41-130.
//
// One warp per centre.  The warp walks the centre's cell bins (the same walk
// and exact pair test as the SOAP kernels, cutoff = the descriptor's cutoff,
// exact self pair included), queues accepted edges in shared memory and,
// 32 at a time, gives each lane one edge: the lane evaluates the edge's real
// spherical harmonics and its orthonormalised radial integrals R_l(n) into
// the warp's shared edge buffer.  Then every lane owns a fixed set of
// (n, lm) coefficients and adds R_l(n) Y_lm of each queued edge, in queue
// order, into the coefficient bank of the edge's species.  The row is
// assembled from the banks and stored coalesced in float64.
#pragma once

#include "neighbors.cuh"

namespace mdsoap {

constexpr int kLocalMaxL = 8;   // largest max_angular of the kernel
constexpr int kLocalMaxN = 16;  // largest radial count (max_radial + 1)
constexpr unsigned kErrLocalSeries = 128u;  // 1F1 series overflowed (the reference throws)
constexpr int kLocalRecip = 256;             // series terms with a tabulated 1 / ((b + k - 1) k)

enum LocalKind : int { kLocalSphericalExpansion = 0, kLocalRadialSpectrum = 2, kLocalPowerSpectrum = 3 };

struct LocalTables {
    int kind;
    int n;               // radial count
    int lc;              // coefficient max angular (0 for the radial spectrum)
    int l_out;           // max angular of the power spectrum rows
    int species;
    int features;
    double cutoff;
    double cutoff2;
    double c;            // density constant 1 / (2 w^2)
    double gf;           // (pi / w^2)^(3/4)
    double log_gf;       // log(gf), host libm as the reference
    const double* g;       // [n] GTO constants 1 / (2 sigma_n^2)
    const double* log_cg;  // [n] log(c + g_n)
    const double* gratio;  // [(lc+1) n] Gamma(a) / Gamma(b)
    const double* ppow;    // [(lc+1) n] (c + g_n)^(-a)
    const double* ortho;   // [n][n] normalisation * S^(-1/2)
    const double* recip;   // [(lc+1)][kLocalRecip]: 1 / ((l + 1.5 + k - 1) k), index k (entry 0 unused)
    const double* ynorm;   // [l(l+1)/2 + m], m <= l <= lc: (-1)^m N_lm, times sqrt 2 for m > 0
};

struct LocalLayout {
    int H;        // (lc+1)^2
    int nH;       // n * H
    int coef;     // doubles of coefficient banks per warp (species * nH)
    int ystride;  // doubles per edge harmonic row
    int rstride;  // doubles per edge radial row ((lc+1) n)
    size_t bytes_per_warp;
};

__host__ __device__ inline LocalLayout local_layout(int species, int n, int lc) {
    LocalLayout L;
    L.H = (lc + 1) * (lc + 1);
    L.nH = n * L.H;
    L.coef = species * L.nH;
    L.ystride = L.H | 1;
    L.rstride = ((lc + 1) * n) | 1;
    // banks + 32 harmonic rows + 32 radial rows + 64-edge queue (4 doubles)
    // + 32 edge species + 64 queued species
    L.bytes_per_warp = 8 * ((size_t)L.coef + 32 * (size_t)L.ystride + 32 * (size_t)L.rstride + 64 * 4) +
                       4 * (32 + 64);
    L.bytes_per_warp = (L.bytes_per_warp + 15) & ~(size_t)15;
    return L;
}

// 1F1(a; b; x) by its power series for x >= 0, with the stopping rule of
// hyp1f1_series (local_spherical_common.hpp:33-47).  The term ratio
// (a + k - 1) x / ((b + k - 1) k) multiplies by the tabulated, correctly
// rounded reciprocal of its exact denominator (a half-integer times an
// integer) instead of dividing: one multiply for the division's reciprocal
// iteration, at most one more rounding per term.
__device__ inline double local_hyp1f1_series(double a, double b, double x, const double* __restrict__ recip,
                                             bool& overflow) {
    double sum = 1.0;
    double term = 1.0;
    for (int k = 1; k < 10000; ++k) {
        const double num = __dmul_rn(a + (double)k - 1.0, x);
        const double ratio = k < kLocalRecip ? __dmul_rn(num, __ldg(recip + k))
                                             : __ddiv_rn(num, __dmul_rn(b + (double)k - 1.0, (double)k));
        term = __dmul_rn(term, ratio);
        sum = __dadd_rn(sum, term);
        if (fabs(term) <= __dmul_rn(fabs(sum), 2e-15)) break;
        if (!isfinite(sum)) {
            overflow = true;
            break;
        }
    }
    return sum;
}

// The 30-term asymptotic sum of regularized_hyp1f1_positive (:148-156).
__device__ inline double local_hyp1f1_asymptotic(double a, double b, double x) {
    double sum = 1.0;
    double term = 1.0;
    for (int i = 1; i <= 30; ++i) {
        const double di = (double)i;
        term = __ddiv_rn(__dmul_rn(__dmul_rn(-term, b - a + di - 1.0), a - di), __dmul_rn(x, di));
        sum = __dadd_rn(sum, term);
    }
    return sum;
}

// Real spherical harmonics of a displacement in the reference's layout
// (index l^2 + l + m; real_spherical_harmonics_into, :376-443, defines the
// values).  Evaluated here as regular solid harmonics of the unit direction
// by the Cartesian recurrence the SOAP kernels use (Y_l^m = N_lm r^l P_l^m
// (cos m phi, sin m phi) with P_mm = -(2m - 1)(x P - y P'), then
// P_lm = ((2l - 1) z P_{l-1,m} - (l + m - 1) r^2 P_{l-2,m}) / (l - m) at
// r = 1), with the reference's sign convention folded into the host table
// ynorm[l(l+1)/2 + m] = (-1)^m N_lm (times sqrt 2 for m > 0).  The direction
// is normalised as the reference does (length below 1e-6: the z axis).
__device__ inline void local_harmonics(const LocalTables& t, double x, double y, double z, int lmax, double* out) {
    const double norm = sqrt(__dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)), __dmul_rn(z, z)));
    double ux, uy, uz;
    if (norm < 1e-6) {
        ux = 0.0;
        uy = 0.0;
        uz = 1.0;
    } else {
        ux = __ddiv_rn(x, norm);
        uy = __ddiv_rn(y, norm);
        uz = __ddiv_rn(z, norm);
    }
    double dr = 1.0, di = 0.0;  // P_mm (cos and sin parts)
    for (int m = 0; m <= lmax; ++m) {
        if (m > 0) {
            const double f = -(2.0 * m - 1.0);
            const double nr = f * fma(ux, dr, -__dmul_rn(uy, di));
            const double ni = f * fma(ux, di, __dmul_rn(uy, dr));
            dr = nr;
            di = ni;
        }
        auto store = [&](int l, double re, double im) {
            const double nrm = __ldg(t.ynorm + l * (l + 1) / 2 + m);
            out[l * l + l + m] = nrm * re;
            if (m > 0) out[l * l + l - m] = nrm * im;
        };
        store(m, dr, di);
        if (m < lmax) {
            const double c = (2.0 * m + 1.0) * uz;
            double pr2 = dr, pi2 = di, pr1 = c * dr, pi1 = c * di;
            store(m + 1, pr1, pi1);
            for (int l = m + 2; l <= lmax; ++l) {
                const double a = (2.0 * l - 1.0) / (double)(l - m) * uz;
                const double b = (double)(l + m - 1) / (double)(l - m);
                const double nr = fma(a, pr1, -b * pr2);
                const double ni = fma(a, pi1, -b * pi2);
                pr2 = pr1;
                pi2 = pi1;
                pr1 = nr;
                pi1 = ni;
                store(l, nr, ni);
            }
        }
    }
}

// Degree l of harmonic index h = l^2 + l + m (h < 81): floor(sqrt(h)).
__device__ __forceinline__ int degree_of(int h) {
    int l = (int)sqrtf((float)h);
    l += (l + 1) * (l + 1) <= h;
    l -= l * l > h;
    return l;
}

// Smooth cosine cutoff of width min(0.5, cutoff) (cutoff_value, :445-454).
__device__ inline double local_cutoff_value(double d, double rc) {
    if (d >= rc) return 0.0;
    const double width = fmin(0.5, rc);
    if (d <= rc - width) return 1.0;
    constexpr double kPi = 3.141592653589793238462643383279502884;
    return __dmul_rn(0.5, __dadd_rn(1.0, cos(__ddiv_rn(__dmul_rn(kPi, __dadd_rn(__dsub_rn(d, rc), width)), width))));
}

// Orthonormalised radial integrals of degree l at distance d, times the
// cutoff factor: out[target] = scaling * sum_n raw_n ortho[n][target]
// (radial_integral_into_prepared, :255-284, then the scaling of :525-527).
__device__ inline void local_radial(const LocalTables& t, int l, double d, double scaling, double* out,
                                    bool& overflow) {
    const double c_r = __dmul_rn(t.c, d);
    const double factor = __dmul_rn(__dmul_rn(t.gf, exp(-__dmul_rn(d, c_r))), pow(c_r, (double)l));
    const double b = (double)l + 1.5;
    double raw[kLocalMaxN];
    for (int k = 0; k < t.n; ++k) {
        const double g = __ldg(t.g + k);
        const double z = __ddiv_rn(__dmul_rn(c_r, c_r), __dadd_rn(t.c, g));
        const double a = 0.5 * ((double)k + (double)l + 3.0);
        if (z > 30.0) {
            const double asym = local_hyp1f1_asymptotic(a, b, z);
            double lg = __dsub_rn(t.log_gf, __dmul_rn(d, c_r));
            lg = __dadd_rn(lg, __dmul_rn((double)l, log(c_r)));
            lg = __dsub_rn(lg, __dmul_rn(a, __ldg(t.log_cg + k)));
            lg = __dadd_rn(lg, z);
            lg = __dadd_rn(lg, __dmul_rn(__dsub_rn(a, b), log(z)));
            raw[k] = __dmul_rn(exp(lg), asym);
        } else {
            const double s = local_hyp1f1_series(a, b, z, t.recip + l * kLocalRecip, overflow);
            raw[k] = __dmul_rn(__dmul_rn(__dmul_rn(__ldg(t.gratio + l * t.n + k), s), __ldg(t.ppow + l * t.n + k)),
                               factor);
        }
    }
    for (int j = 0; j < t.n; ++j) {
        double acc = 0.0;
        for (int k = 0; k < t.n; ++k) acc = __dadd_rn(acc, __dmul_rn(raw[k], __ldg(t.ortho + k * t.n + j)));
        out[j] = __dmul_rn(acc, scaling);
    }
}

// Pair index -> (first, second) species with first <= second
// (local_decode_species_pair, local_layout.hpp:97-113).
__device__ inline void local_species_pair(int pair, int S, int& first, int& second) {
    first = 0;
    second = 0;
    for (int cand = 0; cand < S; ++cand) {
        const int count = S - cand;
        if (pair < count) {
            first = cand;
            second = cand + pair;
            return;
        }
        pair -= count;
    }
}

// Centres [a0, a1); row r of `out` belongs to centre a0 + r.
__global__ void __launch_bounds__(128) local_spectra_kernel(LocalTables t, const double* __restrict__ pos, BinView v,
                                                            int64_t a0, int64_t a1, double* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char local_smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t center = a0 + (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (center >= a1) return;
    const LocalLayout L = local_layout(t.species, t.n, t.lc);
    unsigned char* base = local_smem + (size_t)warp * L.bytes_per_warp;
    double* coef = reinterpret_cast<double*>(base);
    double* ys = coef + L.coef;
    double* rs = ys + 32 * L.ystride;
    double* queue = rs + 32 * L.rstride;  // [64][4]: dx, dy, dz, d2
    int* etype = reinterpret_cast<int*>(queue + 64 * 4);
    int* qtype = etype + 32;

    for (int i = lane; i < L.coef; i += 32) coef[i] = 0.0;
    const StructInfo& si = v.info[v.struct_of[center]];
    const int wi[3] = {v.wrap[3 * center], v.wrap[3 * center + 1], v.wrap[3 * center + 2]};
    bool overflow = false;
    int queued = 0;

    // Evaluate the first `count` queued edges, add them to the banks in queue
    // order and move the rest of the queue to its front.
    auto process = [&](int count) {
        __syncwarp();
        if (lane < count) {
            const double dx = queue[4 * lane], dy = queue[4 * lane + 1], dz = queue[4 * lane + 2];
            const double d = sqrt(fmax(0.0, queue[4 * lane + 3]));
            const double scaling = local_cutoff_value(d, t.cutoff);
            int ty = qtype[lane];
            if (scaling == 0.0) ty = -1;
            etype[lane] = ty;
            if (ty >= 0) {
                local_harmonics(t, dx, dy, dz, t.lc, ys + lane * L.ystride);
                for (int l = 0; l <= t.lc; ++l) local_radial(t, l, d, scaling, rs + lane * L.rstride + l * t.n, overflow);
            }
        }
        __syncwarp();
        for (int e = 0; e < count; ++e) {
            const int ty = etype[e];
            if (ty < 0) continue;
            const double* y = ys + e * L.ystride;
            const double* r = rs + e * L.rstride;
            double* bank = coef + ty * L.nH;
            for (int i = lane; i < L.nH; i += 32) {
                const int k = i / L.H, h = i - k * L.H;
                const int l = degree_of(h);
                bank[i] = __dadd_rn(bank[i], __dmul_rn(r[l * t.n + k], y[h]));
            }
        }
        __syncwarp();
        const int rest = queued - count;
        double tmp[4] = {0, 0, 0, 0};
        int tt = 0;
        if (lane < rest) {
#pragma unroll
            for (int c = 0; c < 4; ++c) tmp[c] = queue[4 * (count + lane) + c];
            tt = qtype[count + lane];
        }
        __syncwarp();
        if (lane < rest) {
#pragma unroll
            for (int c = 0; c < 4; ++c) queue[4 * lane + c] = tmp[c];
            qtype[lane] = tt;
        }
        queued = rest;
        __syncwarp();
    };

    for_each_candidate(si, v, center, lane, [&](bool valid, int j, int tx, int ty, int tz) {
        int n[3];
        double dx, dy, dz, d2;
        const bool ok = valid && accept_candidate(si, v, pos, center, wi, j, tx, ty, tz, t.cutoff2, n, dx, dy, dz, d2);
        const unsigned mask = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            const int slot = queued + __popc(mask & ((1u << lane) - 1u));
            queue[4 * slot] = dx;
            queue[4 * slot + 1] = dy;
            queue[4 * slot + 2] = dz;
            queue[4 * slot + 3] = d2;
            qtype[slot] = v.type[si.atom_begin + j];
        }
        queued += __popc(mask);
        if (queued >= 32) process(32);
    });
    while (queued > 0) process(min(queued, 32));
    if (__any_sync(0xffffffffu, overflow) && lane == 0) atomicOr(v.error, kErrLocalSeries);

    // Row assembly (spherical_expansion.cpp:15-113): the centre species'
    // block holds the values, every other block is zero.
    const int ct = v.type[center];
    double* row = out + (center - a0) * (int64_t)t.features;
    const int S = t.species;
    if (t.kind == kLocalPowerSpectrum) {
        const int n = t.n, n2 = n * n;
        const int per_pair = (t.l_out + 1) * n2;
        const int block = S * (S + 1) / 2 * per_pair;
        for (int f = lane; f < t.features; f += 32) {
            double value = 0.0;
            const int fl = f - ct * block;
            if (fl >= 0 && fl < block) {
                const int p = fl / per_pair;
                const int rem = fl - p * per_pair;
                const int l = rem / n2;
                const int n1 = (rem / n) % n, nn2 = rem % n;
                int first, second;
                local_species_pair(p, S, first, second);
                const double* c1 = coef + first * L.nH + n1 * L.H + l * l;
                const double* c2 = coef + second * L.nH + nn2 * L.H + l * l;
                double acc = 0.0;
                for (int m = 0; m < 2 * l + 1; ++m) acc = __dadd_rn(acc, __dmul_rn(c1[m], c2[m]));
                const double pair_scale = first == second ? 1.0 : 1.41421356237309504880168872420969808;
                const double ang = __ddiv_rn((l % 2 == 0) ? 1.0 : -1.0, sqrt(2.0 * l + 1.0));
                value = __dmul_rn(__dmul_rn(pair_scale, ang), acc);
            }
            row[f] = value;
        }
    } else {
        const int block = S * L.nH;
        for (int f = lane; f < t.features; f += 32) {
            double value = 0.0;
            const int fl = f - ct * block;
            if (fl >= 0 && fl < block) {
                const int s2 = fl / L.nH;
                const int rem = fl - s2 * L.nH;
                const int h = rem / t.n, r = rem % t.n;
                value = coef[s2 * L.nH + r * L.H + h];
            }
            row[f] = value;
        }
    }
}

}  // namespace mdsoap
