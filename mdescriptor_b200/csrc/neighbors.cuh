// Cell-binned neighbour search (sm_100a), bit-exact against the reference CPU graph.
//
// Reference semantics (cpp/src/common/neighbor.cpp:423-679): a pair (i, j, n)
// with n an integer image in [-b, b]^3 is kept iff
//     d = (x_j + ((n0*a0 + n1*a1) + n2*a2)) - x_i,   d2 = (dx*dx + dy*dy) + dz*dz <= cutoff^2
// evaluated in IEEE fp64 without contraction, on UNWRAPPED positions; the
// exact self pair (i, i, 0) is kept.  Which candidates get tested does not
// change that set, so the search here bins each structure once (lattice
// coordinates for periodic cells, bounding box for isolated ones), and every
// centre scans the bins within a half-width K that provably covers its cutoff
// sphere; each candidate is then accepted by the reference's own arithmetic.
#pragma once

#include "common.cuh"

namespace mdsoap {

struct DeviceBatch {
    const int32_t* numbers;
    const double* positions;
    const double* cells;
    const int32_t* pbc;
    const int64_t* offsets;
    int64_t structures;
    int64_t atoms;
};

// ---------------------------------------------------------------------------
// Per-structure setup (thread 0 of the bin kernel).

// math3.hpp:44-68: determinant and inverse with the reference's operation order.
__device__ inline bool exact_inverse(const double* m, double* r) {
    const double c0 = __dsub_rn(__dmul_rn(m[4], m[8]), __dmul_rn(m[5], m[7]));
    const double c1 = __dsub_rn(__dmul_rn(m[3], m[8]), __dmul_rn(m[5], m[6]));
    const double c2 = __dsub_rn(__dmul_rn(m[3], m[7]), __dmul_rn(m[4], m[6]));
    const double det = __dadd_rn(__dsub_rn(__dmul_rn(m[0], c0), __dmul_rn(m[1], c1)), __dmul_rn(m[2], c2));
    if (!isfinite(det) || fabs(det) < 1e-14) return false;
    auto cof = [&](int a, int b, int c, int d) {
        return __ddiv_rn(__dsub_rn(__dmul_rn(m[a], m[b]), __dmul_rn(m[c], m[d])), det);
    };
    r[0] = cof(4, 8, 5, 7);
    r[1] = cof(2, 7, 1, 8);
    r[2] = cof(1, 5, 2, 4);
    r[3] = cof(5, 6, 3, 8);
    r[4] = cof(0, 8, 2, 6);
    r[5] = cof(2, 3, 0, 5);
    r[6] = cof(3, 7, 4, 6);
    r[7] = cof(1, 6, 0, 7);
    r[8] = cof(0, 4, 1, 3);
    return true;
}

// Shrink the bin grid until it has at most `cap` bins.
__device__ inline void cap_bins(int* M, int64_t cap) {
    while ((int64_t)M[0] * M[1] * M[2] > cap) {
        int a = 0;
        if (M[1] > M[a]) a = 1;
        if (M[2] > M[a]) a = 2;
        M[a] = max(1, (M[a] * 3) / 4);
    }
}

// Position of an atom in the frame its bin lives in: periodic structures
// subtract the lattice translation wrap . A (the atom's image in the home
// cell); isolated ones keep the raw position.  Used only for the candidate
// prefilter, never for an accepted displacement.
__device__ __forceinline__ void wrapped_position(const StructInfo& si, const double* __restrict__ x,
                                                 const int32_t* __restrict__ wrap, double* w) {
    if (si.periodic) {
        const double f0 = (double)wrap[0], f1 = (double)wrap[1], f2 = (double)wrap[2];
#pragma unroll
        for (int c = 0; c < 3; ++c) w[c] = x[c] - fma(f2, si.cell[6 + c], fma(f1, si.cell[3 + c], f0 * si.cell[c]));
    } else {
#pragma unroll
        for (int c = 0; c < 3; ++c) w[c] = x[c];
    }
}

// Translation units that only instantiate the centre kernels (k_*.cu) leave
// out the non-template kernels, which the host translation unit defines.
#ifndef MDSOAP_NO_GRAPH_KERNELS
// ---------------------------------------------------------------------------
// Kernel 1: per structure (one CTA each): geometry plan, species lookup, and a
// deterministic counting sort of its atoms into bins.
__global__ void bin_structures_kernel(DeviceBatch b, BinView v, double cutoff,
                                      const int32_t* __restrict__ species, int n_species) {
    const int64_t s = blockIdx.x;
    const int64_t begin = b.offsets[s];
    const int64_t count = b.offsets[s + 1] - begin;
    const int tid = threadIdx.x;
    __shared__ StructInfo si;
    __shared__ double red[7][32];
    __shared__ int32_t flags;
    __shared__ int32_t scan_carry;
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t any_wrapped;

    if (tid == 0) {
        any_wrapped = 0;
        const int32_t* p = b.pbc + 3 * s;
        const bool periodic = p[0] == 1 && p[1] == 1 && p[2] == 1;
        const bool isolated = p[0] == 0 && p[1] == 0 && p[2] == 0;
        flags = periodic ? 1 : (isolated ? 0 : -1);
    }
    __syncthreads();
    const int periodic = flags;
    if (periodic < 0) {
        if (tid == 0) atomicOr(v.error, kErrMixedPbc);
        return;
    }
    // Largest |coordinate| (bounds the prefilter margin).
    {
        double amax = 0.0;
        for (int64_t a = tid; a < 3 * count; a += blockDim.x) amax = fmax(amax, fabs(b.positions[3 * begin + a]));
        for (int o = 16; o > 0; o >>= 1) amax = fmax(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if ((tid & 31) == 0) red[6][tid >> 5] = amax;
        __syncthreads();
    }
    // Bounding box of an isolated structure.
    double lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    if (!periodic) {
        for (int64_t a = tid; a < count; a += blockDim.x) {
            for (int c = 0; c < 3; ++c) {
                const double x = b.positions[3 * (begin + a) + c];
                lo[c] = fmin(lo[c], x);
                hi[c] = fmax(hi[c], x);
            }
        }
        for (int c = 0; c < 3; ++c) {
            for (int o = 16; o > 0; o >>= 1) {
                lo[c] = fmin(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
                hi[c] = fmax(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
            }
        }
        if ((tid & 31) == 0) {
            for (int c = 0; c < 3; ++c) {
                red[c][tid >> 5] = lo[c];
                red[3 + c][tid >> 5] = hi[c];
            }
        }
        __syncthreads();
    }
    if (tid == 0) {
        si.periodic = periodic;
        {
            const double* c = b.cells + 9 * s;
            si.aligned = !periodic || (c[1] == 0.0 && c[2] == 0.0 && c[3] == 0.0 && c[5] == 0.0 && c[6] == 0.0 &&
                                       c[7] == 0.0 && c[0] > 0.0 && c[4] > 0.0 && c[8] > 0.0);
        }
        si.atom_begin = begin;
        si.atom_count = (int32_t)count;
        si.bin_base = bin_base_of(begin, s);
        for (int k = 0; k < 9; ++k) si.cell[k] = b.cells[9 * s + k];
        const int64_t cap = bin_capacity(count);
        int M[3] = {1, 1, 1};
        if (periodic) {
            if (!exact_inverse(si.cell, si.inv)) {
                atomicOr(v.error, kErrSingularCell);
                for (int k = 0; k < 9; ++k) si.inv[k] = 0.0;
            }
            double cn[3];
            for (int a = 0; a < 3; ++a) {
                // neighbor.cpp:459-467, same operation order.
                const double q = __dadd_rn(__dadd_rn(__dmul_rn(si.inv[a], si.inv[a]), __dmul_rn(si.inv[3 + a], si.inv[3 + a])),
                                           __dmul_rn(si.inv[6 + a], si.inv[6 + a]));
                cn[a] = __dsqrt_rn(q);
                const double bound = floor(__dadd_rn(__dmul_rn(cutoff, cn[a]), 1.0));
                if (!(bound >= 0.0) || bound > 4096.0) {
                    atomicOr(v.error, kErrWrapRange);
                    si.bounds[a] = 0;
                } else {
                    si.bounds[a] = (int32_t)bound;
                }
                // Bins at least half a cutoff wide between lattice planes.
                const double planes = cn[a] > 0.0 ? 1.0 / cn[a] : 0.0;
                M[a] = (int)fmin(1024.0, fmax(1.0, floor(planes / (0.5 * cutoff))));
                si.origin[a] = 0.0;
                si.extent[a] = planes;
            }
            cap_bins(M, cap);
            for (int a = 0; a < 3; ++a) {
                si.M[a] = M[a];
                si.K[a] = (int)floor(cutoff * cn[a] * M[a] * (1.0 + 1e-9)) + 1;
            }
        } else {
            for (int a = 0; a < 3; ++a) {
                double l = INFINITY, h = -INFINITY;
                for (int w = 0; w < (int)((blockDim.x + 31) / 32); ++w) {
                    l = fmin(l, red[a][w]);
                    h = fmax(h, red[3 + a][w]);
                }
                if (count == 0) l = h = 0.0;
                si.origin[a] = l;
                si.extent[a] = h - l;
                si.bounds[a] = 0;
                for (int k = 0; k < 9; ++k) si.inv[k] = 0.0;
                M[a] = si.extent[a] > 0.0 ? (int)fmin(1024.0, fmax(1.0, floor(si.extent[a] / (0.5 * cutoff)))) : 1;
            }
            cap_bins(M, cap);
            for (int a = 0; a < 3; ++a) {
                si.M[a] = M[a];
                si.K[a] = si.extent[a] > 0.0
                              ? min(M[a] - 1, (int)floor(cutoff * M[a] / si.extent[a] * (1.0 + 1e-9)) + 1)
                              : 0;
            }
        }
        // Prefilter radius: every quantity in either displacement formula is
        // below Z in magnitude, so both carry rounding errors of a few 1e-16 Z;
        // a margin of 1e-11 (Z + cutoff) keeps every pair the exact test accepts.
        double amax = 0.0;
        for (int w = 0; w < (int)((blockDim.x + 31) / 32); ++w) amax = fmax(amax, red[6][w]);
        double cellsum = 0.0;
        int bmax = 0;
        if (periodic) {
            for (int k = 0; k < 9; ++k) cellsum += fabs(si.cell[k]);
            bmax = max(si.bounds[0], max(si.bounds[1], si.bounds[2]));
        }
        const double Z = 2.0 * amax + (bmax + 4.0) * cellsum;
        const double pre = cutoff + 1e-11 * (Z + cutoff);
        si.pre_cut2 = pre * pre * (1.0 + 1e-14);
        // Inner radius: a displacement of approximate length below it lies
        // within the cutoff by the reference's arithmetic as well.
        const double inner = fmax(0.0, cutoff - 1e-11 * (Z + cutoff));
        si.in_cut2 = inner * inner * (1.0 - 1e-14);
        v.info[s] = si;
    }
    __syncthreads();
    const int64_t bb = si.bin_base;
    const int Mtot = si.M[0] * si.M[1] * si.M[2];
    for (int i = tid; i <= Mtot; i += blockDim.x) v.bin_start[bb + i] = 0;
    __syncthreads();
    for (int64_t a = tid; a < count; a += blockDim.x) {
        const int64_t atom = begin + a;
        const double x = b.positions[3 * atom], y = b.positions[3 * atom + 1], z = b.positions[3 * atom + 2];
        int bin[3];
        int wrap[3] = {0, 0, 0};
        for (int c = 0; c < 3; ++c) {
            if (periodic) {
                // fractional_position (neighbor.cpp:25-31); only used for binning.
                const double f = x * si.inv[c] + y * si.inv[3 + c] + z * si.inv[6 + c];
                const double w = floor(f);
                if (!(fabs(w) < 1073741824.0)) {
                    atomicOr(v.error, kErrWrapRange);
                    bin[c] = 0;
                    continue;
                }
                wrap[c] = (int)w;
                bin[c] = min(si.M[c] - 1, max(0, (int)((f - w) * si.M[c])));
            } else {
                const double e = si.extent[c];
                const double u = e > 0.0 ? ((c == 0 ? x : c == 1 ? y : z) - si.origin[c]) * (si.M[c] / e) : 0.0;
                bin[c] = min(si.M[c] - 1, max(0, (int)floor(u)));
            }
        }
        if (wrap[0] != 0 || wrap[1] != 0 || wrap[2] != 0) any_wrapped = 1;
        const int id = bin[0] + si.M[0] * (bin[1] + si.M[1] * bin[2]);
        v.bin_of[atom] = id;
        v.wrap[3 * atom] = wrap[0];
        v.wrap[3 * atom + 1] = wrap[1];
        v.wrap[3 * atom + 2] = wrap[2];
        v.struct_of[atom] = (int32_t)s;
        const int32_t z_number = b.numbers[atom];
        int t = -1;
        for (int k = 0; k < n_species; ++k) {
            if (species[k] == z_number) {
                t = k;
                break;
            }
        }
        if (t < 0) atomicOr(v.error, kErrUnknownSpecies);
        v.type[atom] = t;
        atomicAdd(&v.bin_start[bb + id + 1], 1);
    }
    __syncthreads();
    // Inclusive scan of the counts in bin_start[bb+1 .. bb+Mtot] -> bin starts.
    if (tid == 0) scan_carry = 0;
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5, warps = (blockDim.x + 31) >> 5;
    for (int base = 1; base <= Mtot; base += blockDim.x) {
        const int i = base + tid;
        int value = i <= Mtot ? v.bin_start[bb + i] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            const int up = __shfl_up_sync(0xffffffffu, value, o);
            if (lane >= o) value += up;
        }
        if (lane == 31) warp_sums[warp] = value;
        __syncthreads();
        if (warp == 0) {
            int w = lane < warps ? warp_sums[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                const int up = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += up;
            }
            warp_sums[lane] = w;
        }
        __syncthreads();
        const int carry = scan_carry;
        value += carry + (warp > 0 ? warp_sums[warp - 1] : 0);
        if (i <= Mtot) v.bin_start[bb + i] = value;
        __syncthreads();
        if (tid == 0) scan_carry = carry + warp_sums[warps - 1];
        __syncthreads();
    }
    for (int i = tid; i < Mtot; i += blockDim.x) v.bin_cursor[bb + i] = v.bin_start[bb + i];
    // The inner radius certifies a pair only when every atom lies inside the
    // cell (then the image range admits every image within the cutoff);
    // otherwise no candidate is certified.
    if (tid == 0 && any_wrapped) v.info[s].in_cut2 = -1.0;
    __syncthreads();
    for (int64_t a = tid; a < count; a += blockDim.x) {
        const int pos = atomicAdd(&v.bin_cursor[bb + v.bin_of[begin + a]], 1);
        v.sorted[begin + pos] = (int32_t)a;
    }
    __syncthreads();
    // Deterministic order inside each bin: ascending atom id (insertion sort;
    // bins hold a handful of atoms).
    for (int i = tid; i < Mtot; i += blockDim.x) {
        const int s0 = v.bin_start[bb + i], s1 = v.bin_start[bb + i + 1];
        int32_t* list = v.sorted + begin;
        for (int p = s0 + 1; p < s1; ++p) {
            const int32_t key = list[p];
            int q = p - 1;
            while (q >= s0 && list[q] > key) {
                list[q + 1] = list[q];
                --q;
            }
            list[q + 1] = key;
        }
    }
    if (v.spos == nullptr) return;
    __syncthreads();
    // Wrapped positions in bin order, with w holding the bits of the int64
    // 128 j + species + 1 (j the structure-local atom id): the centre
    // kernels' prefilter reads one coalesced record and learns both, with no
    // conversion.
    for (int64_t p = tid; p < count; p += blockDim.x) {
        const int32_t j = v.sorted[begin + p];
        const int64_t atom = begin + j;
        double w[3];
        wrapped_position(si, b.positions + 3 * atom, v.wrap + 3 * atom, w);
        v.spos[begin + p] = make_double4(w[0], w[1], w[2], __longlong_as_double((int64_t)j * 128 + v.type[atom] + 1));
    }
}

#endif  // MDSOAP_NO_GRAPH_KERNELS

// ---------------------------------------------------------------------------
// Exact displacement of image n of atom gj seen from centre gi; returns d2.
__device__ __forceinline__ double exact_pair(const StructInfo& si, const double* __restrict__ pos,
                                             int64_t gi, int64_t gj, int n0, int n1, int n2,
                                             double& dx, double& dy, double& dz) {
    double xj = pos[3 * gj], yj = pos[3 * gj + 1], zj = pos[3 * gj + 2];
    if (si.periodic) {
        // Shift vector ((n0*a0 + n1*a1) + n2*a2) (neighbor.cpp:472-474, math3.hpp:19-29).
        const double f0 = (double)n0, f1 = (double)n1, f2 = (double)n2;
        const double sx = __dadd_rn(__dadd_rn(__dmul_rn(f0, si.cell[0]), __dmul_rn(f1, si.cell[3])), __dmul_rn(f2, si.cell[6]));
        const double sy = __dadd_rn(__dadd_rn(__dmul_rn(f0, si.cell[1]), __dmul_rn(f1, si.cell[4])), __dmul_rn(f2, si.cell[7]));
        const double sz = __dadd_rn(__dadd_rn(__dmul_rn(f0, si.cell[2]), __dmul_rn(f1, si.cell[5])), __dmul_rn(f2, si.cell[8]));
        xj = __dadd_rn(xj, sx);
        yj = __dadd_rn(yj, sy);
        zj = __dadd_rn(zj, sz);
    }
    dx = __dsub_rn(xj, pos[3 * gi]);
    dy = __dsub_rn(yj, pos[3 * gi + 1]);
    dz = __dsub_rn(zj, pos[3 * gi + 2]);
    return __dadd_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)), __dmul_rn(dz, dz));
}

// Warp-cooperative candidate walk of one centre.  Every lane calls
// visit(valid, j_local, tx, ty, tz) the same number of times; `valid` is false
// for padding lanes.  (tx, ty, tz) is the lattice image of the visited bin in
// the centre's wrapped frame; the reference image of candidate j is then
// n = t + wrap_i - wrap_j.
template <class Visit>
__device__ __forceinline__ void for_each_candidate(const StructInfo& si, const BinView& v, int64_t center,
                                                   int lane, Visit&& visit) {
    const int Mx = si.M[0], My = si.M[1], Mz = si.M[2];
    const int cb = v.bin_of[center];
    const int cx = cb % Mx, cy = (cb / Mx) % My, cz = cb / (Mx * My);
    const int64_t bb = si.bin_base;
    const int64_t ab = si.atom_begin;
    for (int dz = -si.K[2]; dz <= si.K[2]; ++dz) {
        const int ez = cz + dz;
        const int tz = si.periodic ? floor_div(ez, Mz) : 0;
        if (!si.periodic && (ez < 0 || ez >= Mz)) continue;
        const int bz = ez - tz * Mz;
        for (int dy = -si.K[1]; dy <= si.K[1]; ++dy) {
            const int ey = cy + dy;
            const int ty = si.periodic ? floor_div(ey, My) : 0;
            if (!si.periodic && (ey < 0 || ey >= My)) continue;
            const int by = ey - ty * My;
            const int row = Mx * (by + My * bz);
            const int lo = cx - si.K[0], hi = cx + si.K[0];
            const int tx0 = si.periodic ? floor_div(lo, Mx) : 0;
            const int tx1 = si.periodic ? floor_div(hi, Mx) : 0;
            for (int tx = tx0; tx <= tx1; ++tx) {
                int b0, b1;
                if (si.periodic) {
                    b0 = max(lo, tx * Mx) - tx * Mx;
                    b1 = min(hi, tx * Mx + Mx - 1) - tx * Mx;
                } else {
                    b0 = max(lo, 0);
                    b1 = min(hi, Mx - 1);
                }
                if (b0 > b1) continue;
                const int start = v.bin_start[bb + row + b0];
                const int end = v.bin_start[bb + row + b1 + 1];
                for (int a0 = start; a0 < end; a0 += 32) {
                    const int a = a0 + lane;
                    const bool valid = a < end;
                    const int j = valid ? v.sorted[ab + a] : 0;
                    visit(valid, j, tx, ty, tz);
                }
            }
        }
    }
}

// Accept candidate (j, t) of centre `center`: image shift in range and d2 <= cutoff2.
__device__ __forceinline__ bool accept_candidate(const StructInfo& si, const BinView& v, const double* __restrict__ pos,
                                                 int64_t center, const int* wi, int j, int tx, int ty, int tz,
                                                 double cutoff2, int* n, double& dx, double& dy, double& dz,
                                                 double& d2) {
    const int64_t gj = si.atom_begin + j;
    if (si.periodic) {
        n[0] = tx + wi[0] - v.wrap[3 * gj];
        n[1] = ty + wi[1] - v.wrap[3 * gj + 1];
        n[2] = tz + wi[2] - v.wrap[3 * gj + 2];
        if (abs(n[0]) > si.bounds[0] || abs(n[1]) > si.bounds[1] || abs(n[2]) > si.bounds[2]) return false;
    } else {
        n[0] = n[1] = n[2] = 0;
    }
    d2 = exact_pair(si, pos, center, gj, n[0], n[1], n[2], dx, dy, dz);
    return d2 <= cutoff2;
}

#ifndef MDSOAP_NO_GRAPH_KERNELS
// ---------------------------------------------------------------------------
// Neighbour-graph export: count then fill (warp per centre).
__global__ void graph_count_kernel(const double* __restrict__ pos, BinView v, int64_t atoms, double cutoff2,
                                   int64_t* __restrict__ counts) {
    const int lane = threadIdx.x & 31;
    const int64_t center = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (center >= atoms) return;
    const StructInfo& si = v.info[v.struct_of[center]];
    const int wi[3] = {v.wrap[3 * center], v.wrap[3 * center + 1], v.wrap[3 * center + 2]};
    int64_t total = 0;
    for_each_candidate(si, v, center, lane, [&](bool valid, int j, int tx, int ty, int tz) {
        int n[3];
        double dx, dy, dz, d2;
        const bool ok = valid && accept_candidate(si, v, pos, center, wi, j, tx, ty, tz, cutoff2, n, dx, dy, dz, d2);
        total += __popc(__ballot_sync(0xffffffffu, ok));
    });
    if (lane == 0) counts[center] = total;
}

__global__ void graph_fill_kernel(const double* __restrict__ pos, BinView v, int64_t atoms, double cutoff2,
                                  const int64_t* __restrict__ offsets, int32_t* __restrict__ out_atoms,
                                  int32_t* __restrict__ out_shifts, double* __restrict__ out_disp,
                                  double* __restrict__ out_d2) {
    const int lane = threadIdx.x & 31;
    const int64_t center = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (center >= atoms) return;
    const StructInfo& si = v.info[v.struct_of[center]];
    const int wi[3] = {v.wrap[3 * center], v.wrap[3 * center + 1], v.wrap[3 * center + 2]};
    int64_t cursor = offsets[center];
    const int64_t limit = offsets[center + 1];
    for_each_candidate(si, v, center, lane, [&](bool valid, int j, int tx, int ty, int tz) {
        int n[3];
        double dx, dy, dz, d2;
        const bool ok = valid && accept_candidate(si, v, pos, center, wi, j, tx, ty, tz, cutoff2, n, dx, dy, dz, d2);
        const unsigned mask = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            const int64_t p = cursor + __popc(mask & ((1u << lane) - 1u));
            if (p < limit) {
                out_atoms[p] = (int32_t)(si.atom_begin + j);
                out_shifts[3 * p] = n[0];
                out_shifts[3 * p + 1] = n[1];
                out_shifts[3 * p + 2] = n[2];
                out_disp[3 * p] = dx;
                out_disp[3 * p + 1] = dy;
                out_disp[3 * p + 2] = dz;
                out_d2[p] = d2;
            } else {
                atomicOr(v.error, kErrPairCapacity);
            }
        }
        cursor += __popc(mask);
    });
}
#endif  // MDSOAP_NO_GRAPH_KERNELS

}  // namespace mdsoap
