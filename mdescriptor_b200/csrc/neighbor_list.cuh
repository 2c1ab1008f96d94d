// The NeighborList descriptor on the GPU (sm_100a): pair records in the
// reference CPU graph's own order.
//
// Reference: compute_neighbor_list (cpp/src/standalone/neighbor_list.cpp:15-75)
// over build_neighbor_graph (cpp/src/common/neighbor.cpp:423-608, 703-768).
// The pair SET and the fp64 displacement bits come from the cell-binned walk
// and accept_candidate (neighbors.cuh), exactly as for SOAP.  The ORDER is the
// reference's: it scans, for each centre, the 3 x 3 x 3 cells of a grid built
// over the image-expanded structure (z, then y, then x, i.e. ascending cell
// index) and, inside a cell, the expanded atoms in expansion order (image
// n0 -> n1 -> n2, then atom).  So within a centre the reference order is
// ascending (cell index of the neighbour image, expansion index), and each
// centre's accepted pairs are sorted by that 64-bit key in shared memory
// before they are written.  The grid (bounding box of the expanded atoms
// padded by 1e-10, dimension max(1, int(range / cutoff)) and spacing
// max(cutoff, range / dimension) per axis, neighbor.cpp:135-194) is rebuilt
// per structure with the reference's arithmetic; its bounding box needs no
// expanded list, because rounding is monotonic: the smallest image coordinate
// of an atom is x + (smallest shift component).
#pragma once

#include "neighbors.cuh"

namespace mdsoap {

constexpr int kListCapacity = 2048;  // pairs of one centre sorted in shared memory

struct CanonGrid {
    double minimum[3];
    double spacing[3];
    int32_t dims[3];
    int32_t images[3];  // 2 b + 1 per axis (1 for isolated structures)
};

// Per structure (one CTA of 256 threads): the reference cell grid.
__global__ void canon_grid_kernel(DeviceBatch b, BinView v, double cutoff, CanonGrid* __restrict__ grids) {
    const int64_t s = blockIdx.x;
    const StructInfo& si = v.info[s];
    const int64_t begin = b.offsets[s], count = b.offsets[s + 1] - begin;
    const int tid = threadIdx.x;
    __shared__ double red[6][8];
    int bnd[3] = {0, 0, 0};
    if (si.periodic)
        for (int c = 0; c < 3; ++c) bnd[c] = si.bounds[c];
    const int64_t nimg = (int64_t)(2 * bnd[0] + 1) * (2 * bnd[1] + 1) * (2 * bnd[2] + 1);
    // The reference numbers expanded atoms in int32 (neighbor.cpp:139-141).
    if (tid == 0 && nimg * count > 2147483647LL) atomicOr(v.error, kErrExtendedRange);
    // Extreme shift components over the images: ((n0 a0 + n1 a1) + n2 a2), neighbor.cpp:471-474.
    double smin[3] = {INFINITY, INFINITY, INFINITY}, smax[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int64_t r = tid; r < nimg; r += blockDim.x) {
        const int n2 = (int)(r % (2 * bnd[2] + 1)) - bnd[2];
        const int n1 = (int)((r / (2 * bnd[2] + 1)) % (2 * bnd[1] + 1)) - bnd[1];
        const int n0 = (int)(r / ((int64_t)(2 * bnd[2] + 1) * (2 * bnd[1] + 1))) - bnd[0];
        for (int c = 0; c < 3; ++c) {
            const double sc = si.periodic ? __dadd_rn(__dadd_rn(__dmul_rn((double)n0, si.cell[c]),
                                                                __dmul_rn((double)n1, si.cell[3 + c])),
                                                      __dmul_rn((double)n2, si.cell[6 + c]))
                                          : 0.0;
            smin[c] = fmin(smin[c], sc);
            smax[c] = fmax(smax[c], sc);
        }
    }
    auto block_reduce = [&](double (&lo)[3], double (&hi)[3]) {
        for (int c = 0; c < 3; ++c)
            for (int o = 16; o > 0; o >>= 1) {
                lo[c] = fmin(lo[c], __shfl_xor_sync(0xffffffffu, lo[c], o));
                hi[c] = fmax(hi[c], __shfl_xor_sync(0xffffffffu, hi[c], o));
            }
        __syncthreads();
        if ((tid & 31) == 0)
            for (int c = 0; c < 3; ++c) {
                red[c][tid >> 5] = lo[c];
                red[3 + c][tid >> 5] = hi[c];
            }
        __syncthreads();
        for (int c = 0; c < 3; ++c) {
            lo[c] = INFINITY;
            hi[c] = -INFINITY;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
                lo[c] = fmin(lo[c], red[c][w]);
                hi[c] = fmax(hi[c], red[3 + c][w]);
            }
        }
    };
    block_reduce(smin, smax);
    // Bounding box of the expanded atoms.
    double lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int64_t a = tid; a < count; a += blockDim.x)
        for (int c = 0; c < 3; ++c) {
            const double x = b.positions[3 * (begin + a) + c];
            lo[c] = fmin(lo[c], si.periodic ? __dadd_rn(x, smin[c]) : x);
            hi[c] = fmax(hi[c], si.periodic ? __dadd_rn(x, smax[c]) : x);
        }
    block_reduce(lo, hi);
    if (tid == 0) {
        CanonGrid g;
        for (int c = 0; c < 3; ++c) {
            g.images[c] = 2 * bnd[c] + 1;
            if (count == 0) {
                g.minimum[c] = 0.0;
                g.spacing[c] = cutoff;
                g.dims[c] = 1;
                continue;
            }
            const double mn = __dsub_rn(lo[c], 1e-10), mx = __dadd_rn(hi[c], 1e-10);
            const double range = __dsub_rn(mx, mn);
            const double cells = __ddiv_rn(range, cutoff);
            if (!isfinite(range) || range < 0.0 || !isfinite(cells) || cells > 2147483647.0) {
                atomicOr(v.error, kErrWrapRange);
                g.dims[c] = 1;
            } else {
                g.dims[c] = max(1, (int)cells);
            }
            g.minimum[c] = mn;
            g.spacing[c] = fmax(cutoff, __ddiv_rn(range, (double)g.dims[c]));
        }
        if ((double)g.dims[0] * g.dims[1] * g.dims[2] >= 4294967296.0) atomicOr(v.error, kErrWrapRange);
        grids[s] = g;
    }
}

// CellGrid::coordinate (neighbor.cpp:122-132).
__device__ __forceinline__ int canon_coordinate(double value, double origin, double width, int dimension) {
    const double scaled = __ddiv_rn(__dsub_rn(value, origin), width);
    if (!(scaled > 0.0)) return 0;
    if (!isfinite(scaled) || scaled >= (double)dimension) return dimension - 1;
    return (int)scaled;
}

// keep_half_neighbor (cpp/include/mdescriptor/detail/neighbor_filter.hpp:16-36).
__device__ __forceinline__ bool keep_half(int64_t center, int64_t atom, int sx, int sy, int sz) {
    if (atom != center) return atom > center;
    if (sx != 0) return sx > 0;
    if (sy != 0) return sy > 0;
    if (sz != 0) return sz > 0;
    return true;
}

// Whether accepted pair (centre, local j, image n) is listed.
__device__ __forceinline__ bool list_pair(int64_t center, int64_t gj, const int* n, bool full, bool self_pairs) {
    const bool self = gj == center && n[0] == 0 && n[1] == 0 && n[2] == 0;
    if (!self_pairs && self) return false;
    return full || keep_half(center, gj, n[0], n[1], n[2]);
}

// Pass 1: listed pairs per centre (warp per centre).
__global__ void list_count_kernel(const double* __restrict__ pos, BinView v, int64_t atoms, double cutoff2, int full,
                                  int self_pairs, int64_t* __restrict__ counts) {
    const int lane = threadIdx.x & 31;
    const int64_t center = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (center >= atoms) return;
    const StructInfo& si = v.info[v.struct_of[center]];
    const int wi[3] = {v.wrap[3 * center], v.wrap[3 * center + 1], v.wrap[3 * center + 2]};
    int64_t total = 0;
    for_each_candidate(si, v, center, lane, [&](bool valid, int j, int tx, int ty, int tz) {
        int n[3];
        double dx, dy, dz, d2;
        const bool ok = valid && accept_candidate(si, v, pos, center, wi, j, tx, ty, tz, cutoff2, n, dx, dy, dz, d2) &&
                        list_pair(center, si.atom_begin + j, n, full != 0, self_pairs != 0);
        total += __popc(__ballot_sync(0xffffffffu, ok));
    });
    if (lane == 0) counts[center] = total;
}

// Pass 2: collect each centre's keys, sort them in the reference order,
// recompute every pair from its key and write its record:
//   records [row][5] = centre, atom (batch indices), image shift (as doubles);
//   values  [row][4] = dx, dy, dz, sqrt(max(0, d2))   (neighbor_list.cpp:44-54).
__global__ void list_fill_kernel(const double* __restrict__ pos, BinView v, const CanonGrid* __restrict__ grids,
                                 int64_t atoms, double cutoff2, int full, int self_pairs,
                                 const int64_t* __restrict__ row_offsets, double* __restrict__ records,
                                 double* __restrict__ values) {
    extern __shared__ unsigned long long list_keys[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t center = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (center >= atoms) return;
    unsigned long long* keys = list_keys + (size_t)warp * kListCapacity;
    const int s = v.struct_of[center];
    const StructInfo& si = v.info[s];
    const CanonGrid& g = grids[s];
    const int wi[3] = {v.wrap[3 * center], v.wrap[3 * center + 1], v.wrap[3 * center + 2]};
    const int64_t row0 = row_offsets[center];
    const int count = (int)(row_offsets[center + 1] - row0);
    if (count > kListCapacity) {
        if (lane == 0) atomicOr(v.error, kErrPairCapacity);
        return;
    }
    const int b0 = (g.images[0] - 1) / 2, b1 = (g.images[1] - 1) / 2, b2 = (g.images[2] - 1) / 2;
    int filled = 0;
    for_each_candidate(si, v, center, lane, [&](bool valid, int j, int tx, int ty, int tz) {
        int n[3];
        double dx, dy, dz, d2;
        const bool ok = valid && accept_candidate(si, v, pos, center, wi, j, tx, ty, tz, cutoff2, n, dx, dy, dz, d2) &&
                        list_pair(center, si.atom_begin + j, n, full != 0, self_pairs != 0);
        const unsigned mask = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            // Image position exactly as the reference expands it, then its cell.
            double img[3];
            {
                const int64_t gj = si.atom_begin + j;
                for (int c = 0; c < 3; ++c) img[c] = pos[3 * gj + c];
                if (si.periodic) {
                    const double f0 = (double)n[0], f1 = (double)n[1], f2 = (double)n[2];
                    for (int c = 0; c < 3; ++c)
                        img[c] = __dadd_rn(img[c], __dadd_rn(__dadd_rn(__dmul_rn(f0, si.cell[c]),
                                                                        __dmul_rn(f1, si.cell[3 + c])),
                                                              __dmul_rn(f2, si.cell[6 + c])));
                }
            }
            const int cx = canon_coordinate(img[0], g.minimum[0], g.spacing[0], g.dims[0]);
            const int cy = canon_coordinate(img[1], g.minimum[1], g.spacing[1], g.dims[1]);
            const int cz = canon_coordinate(img[2], g.minimum[2], g.spacing[2], g.dims[2]);
            const unsigned long long cell =
                (unsigned long long)cx + (unsigned long long)g.dims[0] * ((unsigned long long)cy +
                                                                          (unsigned long long)g.dims[1] * cz);
            const unsigned long long replica =
                ((unsigned long long)(n[0] + b0) * g.images[1] + (unsigned long long)(n[1] + b1)) * g.images[2] +
                (unsigned long long)(n[2] + b2);
            const unsigned long long ext = replica * (unsigned long long)si.atom_count + (unsigned long long)j;
            const int q = filled + __popc(mask & ((1u << lane) - 1u));
            if (q < kListCapacity) keys[q] = (cell << 32) | (ext & 0xffffffffull);
        }
        filled += __popc(mask);
    });
    if (filled != count) {  // the two passes disagree: never expected
        if (lane == 0) atomicOr(v.error, kErrPairCapacity);
        return;
    }
    // Bitonic sort of keys[0, P) with P = next power of two >= count (padding = max key).
    int P = 1;
    while (P < count) P <<= 1;
    for (int i = count + lane; i < P; i += 32) keys[i] = ~0ull;
    __syncwarp();
    for (int k = 2; k <= P; k <<= 1) {
        for (int jj = k >> 1; jj > 0; jj >>= 1) {
            for (int i = lane; i < P; i += 32) {
                const int partner = i ^ jj;
                if (partner > i) {
                    const unsigned long long a = keys[i], c = keys[partner];
                    const bool up = (i & k) == 0;
                    if ((a > c) == up) {
                        keys[i] = c;
                        keys[partner] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
    // Records in sorted order, each pair recomputed from its key.
    const int64_t atoms_s = si.atom_count;
    for (int r = lane; r < count; r += 32) {
        const unsigned long long ext = keys[r] & 0xffffffffull;
        const int64_t j = (int64_t)(ext % (unsigned long long)atoms_s);
        const int64_t replica = (int64_t)(ext / (unsigned long long)atoms_s);
        const int n2 = (int)(replica % g.images[2]) - b2;
        const int n1 = (int)((replica / g.images[2]) % g.images[1]) - b1;
        const int n0 = (int)(replica / ((int64_t)g.images[2] * g.images[1])) - b0;
        double dx, dy, dz;
        const int64_t gj = si.atom_begin + j;
        const double d2 = exact_pair(si, pos, center, gj, n0, n1, n2, dx, dy, dz);
        double* rec = records + (row0 + r) * 5;
        rec[0] = (double)center;
        rec[1] = (double)gj;
        rec[2] = (double)n0;
        rec[3] = (double)n1;
        rec[4] = (double)n2;
        double* val = values + (row0 + r) * 4;
        val[0] = dx;
        val[1] = dy;
        val[2] = dz;
        val[3] = sqrt(fmax(0.0, d2));
    }
}

}  // namespace mdsoap
