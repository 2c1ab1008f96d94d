// Shared device-side definitions of the mdsoap engine (sm_100a).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

namespace mdsoap {

constexpr int kMaxSpecies = 64;
constexpr int kMaxL = 20;
constexpr int kMaxN = 32;
constexpr int kMaxGrid = 128;  // polynomial basis quadrature nodes
constexpr int kWarps = 4;             // warps per CTA of the centre kernel
constexpr int kPending = 64;          // accepted-edge queue per warp (>= 2 * 32)
constexpr int kRegionHeader = 544;    // per-warp candidate tables + chunk permutation (bytes)
constexpr int kTri = (kMaxL + 1) * (kMaxL + 2) / 2;

// Bits of the per-device error word that kernels raise instead of trapping.
enum DeviceError : unsigned {
    kErrUnknownSpecies = 1u,   // an atomic number outside the plan's species
    kErrWrapRange = 2u,        // fractional coordinate beyond the int32 image range
    kErrMixedPbc = 4u,         // pbc neither all 0 nor all 1
    kErrSingularCell = 8u,     // |det(cell)| < 1e-14 for a periodic structure
    kErrPairCapacity = 16u,    // neighbour CSR fill overran its counted capacity
    kErrExtendedRange = 32u,   // image-expanded structure beyond int32 atom indices
    kErrTailTimeout = 64u,     // a tail kernel's bulk copy did not complete within its time limit
};

// Per-structure geometry and binning plan, written by bin_structures_kernel.
// Periodic structures are binned in lattice (fractional) coordinates, isolated
// ones in their bounding box; bins of one structure are numbered
// x + Mx (y + My z) and their atom lists are contiguous in `sorted`.
struct StructInfo {
    double cell[9];      // lattice vectors as rows
    double inv[9];       // inverse cell (math3.hpp:52-68 arithmetic)
    double origin[3];    // isolated: bounding-box minimum
    double extent[3];    // isolated: bounding-box extent
    int32_t periodic;
    int32_t bounds[3];   // periodic image range [-b, b] (neighbor.cpp:459-467)
    int32_t M[3];        // bins per axis
    int32_t K[3];        // bin search half-width per axis
    int64_t atom_begin;
    int32_t atom_count;
    int32_t aligned;     // bins are axis-aligned boxes origin + [b, b+1) * extent / M (isolated, or
                         // periodic with a diagonal cell of positive entries)
    int64_t bin_base;    // first bin_start entry of this structure
    double pre_cut2;     // prefilter radius^2: cutoff plus a margin far above fp64 rounding of any displacement
    double in_cut2;      // inner radius^2: cutoff minus the same margin; an approximate d^2 below it implies the
                         // reference's exact d^2 is within the cutoff
};

struct BinView {
    StructInfo* info;        // [structures]
    int32_t* struct_of;      // [atoms]
    int32_t* type;           // [atoms] species index, -1 if unknown
    int32_t* bin_of;         // [atoms] bin index within the structure
    int32_t* wrap;           // [atoms*3] floor of the fractional coordinates (periodic)
    int32_t* sorted;         // [atoms] structure-local atom ids grouped by bin
    int32_t* bin_start;      // [2*atoms + 8*structures] bin offsets (+1 sentinel per structure)
    int32_t* bin_cursor;     // same size, scatter cursors
    unsigned* error;         // device error word
    double4* spos;           // [atoms] in `sorted` order: wrapped position (x, y, z) and
                             // w = the int64 128 * local atom id + species index + 1,
                             // its bits stored as they are (__longlong_as_double);
                             // may be null (then not written)
};

// Capacity of the bin table of a structure with `atoms` atoms: its bin count
// is capped at 2*atoms + 7 so that bin_base has the closed form below.
__host__ __device__ inline int64_t bin_base_of(int64_t atom_begin, int64_t structure) {
    return 2 * atom_begin + 8 * structure;
}
__host__ __device__ inline int64_t bin_capacity(int64_t atoms) { return 2 * atoms + 7; }

__device__ __forceinline__ int floor_div(int a, int b) {
    const int q = a / b;
    return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

__device__ __forceinline__ int tri(int l, int m) { return l * (l + 1) / 2 + m; }

// Compile-time loop: f(std::integral_constant<int, I>) for I in [I0, N).
template <int I0, int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
    if constexpr (I0 < N) {
        f(std::integral_constant<int, I0>{});
        static_for<I0 + 1, N>(f);
    }
}

// Coefficient block layout: [l][t][n][m] with each (t, n) row padded to
// 2l+2 doubles; block l starts at S n l (l+1).
__device__ __forceinline__ int cblock(int S, int n, int l) { return S * n * l * (l + 1); }

// Feature offset of (t1, n1, t2, n2, l) in the compression-off layout
// (t1 <= t2, then l, then n1, then n2 with n2 >= n1 when t1 == t2).
__device__ __forceinline__ int64_t pair_base(int S, int n, int L, int t1, int t2) {
    const int64_t T = (int64_t)n * (n + 1) / 2;
    const int64_t nn = (int64_t)n * n;
    int64_t base = (int64_t)(L + 1) * (t1 * T + nn * ((int64_t)t1 * (S - 1) - (int64_t)t1 * (t1 - 1) / 2));
    if (t2 > t1) base += (int64_t)(L + 1) * (T + (int64_t)(t2 - t1 - 1) * nn);
    return base;
}

}  // namespace mdsoap
