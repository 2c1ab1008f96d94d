// Sparse rows: the feature matrix in CSR form with exact zeros dropped, the
// representation MDescriptor's OutputOptions(sparse=True) asks for
// (src/mdescriptor/core/result.py:64-84, scipy.sparse.csr_matrix of the dense
// rows).  One warp per row, rows in grid-stride order: a count pass, a prefix
// over the row counts, then a fill pass that keeps each row's columns in
// ascending order.  A value v is stored when v != 0 (so -0.0 is dropped and
// NaN kept, as csr_matrix does).
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace mdsoap {

template <class T>
__global__ void csr_count_kernel(const T* __restrict__ dense, int64_t rows, int64_t cols,
                                 int64_t* __restrict__ counts) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
        const T* r = dense + row * cols;
        int c = 0;
        for (int64_t j = lane; j < cols; j += 32) c += r[j] != T(0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        if (lane == 0) counts[row] = c;
    }
}

template <class T>
__global__ void csr_fill_kernel(const T* __restrict__ dense, int64_t rows, int64_t cols,
                                const int64_t* __restrict__ indptr, int32_t* __restrict__ indices,
                                T* __restrict__ data) {
    const int lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
        const T* r = dense + row * cols;
        int64_t base = indptr[row];
        for (int64_t j0 = 0; j0 < cols; j0 += 32) {
            const int64_t j = j0 + lane;
            const T v = j < cols ? r[j] : T(0);
            const bool keep = v != T(0);
            const unsigned mask = __ballot_sync(0xffffffffu, keep);
            if (keep) {
                const int64_t at = base + __popc(mask & below);
                indices[at] = (int32_t)j;
                data[at] = v;
            }
            base += __popc(mask);
        }
    }
}

}  // namespace mdsoap
