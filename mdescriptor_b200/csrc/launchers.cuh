// Host-side launchers of the SOAP centre, tail and structure kernels.
//
// The host runtime (mdsoap.cu) sees only the declarations below and takes the
// launchers' addresses for its variant tables.  The definitions are compiled,
// with one explicit instantiation per kernel the tables name, in the kernel
// translation units k_*.cu (MDSOAP_LAUNCH_DEFINITIONS), so that the template
// instantiations build in parallel instead of in one translation unit.
#pragma once

#include "soap_paired.cuh"

namespace mdsoap {
namespace launch {

using CenterLauncher = void (*)(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);
using StructureLauncher = void (*)(dim3, size_t, cudaStream_t, const SoapTables&, const int64_t*, int64_t, int64_t,
                                   const double*, const double*, void*, int64_t);

// soap_center_kernel (one warp per centre, any n_max <= 32, l_max <= 20).
template <int MAXT, int L0, int L1, int L2, int NMAX, int LMAX, int MINB>
void center(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p);
template <int MAXT, int L0, int L1, int L2, int NMAX, int LMAX, int MINB>
const void* center_symbol();

// Paired-channel kernel, l_max == L exactly; plans with a split tail launch
// the instantiation without tail code (fewer registers).
template <int T, int L, bool PRECISE, int MINB>
void paired(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p);
template <int T, int L, bool PRECISE, int MINB>
const void* paired_symbol();
template <int T, int L, bool PRECISE, int MINB>
const void* paired_split_symbol();

// Edge-list split of the SPLIT path: the walk-only kernel (no channel code,
// one instantiation per accuracy) and the expansion-only kernel.
constexpr int kWalkMinBlocks = 4;
template <bool PRECISE>
void paired_walk(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p);
template <bool PRECISE>
const void* paired_walk_symbol();
template <int T, int L, bool PRECISE, int MINB>
void paired_expand(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p);
template <int T, int L, bool PRECISE, int MINB>
const void* paired_expand_symbol();

// Polynomial radial basis: the paired kernel's POLY instantiation
// (full-accuracy radial factors, tail fused).
template <int T, int L>
void poly(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p);
template <int T, int L>
const void* poly_symbol();

// Split tails of the paired kernel.
template <int L, int T>
void tail(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p);
template <int L, int T>
const void* tail_symbol();
template <int L>
void tail_generic(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p);
template <int L>
const void* tail_generic_symbol();

// Structure-level averages.
template <int LMAX>
void structure(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const int64_t* offsets,
               int64_t s0, int64_t s1, const double* cbuf, const double* pbuf, void* out, int64_t row0);
template <int LMAX>
const void* structure_symbol();

#ifdef MDSOAP_LAUNCH_DEFINITIONS

template <int MAXT, int L0, int L1, int L2, int NMAX, int LMAX, int MINB>
void center(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p) {
    soap_center_kernel<MAXT, L0, L1, L2, NMAX, LMAX, MINB><<<grid, kWarps * 32, smem, stream>>>(tab, p);
}
template <int MAXT, int L0, int L1, int L2, int NMAX, int LMAX, int MINB>
const void* center_symbol() {
    return reinterpret_cast<const void*>(&soap_center_kernel<MAXT, L0, L1, L2, NMAX, LMAX, MINB>);
}

template <int T, int L, bool PRECISE, int MINB>
void paired(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p) {
    if (tab.split_tail)
        soap_paired_kernel<T, L, PRECISE, MINB, true><<<grid, kWarps * 32, smem, stream>>>(tab, p);
    else
        soap_paired_kernel<T, L, PRECISE, MINB, false><<<grid, kWarps * 32, smem, stream>>>(tab, p);
}
template <int T, int L, bool PRECISE, int MINB>
const void* paired_symbol() {
    return reinterpret_cast<const void*>(&soap_paired_kernel<T, L, PRECISE, MINB, false>);
}
template <int T, int L, bool PRECISE, int MINB>
const void* paired_split_symbol() {
    return reinterpret_cast<const void*>(&soap_paired_kernel<T, L, PRECISE, MINB, true>);
}

template <bool PRECISE>
void paired_walk(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p) {
    soap_paired_kernel<1, 0, PRECISE, kWalkMinBlocks, true, false, 1><<<grid, kWarps * 32, smem, stream>>>(tab, p);
}
template <bool PRECISE>
const void* paired_walk_symbol() {
    return reinterpret_cast<const void*>(&soap_paired_kernel<1, 0, PRECISE, kWalkMinBlocks, true, false, 1>);
}
template <int T, int L, bool PRECISE, int MINB>
void paired_expand(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p) {
    soap_paired_kernel<T, L, PRECISE, MINB, true, false, 2><<<grid, kWarps * 32, smem, stream>>>(tab, p);
}
template <int T, int L, bool PRECISE, int MINB>
const void* paired_expand_symbol() {
    return reinterpret_cast<const void*>(&soap_paired_kernel<T, L, PRECISE, MINB, true, false, 2>);
}

template <int T, int L>
void poly(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p) {
    soap_paired_kernel<T, L, true, 2, false, true><<<grid, kWarps * 32, smem, stream>>>(tab, p);
}
template <int T, int L>
const void* poly_symbol() {
    return reinterpret_cast<const void*>(&soap_paired_kernel<T, L, true, 2, false, true>);
}

template <int L, int T>
void tail(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p) {
    soap_tail_kernel<L, T><<<grid, kWarps * 32, smem, stream>>>(tab, p);
}
template <int L, int T>
const void* tail_symbol() {
    return reinterpret_cast<const void*>(&soap_tail_kernel<L, T>);
}
template <int L>
void tail_generic(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const SoapPointers& p) {
    soap_tail_generic_kernel<L><<<grid, kWarps * 32, smem, stream>>>(tab, p);
}
template <int L>
const void* tail_generic_symbol() {
    return reinterpret_cast<const void*>(&soap_tail_generic_kernel<L>);
}

template <int LMAX>
void structure(dim3 grid, size_t smem, cudaStream_t stream, const SoapTables& tab, const int64_t* offsets,
               int64_t s0, int64_t s1, const double* cbuf, const double* pbuf, void* out, int64_t row0) {
    soap_structure_kernel<LMAX><<<grid, kWarps * 32, smem, stream>>>(tab, offsets, s0, s1, cbuf, pbuf, out, row0);
}
template <int LMAX>
const void* structure_symbol() {
    return reinterpret_cast<const void*>(&soap_structure_kernel<LMAX>);
}

// Explicit instantiations of every launcher of one paired l_max.
#define MDSOAP_INSTANTIATE_PAIRED(L)                                                                              \
    template void paired<4, L, false, 2>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);    \
    template void paired<4, L, true, 2>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);     \
    template const void* paired_symbol<4, L, false, 2>();                                                         \
    template const void* paired_symbol<4, L, true, 2>();                                                          \
    template const void* paired_split_symbol<4, L, false, 2>();                                                   \
    template const void* paired_split_symbol<4, L, true, 2>();                                                    \
    template void paired_expand<1, L, false, 3>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&); \
    template void paired_expand<2, L, true, 3>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&); \
    template const void* paired_expand_symbol<1, L, false, 3>();                                                  \
    template const void* paired_expand_symbol<2, L, true, 3>();                                                   \
    template void poly<4, L>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);                \
    template const void* poly_symbol<4, L>();                                                                     \
    template void tail<L, 4>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);                \
    template const void* tail_symbol<L, 4>();                                                                     \
    template void tail_generic<L>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);           \
    template const void* tail_generic_symbol<L>();

// Expansion kernels and the register tail with T species register banks
// (plans with fewer species than the default four banks).
#define MDSOAP_INSTANTIATE_PAIRED_BANKS(T, L)                                                                     \
    template void paired<T, L, false, 2>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);    \
    template void paired<T, L, true, 2>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);     \
    template const void* paired_symbol<T, L, false, 2>();                                                         \
    template const void* paired_symbol<T, L, true, 2>();                                                          \
    template const void* paired_split_symbol<T, L, false, 2>();                                                   \
    template const void* paired_split_symbol<T, L, true, 2>();                                                    \
    template void tail<L, T>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);                \
    template const void* tail_symbol<L, T>();

#endif  // MDSOAP_LAUNCH_DEFINITIONS

}  // namespace launch
}  // namespace mdsoap
