// soap_center_kernel variants (shapes outside the paired-channel kernel) and
// the structure-average kernels: explicit instantiations of the launchers in
// launchers.cuh.  The variant table in mdsoap.cu names exactly these.
#define MDSOAP_LAUNCH_DEFINITIONS
#define MDSOAP_NO_GRAPH_KERNELS
#include "launchers.cuh"

namespace mdsoap {
namespace launch {

#define MDSOAP_INSTANTIATE_CENTER(T, A, B, C, N, L, MB)                                                     \
    template void center<T, A, B, C, N, L, MB>(dim3, size_t, cudaStream_t, const SoapTables&,             \
                                               const SoapPointers&);                                       \
    template const void* center_symbol<T, A, B, C, N, L, MB>();

MDSOAP_INSTANTIATE_CENTER(4, 7, 0, 0, 8, 3, 3)
MDSOAP_INSTANTIATE_CENTER(8, 7, 0, 0, 8, 3, 2)
MDSOAP_INSTANTIATE_CENTER(3, 9, 1, 0, 8, 4, 3)
MDSOAP_INSTANTIATE_CENTER(6, 9, 1, 0, 8, 4, 2)
MDSOAP_INSTANTIATE_CENTER(4, 13, 5, 0, 8, 6, 2)
MDSOAP_INSTANTIATE_CENTER(2, 17, 9, 1, 8, 8, 2)
MDSOAP_INSTANTIATE_CENTER(1, 41, 0, 0, 32, 20, 1)

#define MDSOAP_INSTANTIATE_STRUCTURE(L)                                                                     \
    template void structure<L>(dim3, size_t, cudaStream_t, const SoapTables&, const int64_t*, int64_t,     \
                               int64_t, const double*, const double*, void*, int64_t);                     \
    template const void* structure_symbol<L>();

MDSOAP_INSTANTIATE_STRUCTURE(0)
MDSOAP_INSTANTIATE_STRUCTURE(1)
MDSOAP_INSTANTIATE_STRUCTURE(2)
MDSOAP_INSTANTIATE_STRUCTURE(3)
MDSOAP_INSTANTIATE_STRUCTURE(4)
MDSOAP_INSTANTIATE_STRUCTURE(5)
MDSOAP_INSTANTIATE_STRUCTURE(6)
MDSOAP_INSTANTIATE_STRUCTURE(8)
MDSOAP_INSTANTIATE_STRUCTURE(20)

}  // namespace launch
}  // namespace mdsoap
