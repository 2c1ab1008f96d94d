// Walk-only instantiations of the paired kernel (edge-list split of the
// SPLIT path): explicit instantiations of the launchers in launchers.cuh.
#define MDSOAP_LAUNCH_DEFINITIONS
#define MDSOAP_NO_GRAPH_KERNELS
#include "launchers.cuh"

namespace mdsoap {
namespace launch {
template void paired_walk<false>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);
template void paired_walk<true>(dim3, size_t, cudaStream_t, const SoapTables&, const SoapPointers&);
template const void* paired_walk_symbol<false>();
template const void* paired_walk_symbol<true>();
}  // namespace launch
}  // namespace mdsoap
