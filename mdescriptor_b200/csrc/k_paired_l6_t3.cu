// Paired-channel SOAP kernels for l_max = 6 with three species register
// banks (three-species plans): explicit instantiations of the launchers in
// launchers.cuh.
#define MDSOAP_LAUNCH_DEFINITIONS
#define MDSOAP_NO_GRAPH_KERNELS
#include "launchers.cuh"

namespace mdsoap {
namespace launch {
MDSOAP_INSTANTIATE_PAIRED_BANKS(3, 6)
}  // namespace launch
}  // namespace mdsoap
