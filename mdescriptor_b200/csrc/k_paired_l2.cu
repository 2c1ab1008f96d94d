// Paired-channel SOAP kernels (expansion, split tails, polynomial basis) for
// l_max = 2: explicit instantiations of the launchers in launchers.cuh.
#define MDSOAP_LAUNCH_DEFINITIONS
#define MDSOAP_NO_GRAPH_KERNELS
#include "launchers.cuh"

namespace mdsoap {
namespace launch {
MDSOAP_INSTANTIATE_PAIRED(2)
}  // namespace launch
}  // namespace mdsoap
