// Row kernels without the list paths (calls with list_max = 0) for ES_F64
// logits, in a translation unit of their own (see launch_rows_full).
#include "es_kernel.cuh"

namespace es {
template <> cudaError_t launch_rows_full<ES_F64>(const Params& p, int cluster, cudaStream_t stream) {
  return launch_family<ES_F64, false>(p, cluster, stream);
}
}  // namespace es
