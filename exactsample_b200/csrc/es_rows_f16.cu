// Row kernel instantiation for ES_F16 logits (one dtype per translation unit,
// so the four compile in parallel).
#include "es_kernel.cuh"

namespace es {
template cudaError_t launch_rows<ES_F16>(const Params&, int, cudaStream_t);
template cudaError_t launch_reference<ES_F16>(const Params&, cudaStream_t);
}  // namespace es
