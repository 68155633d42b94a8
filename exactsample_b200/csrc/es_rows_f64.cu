// Row kernel instantiation for ES_F64 logits (one dtype per translation unit,
// so the four compile in parallel).
#include "es_kernel.cuh"

namespace es {
template cudaError_t launch_rows<ES_F64>(const Params&, int, cudaStream_t);
template cudaError_t launch_reference<ES_F64>(const Params&, cudaStream_t);
}  // namespace es
