// prefill.cu -- placeholder until the tcgen05 kernel lands.
#include "prefill.cuh"

namespace bml {
cudaError_t launch_prefill(const PrefillArgs &, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace bml
