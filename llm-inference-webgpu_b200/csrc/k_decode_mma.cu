// Tensor-core split-KV decode (placeholder until the kernel lands).
#include "b2a_internal.cuh"

namespace b2a {
bool attn_mma_supported(const AttnParams&) { return false; }
cudaError_t launch_attn_mma(const AttnParams&, int, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace b2a
