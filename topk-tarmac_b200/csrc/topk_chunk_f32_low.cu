// topk_chunk_f32_low.cu — chunked top-k kernel instantiations: f32 inputs,
// lowest index wins a tie at the k-th score.
#include "topk_chunk.cuh"

namespace tarmac {
cudaError_t launch_topk_chunk_f32_low(const AttnParams& p, cudaStream_t s) {
  return launch_chunk_dt<false, float>(p, s);
}
}  // namespace tarmac
