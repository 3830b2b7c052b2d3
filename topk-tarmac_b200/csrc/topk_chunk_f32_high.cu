// topk_chunk_f32_high.cu — chunked top-k kernel instantiations: f32 inputs,
// highest index wins a tie at the k-th score.
#include "topk_chunk.cuh"

namespace tarmac {
cudaError_t launch_topk_chunk_f32_high(const AttnParams& p, cudaStream_t s) {
  return launch_chunk_dt<true, float>(p, s);
}
}  // namespace tarmac
