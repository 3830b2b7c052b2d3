// topk_chunk_bf16_high.cu — chunked top-k kernel instantiations: bf16 inputs,
// highest index wins a tie at the k-th score.
#include "topk_chunk.cuh"

namespace tarmac {
cudaError_t launch_topk_chunk_bf16_high(const AttnParams& p, cudaStream_t s) {
  return launch_chunk_dt<true, __nv_bfloat16>(p, s);
}
}  // namespace tarmac
