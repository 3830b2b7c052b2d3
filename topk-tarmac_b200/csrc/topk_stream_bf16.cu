// topk_stream_bf16.cu — bf16 instantiations of the streaming top-k kernel
// (bf16 inputs widened to fp32 on load; fp32 scores and accumulation).
#include "topk_stream.cuh"

namespace tarmac {
cudaError_t launch_topk_stream_bf16(const AttnParams& p, bool tie_high,
                                    cudaStream_t s) {
  return launch_stream_dt<__nv_bfloat16>(p, tie_high, s);
}
}  // namespace tarmac
