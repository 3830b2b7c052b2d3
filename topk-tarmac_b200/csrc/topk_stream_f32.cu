// topk_stream_f32.cu — fp32 instantiations of the streaming top-k kernel.
#include "topk_stream.cuh"

namespace tarmac {
cudaError_t launch_topk_stream_f32(const AttnParams& p, bool tie_high,
                                   cudaStream_t s) {
  return launch_stream_dt<float>(p, tie_high, s);
}
}  // namespace tarmac
