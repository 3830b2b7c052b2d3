// comm.cuh — operand block and launcher of the fused communication-module
// kernel (comm.cu).
#pragma once

#include "common.cuh"

namespace tarmac {

struct CommParams {
  const float* x;        // [B, N, in_dim] contiguous
  const float* wqkv;     // [3m, in_dim]
  const float* bqkv;     // [3m]
  const float* wproj;    // [m, m]
  const float* bproj;    // [m]
  float* out;            // [B, N, m]
  int B, N, in_dim, m;
  int topk;              // 0: dense
  float scale;           // 1/sqrt(m)
  int w_smem;            // W_qkv staged in shared memory (set by the launcher)
};

cudaError_t launch_comm_forward(const CommParams& p, cudaStream_t s);
// dynamic shared memory without the staged W_qkv
size_t comm_smem_bytes(int N, int in_dim, int m, int MP, bool vec);
// x and W_qkv rows move as 16-byte pieces
bool comm_vec(const float* x, const float* wqkv, int in_dim);
int comm_padded_m(int m);

}  // namespace tarmac
