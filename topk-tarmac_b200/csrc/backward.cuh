// backward.cuh — operand block and launchers of the gradient kernels
// (backward.cu).
#pragma once

#include "common.cuh"

namespace tarmac {

struct BwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* o;     // forward output (dense only)
  const void* g;     // dL/dout
  int64_t qb, qn, kb, kn, vb, vn, ob, on, gb, gn;
  int B, N, d;
  float scale;
  float* dq;
  float* dk;
  float* dv;
  float* work;       // dense: [2][B][N] row log-sum-exp (base 2), then D
  const void* idx;   // gather: [B, N, kk]
  int idx_i64;
  int kk;
  int vec;           // 4-element vector loads of q, k, v, o, g
};

cudaError_t launch_gather_bwd(const BwdParams& p, int bf16, cudaStream_t s);
cudaError_t launch_dense_bwd(const BwdParams& p, int bf16, cudaStream_t s);

}  // namespace tarmac
