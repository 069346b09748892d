// GroupNorm (+ SiLU) forward/backward for channels-last activations [B, P, C].
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ddb {

struct GroupNormArgs {
  int B = 0, C = 0, G = 0;
  long P = 0;               // positions per sample (T*H*W)
  float eps = 1e-5f;
  bool silu = true;
  const __nv_bfloat16* x = nullptr;
  const float* w = nullptr;  // [C]
  const float* b = nullptr;  // [C] or null
  __nv_bfloat16* y = nullptr;
  float* stats = nullptr;    // [B, G, 2] (mean, rstd): written by fwd, read by bwd
  double* acc = nullptr;     // [B, C, 2] scratch (fwd: sum x, x^2; bwd: sum dpre, dpre*xhat)
  // backward
  const __nv_bfloat16* dy = nullptr;
  __nv_bfloat16* dx = nullptr;
  float* coef = nullptr;     // [B, G, 2] scratch
};

void groupnorm_fwd(const GroupNormArgs& a, cudaStream_t stream);
// dx; per-channel sums (dbias, dweight per sample) are left in acc for the caller.
void groupnorm_bwd(const GroupNormArgs& a, cudaStream_t stream);

}  // namespace ddb
