// Causal 3-D convolution as an implicit GEMM on tcgen05 (channels-last activations).
#pragma once
#include <cuda_runtime.h>

namespace ddb {

struct Conv3dArgs {
  // input activations, channels-last [B, T, H, W, Cin] bf16 (Cin a multiple of 64)
  const void* x = nullptr;
  int B = 0, T = 0, H = 0, W = 0, Cin = 0;
  // output extents; input coordinate = output coordinate + tap - pad (per dim)
  int To = 0, Ho = 0, Wo = 0;
  int kt = 1, kh = 1, kw = 1;
  int pt = 0, ph = 0, pw = 0;
  int Cout = 0;
  // forward: weights [Cout, kt, kh, kw, Cin] bf16, optional fp32 bias [Cout] and bf16
  // residual [B, To, Ho, Wo, Cout]; output y bf16 [B, To, Ho, Wo, Cout]
  const void* w = nullptr;
  const float* bias = nullptr;
  const void* residual = nullptr;
  void* y = nullptr;
  // weight gradient: dy bf16 [B, To, Ho, Wo, Cout]; dw fp32 [Cout, kt*kh*kw*Cin] is
  // accumulated into (vector reductions), so it must be zeroed by the caller
  const void* dy = nullptr;
  float* dw = nullptr;
  int splits = 0;    // position-range splits for the weight gradient (0 = automatic)
  int max_ctas = 0;  // 0 = one CTA per SM
};

// y = conv(x, w) (+ bias) (+ residual).
void conv3d_fwd(const Conv3dArgs& a, cudaStream_t stream);
// dw += sum over output positions of dy (x) shifted input.
void conv3d_wgrad(const Conv3dArgs& a, cudaStream_t stream);

}  // namespace ddb
