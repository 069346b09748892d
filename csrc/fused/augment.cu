// Fused video augmentation + normalisation (sm_100a), one pass over the clip.
//
//   y[b,t,c,h,w] = (clamp(contrast_b * (x[b,t,c,h,w'] + bright_b - 0.5) + 0.5, 0, 1)
//                   - mean_c) / std_c,          w' = flip_b ? W-1-w : w
//
// Input is either uint8 channels-last [B, T, H, W, C] (decoded frames, scaled by 1/255)
// or float32 channels-first [B, T, C, H, W] in [0, 1]; output is channels-first float32
// or bf16. Per-clip flip / brightness / contrast come from device arrays, so a batch of
// clips with different parameters is one launch. Replaces the reference's three Triton
// kernels (training/kernels/fused_augment.py:20-196: flip+normalise, flip+brightness/
// contrast, flip+normalise+brightness/contrast) with one kernel and the layout change.
#include <cuda_bf16.h>

#include <algorithm>
#include <stdexcept>

#include "../common/tma.h"
#include "fused.h"

namespace ddb {
namespace {

template <bool U8_HWC, bool BF16_OUT>
__global__ void __launch_bounds__(256) augment_kernel(AugmentArgs a) {
  const long total = static_cast<long>(a.B) * a.T * a.C * a.H * a.W;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < total; i += static_cast<long>(gridDim.x) * 256) {
    const int w = static_cast<int>(i % a.W);
    long r = i / a.W;
    const int h = static_cast<int>(r % a.H);
    r /= a.H;
    const int c = static_cast<int>(r % a.C);
    r /= a.C;
    const long bt = r;  // b * T + t
    const int b = static_cast<int>(bt / a.T);
    const int ws = (a.flip != nullptr && a.flip[b]) ? a.W - 1 - w : w;
    float x;
    if constexpr (U8_HWC) {
      const uint8_t* src = static_cast<const uint8_t*>(a.x);
      x = src[((bt * a.H + h) * a.W + ws) * a.C + c] * (1.f / 255.f);
    } else {
      const float* src = static_cast<const float*>(a.x);
      x = src[((bt * a.C + c) * a.H + h) * a.W + ws];
    }
    if (a.brightness != nullptr || a.contrast != nullptr) {
      const float br = a.brightness ? a.brightness[b] : 0.f;
      const float ct = a.contrast ? a.contrast[b] : 1.f;
      x = fminf(fmaxf(ct * (x + br - 0.5f) + 0.5f, 0.f), 1.f);
    }
    if (a.mean != nullptr) x = (x - a.mean[c]) / a.std[c];
    if constexpr (BF16_OUT)
      static_cast<__nv_bfloat16*>(a.y)[i] = __float2bfloat16(x);
    else
      static_cast<float*>(a.y)[i] = x;
  }
}

}  // namespace

void video_augment(const AugmentArgs& a, cudaStream_t stream) {
  const long total = static_cast<long>(a.B) * a.T * a.C * a.H * a.W;
  if (total <= 0) return;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const int grid = static_cast<int>(std::min<long>((total + 255) / 256, 16L * num_sms(dev)));
  if (a.input_u8_hwc) {
    if (a.out_bf16)
      augment_kernel<true, true><<<grid, 256, 0, stream>>>(a);
    else
      augment_kernel<true, false><<<grid, 256, 0, stream>>>(a);
  } else {
    if (a.out_bf16)
      augment_kernel<false, true><<<grid, 256, 0, stream>>>(a);
    else
      augment_kernel<false, false><<<grid, 256, 0, stream>>>(a);
  }
  count_launch();
  check_cuda(cudaGetLastError(), "augment_kernel launch");
}

}  // namespace ddb
