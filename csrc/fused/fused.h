// Memory-bound fused kernels: AdaLN-RMSNorm, AdamW, casts, rotary backward, reductions.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdexcept>

namespace ddb {

struct AdaLNArgs {
  int M = 0, D = 0;
  const __nv_bfloat16* x = nullptr;
  const float* w = nullptr;          // RMSNorm weight [D]
  const float* mod = nullptr;        // fp32 [groups, ld_mod]
  long ld_mod = 0;
  int scale_off = 0, shift_off = 0;  // column offsets of scale / shift in mod
  int rows_per_group = 1;
  float eps = 1e-6f;
  __nv_bfloat16* h = nullptr;        // fwd output
  float* rstd = nullptr;             // fwd output / bwd input [M]
  const __nv_bfloat16* dh = nullptr; // bwd input
  const __nv_bfloat16* dres = nullptr;  // optional residual gradient added to dx
  __nv_bfloat16* dx = nullptr;
  float* dw = nullptr;               // += column sums
  float* dmod = nullptr;             // += per-group column sums (same layout as mod)
  long ld_dmod = 0;
};

struct LayerNormArgs {
  long M = 0;
  int D = 0;
  float eps = 1e-5f;
  const __nv_bfloat16* x = nullptr;
  const float* w = nullptr;  // [D] or null
  const float* b = nullptr;  // [D] or null
  __nv_bfloat16* y = nullptr;
  float* mean = nullptr;     // [M] fwd output / bwd input
  float* rstd = nullptr;     // [M]
  const __nv_bfloat16* dy = nullptr;
  __nv_bfloat16* dx = nullptr;
  float* dw = nullptr;       // += sum dy * xhat (may be null)
  float* db = nullptr;       // += sum dy (may be null)
};
void layernorm_fwd(const LayerNormArgs& a, cudaStream_t s);
void layernorm_bwd(const LayerNormArgs& a, cudaStream_t s);

struct AugmentArgs {
  int B = 0, T = 0, C = 0, H = 0, W = 0;
  const void* x = nullptr;          // uint8 [B,T,H,W,C] or float [B,T,C,H,W]
  bool input_u8_hwc = false;
  void* y = nullptr;                // [B,T,C,H,W] float32 or bf16
  bool out_bf16 = false;
  const int* flip = nullptr;        // [B] or null
  const float* brightness = nullptr;  // [B] additive, or null
  const float* contrast = nullptr;    // [B] multiplicative, or null
  const float* mean = nullptr;      // [C] or null (no normalisation)
  const float* std = nullptr;       // [C]
};
void video_augment(const AugmentArgs& a, cudaStream_t s);

void adaln_rmsnorm_fwd(const AdaLNArgs& a, cudaStream_t s);
void adaln_rmsnorm_bwd(const AdaLNArgs& a, cudaStream_t s);

struct AdamWArgs {
  float* master = nullptr;
  const float* grad = nullptr;
  float* m = nullptr;
  float* v = nullptr;
  __nv_bfloat16* compute = nullptr;  // bf16 copy written after the update (may be null)
  const float* clip = nullptr;       // device scalar multiplier (grad clipping)
  long n = 0, decay_end = 0;
  float lr = 0, b1 = 0, b2 = 0, eps = 0, wd = 0, bc1 = 1, bc2 = 1, grad_scale = 1;
};
void adamw_flat(const AdamWArgs& a, cudaStream_t s);

void cast_f32_bf16(const float* src, __nv_bfloat16* dst, long n, cudaStream_t s);
// out[0] += sum(x^2)
void sq_norm_f32(const float* x, long n, float* out, cudaStream_t s);
// in-place inverse (or forward) rotation of the first `rot_cols` columns of rows of x
void rope_rotate_bf16(__nv_bfloat16* x, long ld, int M, int rot_cols, const float2* tab,
                      int head_dim, int rows_per_seq, int pos_offset, bool inverse,
                      cudaStream_t s);

}  // namespace ddb
