// MoE routing / permutation / combine kernels (see moe.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace ddb {

struct MoeRouteArgs {
  const float* logits = nullptr;  // [N, ld_logits]: E routed, then ns shared-gate logits
  long ld_logits = 0;
  const float* bias = nullptr;    // [E] load-balancing bias (may be null)
  int N = 0, E = 0, k = 0, ns = 0;
  int* topk_idx = nullptr;        // [N, k]
  float* topk_w = nullptr;        // [N, k] renormalised
  float* shared_w = nullptr;      // [N, ns]
  float* probs = nullptr;         // [N, E] (optional, for the router backward)
  int* counts = nullptr;          // [E] += tokens per expert
  float* psum = nullptr;          // [E] += sum of probabilities
};

struct MoeCombineArgs {
  int N = 0, d = 0, k = 0, ns = 0;
  const float* topk_w = nullptr;
  const float* shared_w = nullptr;
  const int* slot_of = nullptr;        // [N, k + ns]
  const __nv_bfloat16* y = nullptr;    // permuted expert outputs
  long ld_y = 0;
  const __nv_bfloat16* residual = nullptr;
  long ld_res = 0;
  __nv_bfloat16* out = nullptr;
  long ld_out = 0;
};

void moe_route(const MoeRouteArgs& a, cudaStream_t s);
void moe_plan(const int* counts, int E, int ns, int N, int* seg_start, int* seg_count,
              int* tile_expert, int* tile_row, int* total_mtiles, int* kstart, int* kend,
              int* cursor, int max_mtiles, cudaStream_t s);
void moe_dispatch(const __nv_bfloat16* x, long ldx, int N, int d, int k, int ns, int E,
                  const int* topk_idx, const int* seg_start, const int* seg_count, int* cursor,
                  __nv_bfloat16* xp, long ldp, int* slot_of, cudaStream_t s);
void moe_combine(const MoeCombineArgs& a, cudaStream_t s);
void moe_combine_bwd(const MoeCombineArgs& a, const __nv_bfloat16* dout, long ld_dout,
                     __nv_bfloat16* dy, float* dw, cudaStream_t s);
void moe_unpermute(const __nv_bfloat16* dxp, long ldp, const int* slot_of, int N, int R, int d,
                   __nv_bfloat16* dx, long ldx, cudaStream_t s);

}  // namespace ddb
