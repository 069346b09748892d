// SLA routing and linear-branch kernels (see sla.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ddb {

struct SlaRouteArgs {
  const float* qm = nullptr;   // [B*H, nb, 64] block means of q
  const float* km = nullptr;
  int nb = 0;                  // 64-token blocks per sequence
  int topk = 1;
  int causal = 1;              // 0 none, 1 frame, 2 token (block granularity)
  int bpf = 1;                 // blocks per frame
  int always_diag = 1;
  uint32_t* sel_bits = nullptr;   // [B*H, nb, nb/32] (optional)
  __nv_bfloat16* wlin = nullptr;  // [B*H, nb, nb]: valid & ~selected (optional)
  int* pair_blocks = nullptr;     // [B*H*nb/2, max_pairs]
  uint8_t* pair_mask = nullptr;
  int* pair_count = nullptr;      // [B*H*nb/2]
  int max_pairs = 0;
  int* kv_qtiles = nullptr;       // [B*H*nb/2, nb/2]: query-block pairs qa | qb << 16
  uint8_t* kv_qmask = nullptr;
  int* kv_count = nullptr;
};

void sla_pool(const __nv_bfloat16* qkv, long ld, int B, int T, int H, float* qm, float* km,
              cudaStream_t s);
void sla_route(const SlaRouteArgs& a, int BH, cudaStream_t s);
void sla_kv_state(const __nv_bfloat16* qkv, long ld, int B, int T, int H, __nv_bfloat16* kvz,
                  cudaStream_t s);
void sla_lin_out(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                 __nv_bfloat16* o, long ldo, float* den, float eps, cudaStream_t s);
void sla_lin_bwd_q(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* state,
                   const __nv_bfloat16* o, long ldo, const __nv_bfloat16* dout, long lddo,
                   const float* den, __nv_bfloat16* dsz, __nv_bfloat16* dqkv, long lddq,
                   cudaStream_t s);
void sla_lin_bwd_kv(const __nv_bfloat16* qkv, long ld, int B, int T, int H, const float* dkvz,
                    __nv_bfloat16* dqkv, long lddq, cudaStream_t s);

}  // namespace ddb
