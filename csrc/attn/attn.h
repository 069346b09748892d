// tcgen05 flash attention (d_head = 64) for sm_100a: forward, backward, SLA routing.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ddb {

enum AttnCausal : int { kCausalNone = 0, kCausalFrame = 1, kCausalToken = 2 };

struct AttnArgs {
  int B = 0, H = 0;
  int Tq = 0;                 // queries per sample
  int S = 0;                  // keys per sample
  long q_rows_per_b = 0;      // row stride between samples in the q tensor (usually Tq)
  long kv_rows_per_b = 0;     // row stride between samples in the k/v tensors (usually S)
  long q_rows_total = 0;      // rows addressable in q / k,v (0: B * rows_per_b)
  long kv_rows_total = 0;
  const void* q = nullptr;    // bf16 rows; head h at column q_col + 64 h
  long ldq = 0;
  int q_col = 0;
  const void* k = nullptr;
  long ldk = 0;
  int k_col = 0;
  const void* v = nullptr;
  long ldv = 0;
  int v_col = 0;
  void* o = nullptr;          // bf16 rows; head h at column o_col + 64 h
  long ldo = 0;
  int o_col = 0;
  float* lse = nullptr;       // [B, H, Tq], log2 domain (max*scale*log2e + log2 sum)
  int causal = kCausalNone;
  int tpf = 1;                // tokens per frame (frame-causal)
  int q_pos_offset = 0;       // absolute position of query 0
  int kv_pos_offset = 0;      // absolute position of key 0
  float scale = 0.125f;       // softmax scale
  // block-sparse (SLA) mode: per (b, h, q-tile of 128) a list of 64-key block pairs
  const int* pair_blocks = nullptr;  // [B*H*n_qtiles, max_pairs]: blk0 | blk1 << 16
  const uint8_t* pair_mask = nullptr;  // 4 bits: (q half)*2 + (key half)
  const int* pair_count = nullptr;     // [B*H*n_qtiles]
  int max_pairs = 0;
  // split-KV (dense / causal modes): kv_splits CTAs share a query tile's key range; each
  // writes its normalised fp32 O rows to o_part [kv_splits][B*Tq][H*64] and its log2-domain
  // lse to lse_part [kv_splits][B*H*Tq], and attn_fwd merges them into o (and lse).
  // attn_fwd chooses kv_splits (> 1 only when the grid would leave SMs idle) and needs
  // the two scratch buffers then (attn_fwd_split_scratch gives their sizes).
  int kv_splits = 1;
  float* o_part = nullptr;
  float* lse_part = nullptr;
};

void attn_fwd(const AttnArgs& a, cudaStream_t s);
// key-range splits attn_fwd would use for `a` on this device (1: no scratch needed) and
// the fp32 element counts of the two scratch buffers for that many splits
int attn_fwd_kv_splits(const AttnArgs& a);
void attn_fwd_split_scratch(const AttnArgs& a, int splits, long* o_part_elems, long* lse_part_elems);
// pipeline-study hook: record clock64 events of CTA `cta` into buf[3 * 8 * 64] (nullptr: off)
void attn_fwd_set_trace(long long* buf, int cta);

struct AttnBwdArgs {
  AttnArgs f;                 // forward description (q/k/v/o/lse, masks)
  const void* dout = nullptr; // bf16 rows like o
  long lddo = 0;
  int do_col = 0;
  const float* delta = nullptr;  // [B, H, Tq] rowsum(dO * O)
  float* dq_acc = nullptr;    // fp32 [B*Tq rows, ld_dqacc] (zeroed), head h at 64 h
  long ld_dqacc = 0;
  void* dk = nullptr;         // bf16 rows, head h at dk_col + 64 h
  long lddk = 0;
  int dk_col = 0;
  void* dv = nullptr;
  long lddv = 0;
  int dv_col = 0;
  // block-sparse transpose lists: per (b, h, kv-tile of 128) the 64-query blocks that see
  // it, two per 128-query unit: qa | qb << 16 (rows 0-63 of the unit are block qa, rows
  // 64-127 block qb; qb == qa with its half masked off for an odd last block)
  const int* kv_qtiles = nullptr;    // [B*H*n_kvtiles, max_q]
  const uint8_t* kv_qmask = nullptr; // 4 bits: (q half)*2 + (key half)
  const int* kv_count = nullptr;
  int max_q = 0;
  int debug_flags = 0;        // bit 0: skip the dQ reductions (timing experiments only)
  long long* trace = nullptr; // optional per-role clock64 trace of CTA `trace_cta`
  int trace_cta = 0;
};

void attn_bwd(const AttnBwdArgs& a, cudaStream_t s);
void attn_bwd_with_status(const AttnBwdArgs& a, int* status, cudaStream_t s);

// delta[b,h,t] = sum_d dO * O over each head's 64 columns
void attn_bwd_delta(const void* o, long ldo, int o_col, const void* dout, long lddo,
                    int do_col, float* delta, int B, int H, int Tq, long rows_per_b,
                    cudaStream_t s);
// dq (bf16, optionally rotated back by a rotary table) from the fp32 accumulator
void attn_dq_finalize(const float* dq_acc, long ld_acc, void* dq, long lddq, int dq_col,
                      int rows, int H, const float2* rope_tab, int rows_per_seq,
                      int pos_offset, cudaStream_t s);

}  // namespace ddb
