// Persistent tcgen05 GEMM for sm_100a: D[M,N] = A[M,K] * B[N,K]^T with fused epilogues.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace ddb {

enum GemmEpilogue : int {
  kEpiBf16 = 0,        // D(bf16) = acc (+ bias[n]) (+ C[m,n])
  kEpiF32 = 1,         // D(f32)  = acc (+ bias[n])
  kEpiF32Atomic = 2,   // D(f32) += acc   (split-K capable)
  kEpiSwiGLU = 3,      // D(bf16) = acc (gate/up interleaved by 32), D2(bf16) = silu(g)*u
  kEpiDSwiGLU = 4,     // acc = dA; C = gu (bf16); D(bf16) = d(gu) in gu's layout
  kEpiRope = 5,        // D(bf16) = acc with rotary pairs applied to columns < rope_cols
  kEpiGateResidual = 6, // D(bf16) = C + gate[row_group, n] * acc (AdaLN-Zero residual)
  kEpiGelu = 7          // D(bf16) = gelu(acc + bias[n]) (erf form)
};

constexpr int kMaxGemmPeers = 8;

struct GemmArgs {
  int M = 0, N = 0, K = 0;
  const void* A = nullptr;  // bf16
  long lda = 0;             // elements between rows of A's storage
  bool a_mn_major = false;  // storage is [K][M] instead of [M][K]
  const void* B = nullptr;  // bf16
  long ldb = 0;
  bool b_mn_major = false;  // storage is [K][N] instead of [N][K]
  void* D = nullptr;
  long ldd = 0;
  const void* C = nullptr;  // bf16 residual / gu for dswiglu (may alias D)
  long ldc = 0;
  const float* bias = nullptr;
  void* D2 = nullptr;       // swiglu activation output
  long ldd2 = 0;
  // rotary table: float2 (cos, sin) [positions][pairs_per_head], row -> position
  const float2* rope_tab = nullptr;
  int rope_cols = 0;        // columns [0, rope_cols) are rotated (q and k)
  int rope_rows_per_seq = 1;
  int rope_pos_offset = 0;
  int rope_head_dim = 64;
  // gated residual: gate is bf16 [M / gate_rows_per_group][ldg]
  const void* gate = nullptr;
  long ldg = 0;
  int gate_rows_per_group = 1;
  int batch = 1;            // strided batch: A, B advance by stride_a / stride_b elements,
  long stride_a = 0;        // D (and C) by M rows (batches stacked row-wise)
  long stride_b = 0;
  // grouped (MoE) scheduling with device-side tables:
  //  1: A rows are expert segments of a permuted buffer; m-tile i covers rows
  //     [grp_tile_row[i], +128) of expert grp_tile_expert[i] (B batch = expert);
  //     *grp_total_mtiles tiles are valid (launched for an upper bound)
  //  2: reduction over expert segments (weight gradients): expert e reduces k-blocks
  //     [grp_kstart[e], grp_kend[e]) of A/B and writes D batch e
  int grouped = 0;
  const int* grp_tile_expert = nullptr;
  const int* grp_tile_row = nullptr;
  const int* grp_total_mtiles = nullptr;
  const int* grp_kstart = nullptr;
  const int* grp_kend = nullptr;
  int grp_max_mtiles = 0;
  // Tensor parallelism, all-gather fused into the A loads (K-major A, no batch): A rows
  // [p * a_rows_per_peer, (p + 1) * a_rows_per_peer) are read by TMA straight from rank p's
  // buffer a_peer_ptrs[p] (a CUDA-IPC mapping; plain loads, no multicast), row-major with lda.
  int a_npeers = 0;
  int a_rows_per_peer = 0;
  const void* a_peer_ptrs[kMaxGemmPeers] = {};
  // Reduce-scatter fused into the bf16 store (epilogue kEpiBf16 without residual): output row
  // r is stored into rank (r / d_rows_per_peer)'s buffer d_peers[...] at row
  // d_slot * d_rows_per_peer + r % d_rows_per_peer (d_peers: device array of base pointers).
  void* const* d_peers = nullptr;
  int d_rows_per_peer = 0;
  int d_slot = 0;
  // FSDP parameter all-gather fused into the B (weight) loads. B is a K-major [N][K]
  // weight (ldb == K) inside a flat parameter buffer that is sharded over gb_world ranks
  // in contiguous ranges of gb_shard elements; B[0][0] is flat element gb_elem0, and
  // gb_peers[r] is B's address in rank r's copy of the buffer (gb_peers[gb_rank] == B,
  // a CUDA-IPC mapping for the others). Before its first tile, every CTA's epilogue warps
  // copy their share of B's peer-owned pieces into this rank's copy (plain 16-byte P2P
  // loads, local stores) and publish one counter per 128-row group of B
  // (red.release.gpu); the TMA producer acquires the counters of a tile's row groups
  // (bounded wait) before it loads that tile's B. gb_counters [ceil(N / 128)] start at
  // zero and are never reset: launch number gb_epoch (1, 2, ...) waits for gb_epoch x the
  // pieces of a group. No TMA ever reads peer memory here.
  int gb_world = 0;
  int gb_rank = 0;
  long gb_elem0 = 0;
  long gb_shard = 0;
  const void* gb_peers[kMaxGemmPeers] = {};
  unsigned* gb_counters = nullptr;
  unsigned gb_epoch = 0;
  int splits = 1;           // split-K factor (kEpiF32Atomic only)
  int bn = 0;               // 0 = auto (128 or 256)
  int max_ctas = 0;         // 0 = all SMs
};

void gemm(const GemmArgs& args, int epilogue, cudaStream_t stream);
// CTA-pair (256-row, cta_group::2) tiles for plain GEMMs: -1 chosen by the cost estimate
// (default), 0 never, 1 whenever the GEMM is eligible. Returns the previous mode.
int gemm_set_pair_mode(int mode);

}  // namespace ddb
