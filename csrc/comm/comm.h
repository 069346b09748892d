// NVLink peer-memory collectives fused with compute (sm_100a): CUDA-IPC symmetric
// buffers, bounded cross-rank barriers, and the sharded optimizer step that reduces
// gradients from every peer and writes the updated weights into every peer.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <string>

namespace ddb {

// ---- CUDA IPC buffers (host)
struct IpcAlloc {
  void* ptr = nullptr;
  std::string handle;  // cudaIpcMemHandle_t bytes
};
IpcAlloc ipc_alloc(size_t bytes);
void* ipc_open(const std::string& handle);
void ipc_close(void* peer_ptr);
void ipc_free(void* ptr);

// ---- kernels
// Cross-rank barrier on `epoch`: rank r writes epoch (and an optional float payload) into
// slot r of every peer's flag array, then waits (bounded) until every slot of its own array
// holds >= epoch. flags layout per rank: [world] uint32 flags, then [world] float payloads.
// out[r] = residual[r] + sum_s recv[s * rows + r] over d bf16 columns (d % 8 == 0).
// out = residual + sum of the n-element bf16 partials of every rank (peer_parts: device
// array of the ranks' buffer pointers, P2P mappings for the peers), read by peer loads
void tp_allreduce_sum(const __nv_bfloat16* const* peer_parts, long world, long n, const __nv_bfloat16* residual,
                      __nv_bfloat16* out, cudaStream_t s);
void tp_sum_rows(const __nv_bfloat16* recv, long world, long rows, long d, const __nv_bfloat16* residual,
                 __nv_bfloat16* out, cudaStream_t s);
void xrank_barrier(void* const* peer_flag_bufs, void* local_flag_buf, int rank, int world,
                   uint32_t epoch, const float* payload, int* status, cudaStream_t s);

// red[i] = sum_p grad_p[off + i] for i < len (peer loads), sumsq[0] += sum red^2
void rs_sum_sqnorm(const float* const* peer_grads, int world, long off, long len, float* red,
                   float* sumsq, cudaStream_t s);

struct ShardAdamWArgs {
  const float* red = nullptr;          // reduced gradient shard [len]
  const float* master_local = nullptr; // this rank's full fp32 master (current values)
  float* m = nullptr;                  // moments of the shard
  float* v = nullptr;
  float* const* peer_master = nullptr; // device array [world] of full fp32 master buffers
  __nv_bfloat16* const* peer_compute = nullptr;  // device array [world] of bf16 copies
  int world = 1;
  int rank = 0;
  long off = 0, len = 0, decay_end = 0;  // decay_end is a global element index
  // elements below local_end (global index) are weights that their consuming GEMM
  // all-gathers itself (weight-sharded mode): stored into this rank's buffers only
  long local_end = 0;
  const float* norm_payloads = nullptr;  // [world] squared-norm partials (clipping), or null
  float max_norm = 0.f;
  float lr = 0, b1 = 0, b2 = 0, eps = 0, wd = 0, bc1 = 1, bc2 = 1, grad_scale = 1;
};
// AdamW on the shard; the updated fp32 and bf16 values are stored into every rank's
// buffers at [off, off + len) (peer stores = the all-gather), except elements below
// local_end, which go to this rank's buffers only.
void shard_adamw_allgather(const ShardAdamWArgs& a, cudaStream_t s);

}  // namespace ddb
