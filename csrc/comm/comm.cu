// NVLink peer-memory collectives fused with the sharded optimizer step (sm_100a).
//
// A training step on W ranks (data parallel, optimizer state sharded W ways):
//   1. rs_sum_sqnorm       each rank reads its 1/W shard of every peer's fp32 gradient
//                          buffer over NVLink (16-byte peer loads), sums them into a local
//                          reduced shard and accumulates the shard's squared norm;
//   2. xrank_barrier       exchanges the squared-norm partials (payload) so every rank knows
//                          the global gradient norm, and orders step 1 before step 3;
//   3. shard_adamw_allgather  AdamW (clip factor from the global norm) on the shard, then the
//                          updated fp32 master values and their bf16 copies are stored into
//                          every rank's buffers (16-byte peer stores) — the all-gather;
//   4. xrank_barrier       every rank's buffers are complete before anyone's next forward.
// This replaces FSDP's reduce-scatter + optimizer + all-gather (reference
// training/cuda_optimized.py:571-615, NCCL) with two bandwidth-bound kernels whose
// communication is their memory traffic. All waits are bounded (status word, no trap).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdexcept>

#include "../common/ptx.cuh"
#include "../common/tma.h"
#include "comm.h"

namespace ddb {

IpcAlloc ipc_alloc(size_t bytes) {
  IpcAlloc a;
  check_cuda(cudaMalloc(&a.ptr, bytes), "cudaMalloc(ipc buffer)");
  check_cuda(cudaMemset(a.ptr, 0, bytes), "cudaMemset(ipc buffer)");
  cudaIpcMemHandle_t h;
  check_cuda(cudaIpcGetMemHandle(&h, a.ptr), "cudaIpcGetMemHandle");
  a.handle.assign(reinterpret_cast<const char*>(&h), sizeof(h));
  return a;
}

void* ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return p;
}

void ipc_close(void* p) { check_cuda(cudaIpcCloseMemHandle(p), "cudaIpcCloseMemHandle"); }
void ipc_free(void* p) { check_cuda(cudaFree(p), "cudaFree(ipc buffer)"); }

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void xrank_barrier_kernel(void* const* peer_bufs, void* local_buf, int rank, int world,
                                     uint32_t epoch, const float* payload, int* status) {
  const int p = threadIdx.x;
  if (p < world) {
    uint32_t* peer_flags = reinterpret_cast<uint32_t*>(peer_bufs[p]);
    float* peer_pay = reinterpret_cast<float*>(peer_flags + world);
    if (payload) peer_pay[rank] = payload[0];
    __threadfence_system();
    st_release_sys(peer_flags + rank, epoch);
    // wait for peer p's arrival in our own flag array
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(local_buf) + p;
    long long t0 = clock64();
    while (true) {
      const uint32_t v = ld_acquire_sys(mine);
      if (static_cast<int32_t>(v - epoch) >= 0) break;
      if (clock64() - t0 > kSpinLimitCycles) {
        if (status) atomicCAS(status, 0, kStatusTimeoutPeer);
        break;
      }
    }
  }
}

__global__ void __launch_bounds__(256) rs_kernel(const float* const* peers, int world, long off,
                                                 long len4, float* __restrict__ red,
                                                 float* __restrict__ sumsq) {
  float acc_sq = 0.f;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < len4; i += static_cast<long>(gridDim.x) * 256) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < world; ++p) {
      const float4 g = reinterpret_cast<const float4*>(peers[p] + off)[i];
      s.x += g.x;
      s.y += g.y;
      s.z += g.z;
      s.w += g.w;
    }
    reinterpret_cast<float4*>(red)[i] = s;
    acc_sq += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc_sq += __shfl_xor_sync(0xffffffffu, acc_sq, o);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc_sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += part[k];
    atomicAdd(sumsq, t);
  }
}

__global__ void __launch_bounds__(256) shard_adamw_kernel(ShardAdamWArgs a) {
  float clip = 1.f;
  if (a.norm_payloads && a.max_norm > 0.f) {
    float sq = 0.f;
    for (int p = 0; p < a.world; ++p) sq += a.norm_payloads[p];
    const float norm = sqrtf(sq) * a.grad_scale;
    clip = fminf(1.f, a.max_norm / (norm + 1e-6f));
  }
  const float gs = a.grad_scale * clip;
  const float step = a.lr / a.bc1;
  const float inv_bc2 = 1.f / a.bc2;
  const long len4 = a.len / 4;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < len4; i += static_cast<long>(gridDim.x) * 256) {
    const long gi = a.off + 4 * i;  // global element index
    float4 g = reinterpret_cast<const float4*>(a.red)[i];
    float4 m = reinterpret_cast<float4*>(a.m)[i];
    float4 v = reinterpret_cast<float4*>(a.v)[i];
    // this rank's own master copy holds the current value of the shard
    const float4 cur = *reinterpret_cast<const float4*>(a.master_local + gi);
    float pa[4] = {cur.x, cur.y, cur.z, cur.w}, ga[4] = {g.x, g.y, g.z, g.w};
    float ma[4] = {m.x, m.y, m.z, m.w}, va[4] = {v.x, v.y, v.z, v.w};
    const bool decay = gi < a.decay_end;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gg = ga[j] * gs;
      ma[j] = a.b1 * ma[j] + (1.f - a.b1) * gg;
      va[j] = a.b2 * va[j] + (1.f - a.b2) * gg * gg;
      if (decay) pa[j] *= (1.f - a.lr * a.wd);
      pa[j] -= step * ma[j] / (sqrtf(va[j] * inv_bc2) + a.eps);
    }
    reinterpret_cast<float4*>(a.m)[i] = make_float4(ma[0], ma[1], ma[2], ma[3]);
    reinterpret_cast<float4*>(a.v)[i] = make_float4(va[0], va[1], va[2], va[3]);
    const float4 np = make_float4(pa[0], pa[1], pa[2], pa[3]);
    const uint2 nb = make_uint2(pack_bf16(pa[0], pa[1]), pack_bf16(pa[2], pa[3]));
    if (gi < a.local_end) {  // gathered by the consuming GEMM: own buffers only
      *reinterpret_cast<float4*>(a.peer_master[a.rank] + gi) = np;
      *reinterpret_cast<uint2*>(a.peer_compute[a.rank] + gi) = nb;
    } else {
      for (int r = 0; r < a.world; ++r) {
        *reinterpret_cast<float4*>(a.peer_master[r] + gi) = np;
        *reinterpret_cast<uint2*>(a.peer_compute[r] + gi) = nb;
      }
    }
  }
  __threadfence_system();
}

int grid_for(long n4) {
  long g = (n4 + 255) / 256;
  return static_cast<int>(g < 148L * 8 ? (g < 1 ? 1 : g) : 148L * 8);
}

}  // namespace

void xrank_barrier(void* const* peer_flag_bufs, void* local_flag_buf, int rank, int world,
                   uint32_t epoch, const float* payload, int* status, cudaStream_t s) {
  if (world > 1024) throw std::runtime_error("xrank_barrier: too many ranks");
  xrank_barrier_kernel<<<1, 32 * ((world + 31) / 32), 0, s>>>(peer_flag_bufs, local_flag_buf, rank,
                                                              world, epoch, payload, status);
  count_launch();
}

void rs_sum_sqnorm(const float* const* peer_grads, int world, long off, long len, float* red,
                   float* sumsq, cudaStream_t s) {
  if (len % 4 != 0 || off % 4 != 0) throw std::runtime_error("rs_sum_sqnorm: 16-byte granularity");
  rs_kernel<<<grid_for(len / 4), 256, 0, s>>>(peer_grads, world, off, len / 4, red, sumsq);
  count_launch();
}

void shard_adamw_allgather(const ShardAdamWArgs& a, cudaStream_t s) {
  if (a.len % 4 != 0 || a.off % 4 != 0 || a.local_end % 4 != 0)
    throw std::runtime_error("shard_adamw: 16-byte granularity");
  if (a.rank < 0 || a.rank >= a.world) throw std::runtime_error("shard_adamw: bad rank");
  shard_adamw_kernel<<<grid_for(a.len / 4), 256, 0, s>>>(a);
  count_launch();
}


namespace {
__global__ void __launch_bounds__(256) tp_sum_rows_kernel(const __nv_bfloat16* __restrict__ recv, long world,
                                                          long rows, long d, const __nv_bfloat16* __restrict__ res,
                                                          __nv_bfloat16* __restrict__ out) {
  const long n8 = rows * d / 8;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n8; i += static_cast<long>(gridDim.x) * 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    auto add = [&](const __nv_bfloat16* p) {
      const uint4 v = *reinterpret_cast<const uint4*>(p + i * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[q]));
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    };
    if (res) add(res);
    for (long s = 0; s < world; ++s) add(recv + s * rows * d);
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      o[q] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(out + i * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// All-reduce by peer loads: out = residual + sum over ranks p of peer p's partial
// (peer_parts[p] is rank p's buffer, this rank's own entry included), 16 bytes per
// thread per rank, fp32 sums in a fixed rank order (every rank computes bit-identical
// rows).
__global__ void __launch_bounds__(256) tp_allreduce_sum_kernel(const __nv_bfloat16* const* __restrict__ peer_parts,
                                                               long world, long n8,
                                                               const __nv_bfloat16* __restrict__ res,
                                                               __nv_bfloat16* __restrict__ out) {
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n8; i += static_cast<long>(gridDim.x) * 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    auto add = [&](const __nv_bfloat16* p) {
      const uint4 v = *reinterpret_cast<const uint4*>(p + i * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[q]));
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    };
    for (long s = 0; s < world; ++s) add(peer_parts[s]);
    if (res) add(res);
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      o[q] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(out + i * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}
}  // namespace

void tp_allreduce_sum(const __nv_bfloat16* const* peer_parts, long world, long n, const __nv_bfloat16* residual,
                      __nv_bfloat16* out, cudaStream_t s) {
  if (n % 8 != 0) throw std::runtime_error("tp_allreduce_sum: element count % 8");
  const long n8 = n / 8;
  if (n8 == 0) return;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = static_cast<int>(std::min<long>((n8 + 255) / 256, 4L * num_sms(dev)));
  tp_allreduce_sum_kernel<<<grid, 256, 0, s>>>(peer_parts, world, n8, residual, out);
  count_launch();
}

void tp_sum_rows(const __nv_bfloat16* recv, long world, long rows, long d, const __nv_bfloat16* residual,
                 __nv_bfloat16* out, cudaStream_t s) {
  if (d % 8 != 0) throw std::runtime_error("tp_sum_rows: d % 8");
  const long n8 = rows * d / 8;
  if (n8 == 0) return;
  int dev = 0;
  cudaGetDevice(&dev);
  const int grid = static_cast<int>(std::min<long>((n8 + 255) / 256, 4L * num_sms(dev)));
  tp_sum_rows_kernel<<<grid, 256, 0, s>>>(recv, world, rows, d, residual, out);
  count_launch();
}

}  // namespace ddb
