// Allocation-free attention backward: the implementation of the extern "C" interface
// declared in attn_noalloc.h (which states who it is for, its limits and its rules).
//
// This entry point has no counterpart in the reference (DriveDiT has no CUDA code at
// all); it is an addition of this library.
//
// Scratch: two file-scope ``static __device__`` arrays, 16 MiB for the dQ accumulator
// and 1 MiB for ``delta``, plus an int status word. Host code never passes the
// arrays' names to a kernel (in host code they are host-side stand-ins, not device
// addresses): the first call on a device looks up their device addresses with
// cudaGetSymbolAddress, with that device current, and every launch gets those.
#include <cuda_runtime.h>

#include <cstdio>
#include <exception>
#include <mutex>

#include "../common/tma.h"
#include "attn.h"
#include "attn_noalloc.h"

namespace {

constexpr long kNoAllocMaxDqFloats = DDB_NOALLOC_MAX_DQ_FLOATS;        // 16 MiB
constexpr long kNoAllocMaxDeltaFloats = DDB_NOALLOC_MAX_DELTA_FLOATS;  // 1 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_dq_acc[kNoAllocMaxDqFloats];
static __device__ __align__(256) float g_noalloc_delta[kNoAllocMaxDeltaFloats];
static __device__ __align__(256) int g_noalloc_status[8];

struct ScratchPtrs {
  float* dq_acc = nullptr;
  float* delta = nullptr;
  int* status = nullptr;
};

std::mutex g_mu;
ScratchPtrs g_ptrs[kMaxDevices];

// Device addresses of the static arrays for the current device (looked up once).
int scratch_for_current_device(ScratchPtrs* out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  std::lock_guard<std::mutex> lock(g_mu);
  ScratchPtrs& p = g_ptrs[dev];
  if (p.dq_acc == nullptr) {
    void* a = nullptr;
    void* b = nullptr;
    void* c = nullptr;
    if (cudaGetSymbolAddress(&a, g_noalloc_dq_acc) != cudaSuccess ||
        cudaGetSymbolAddress(&b, g_noalloc_delta) != cudaSuccess ||
        cudaGetSymbolAddress(&c, g_noalloc_status) != cudaSuccess || a == nullptr ||
        b == nullptr || c == nullptr) {
      return -1;
    }
    p.delta = static_cast<float*>(b);
    p.status = static_cast<int*>(c);
    p.dq_acc = static_cast<float*>(a);
  }
  *out = p;
  return 0;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) unsigned long long ddb_attn_bwd_noalloc_args_size(void) {
  return sizeof(ddb_attn_bwd_noalloc_args);
}

__attribute__((visibility("default"))) int ddb_attn_bwd_noalloc(
    const ddb_attn_bwd_noalloc_args* args, cudaStream_t stream) {
  if (args == nullptr) return DDB_NOALLOC_BAD_ARGUMENT;
  const ddb_attn_bwd_noalloc_args& x = *args;
  if (x.B <= 0 || x.H <= 0 || x.Tq <= 0 || x.S <= 0 || !x.q || !x.k || !x.v || !x.o ||
      !x.dout || !x.lse || !x.dq || !x.dk || !x.dv || x.tokens_per_frame < 1 ||
      x.q_rows_per_b < x.Tq || x.kv_rows_per_b < x.S) {
    fprintf(stderr, "ddb_attn_bwd_noalloc: invalid argument (null pointer or bad shape)\n");
    return DDB_NOALLOC_BAD_ARGUMENT;
  }
  if (x.Tq % 128 != 0) {
    fprintf(stderr, "ddb_attn_bwd_noalloc: queries per sample (%d) must be a multiple of 128\n",
            x.Tq);
    return DDB_NOALLOC_BAD_ARGUMENT;
  }
  // bound each factor by division first, so the products below cannot overflow
  const long per_row = static_cast<long>(x.H) * 64;
  if (x.q_rows_per_b > kNoAllocMaxDqFloats / per_row / x.B ||
      x.Tq > kNoAllocMaxDeltaFloats / x.H / x.B) {
    fprintf(stderr,
            "ddb_attn_bwd_noalloc: problem too large for the static scratch: needs "
            "batch*rows*heads*64 <= %ld and batch*heads*queries <= %ld (batch %d, heads %d, "
            "rows per sample %lld, queries %d)\n",
            kNoAllocMaxDqFloats, kNoAllocMaxDeltaFloats, x.B, x.H, x.q_rows_per_b, x.Tq);
    return DDB_NOALLOC_TOO_LARGE;
  }
  const long q_rows = static_cast<long>(x.B) * x.q_rows_per_b;
  const long dq_floats = q_rows * per_row;
  ScratchPtrs sp;
  if (scratch_for_current_device(&sp) != 0) {
    fprintf(stderr, "ddb_attn_bwd_noalloc: cudaGetSymbolAddress failed on this device\n");
    return DDB_NOALLOC_SETUP_FAILED;
  }
  try {
    ddb::AttnBwdArgs g;
    ddb::AttnArgs& a = g.f;
    a.B = x.B; a.H = x.H; a.Tq = x.Tq; a.S = x.S;
    a.q_rows_per_b = x.q_rows_per_b; a.kv_rows_per_b = x.kv_rows_per_b;
    a.q = x.q; a.ldq = x.ldq; a.q_col = x.q_col;
    a.k = x.k; a.ldk = x.ldk; a.k_col = x.k_col;
    a.v = x.v; a.ldv = x.ldv; a.v_col = x.v_col;
    a.o = const_cast<void*>(x.o); a.ldo = x.ldo; a.o_col = x.o_col;
    a.lse = const_cast<float*>(x.lse);
    a.causal = x.causal; a.tpf = x.tokens_per_frame;
    a.q_pos_offset = x.q_pos_offset; a.kv_pos_offset = x.kv_pos_offset;
    a.scale = x.scale;
    g.dout = x.dout; g.lddo = x.lddo; g.do_col = x.do_col;
    g.delta = sp.delta;
    g.dq_acc = sp.dq_acc; g.ld_dqacc = per_row;
    g.dk = x.dk; g.lddk = x.lddk; g.dk_col = x.dk_col;
    g.dv = x.dv; g.lddv = x.lddv; g.dv_col = x.dv_col;
    // the status word keeps the first error of a launch: clear what the last call left
    if (cudaMemsetAsync(sp.status, 0, 8 * sizeof(int), stream) != cudaSuccess ||
        cudaMemsetAsync(sp.dq_acc, 0, dq_floats * sizeof(float), stream) != cudaSuccess)
      return DDB_NOALLOC_LAUNCH_FAILED;
    ddb::attn_bwd_delta(x.o, x.ldo, x.o_col, x.dout, x.lddo, x.do_col, sp.delta, x.B, x.H,
                        x.Tq, x.q_rows_per_b, stream);
    ddb::attn_bwd_with_status(g, sp.status, stream);
    // finalize each sample's Tq rows only: rows between samples belong to the caller
    for (int b = 0; b < x.B; ++b) {
      const long row0 = static_cast<long>(b) * x.q_rows_per_b;
      ddb::attn_dq_finalize(sp.dq_acc + row0 * per_row, per_row,
                            static_cast<__nv_bfloat16*>(x.dq) + row0 * x.lddq, x.lddq, x.dq_col,
                            x.Tq, x.H, nullptr, 1, 0, stream);
    }
    if (cudaGetLastError() != cudaSuccess) return DDB_NOALLOC_LAUNCH_FAILED;
  } catch (const std::exception& e) {
    fprintf(stderr, "ddb_attn_bwd_noalloc: %s\n", e.what());
    return DDB_NOALLOC_LAUNCH_FAILED;
  }
  return DDB_NOALLOC_OK;
}

__attribute__((visibility("default"))) int ddb_attn_bwd_noalloc_status(cudaStream_t stream,
                                                                       int* device_status) {
  if (device_status == nullptr) return DDB_NOALLOC_BAD_ARGUMENT;
  ScratchPtrs sp;
  if (scratch_for_current_device(&sp) != 0) return DDB_NOALLOC_SETUP_FAILED;
  int v = 0;
  if (cudaMemcpyAsync(&v, sp.status, sizeof(int), cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return DDB_NOALLOC_LAUNCH_FAILED;
  *device_status = v;
  return v == 0 ? DDB_NOALLOC_OK : DDB_NOALLOC_DEVICE_ERROR;
}

}  // extern "C"
