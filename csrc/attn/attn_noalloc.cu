// Allocation-free attention backward: one extern "C" entry point.
//
// This entry point has no counterpart in the reference (DriveDiT has no CUDA code at
// all); it is an addition of this library.
//
// Who needs it: code that cannot call cudaMalloc while it runs. Examples are a host
// runtime that pre-plans every byte of device memory (a static memory planner or an
// embedded/serving executor that forbids allocation after start-up), a caller that
// holds a non-CUDA allocator and must not let a library grow its own pool, and code
// running in a context where allocation would stall or is not permitted. The regular
// backward (``attn_bwd`` through the Python extension) needs two scratch buffers — the
// fp32 dQ accumulator and the per-row ``delta`` vector — which its caller allocates;
// here they live in fixed device arrays instead.
//
// Scratch: two file-scope ``static __device__`` arrays, 16 MiB for the dQ accumulator
// (``kNoAllocMaxDqFloats`` floats, i.e. rows * heads * 64 <= 4,194,304) and 1 MiB for
// ``delta`` (``kNoAllocMaxDeltaFloats`` floats, i.e. batch * heads * queries <= 262,144),
// plus an int status word. Every GPU that loads this library holds these 17 MiB until
// the process exits.
//
// Use:
//  * The caller passes inputs (q, k, v, o, dO, lse) and outputs (dq, dk, dv) as device
//    pointers with row strides and column offsets, exactly like the regular backward.
//  * The first call on a device (with that device current) looks up the device address
//    of the arrays once with cudaGetSymbolAddress; make that first call before any
//    stream capture on that device.
//  * Every call shares the same arrays and each call overwrites them (the dQ
//    accumulator is cleared with cudaMemsetAsync at the start of each call). Calls
//    that overlap on the GPU — on different streams, or from different threads without
//    ordering — race on the scratch and give wrong results; serialise them.
//  * Sizes beyond the maxima are rejected (return code kNoAllocTooLarge, message on
//    stderr); nothing is launched then.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <cstdio>
#include <exception>
#include <mutex>

#include "../common/tma.h"
#include "attn.h"

namespace {

constexpr long kNoAllocMaxDqFloats = 4L << 20;     // 16 MiB
constexpr long kNoAllocMaxDeltaFloats = 256L << 10;  // 1 MiB
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

// Arguments of ddb_attn_bwd_noalloc. Row strides and column offsets are in elements;
// head h of q/k/v/o/dO/dq/dk/dv occupies columns [col + 64 h, col + 64 h + 64).
typedef struct {
  int B, H, Tq, S;                 // batch, heads (d_head = 64), queries, keys per sample
  long long q_rows_per_b, kv_rows_per_b;  // rows between samples in q/o/dO/dq and in k/v/dk/dv
  const void* q; long long ldq; int q_col;
  const void* k; long long ldk; int k_col;
  const void* v; long long ldv; int v_col;
  const void* o; long long ldo; int o_col;
  const void* dout; long long lddo; int do_col;
  const float* lse;                // [B, H, Tq] from the forward (log2 domain)
  void* dq; long long lddq; int dq_col;
  void* dk; long long lddk; int dk_col;
  void* dv; long long lddv; int dv_col;
  int causal;                      // 0 none, 1 frame-causal, 2 token-causal
  int tokens_per_frame;
  int q_pos_offset, kv_pos_offset;
  float scale;                     // softmax scale (1/sqrt(64) normally)
} ddb_attn_bwd_noalloc_args;

enum {
  kNoAllocOk = 0,
  kNoAllocBadArgument = 1,
  kNoAllocTooLarge = 2,
  kNoAllocSetupFailed = 3,
  kNoAllocLaunchFailed = 4,
};

// Backward of flash attention (bf16, d_head = 64) writing dq, dk, dv without allocating.
// Returns 0 on success or one of the codes above; `stream` may be 0 (legacy stream).
__attribute__((visibility("default"))) int ddb_attn_bwd_noalloc(
    const ddb_attn_bwd_noalloc_args* args, cudaStream_t stream) {
  if (args == nullptr) return kNoAllocBadArgument;
  const ddb_attn_bwd_noalloc_args& x = *args;
  if (x.B <= 0 || x.H <= 0 || x.Tq <= 0 || x.S <= 0 || !x.q || !x.k || !x.v || !x.o ||
      !x.dout || !x.lse || !x.dq || !x.dk || !x.dv || x.tokens_per_frame < 1 ||
      x.q_rows_per_b < x.Tq || x.kv_rows_per_b < x.S) {
    fprintf(stderr, "ddb_attn_bwd_noalloc: invalid argument (null pointer or bad shape)\n");
    return kNoAllocBadArgument;
  }
  const long q_rows = static_cast<long>(x.B) * x.q_rows_per_b;
  const long dq_floats = q_rows * x.H * 64;
  const long delta_floats = static_cast<long>(x.B) * x.H * x.Tq;
  if (dq_floats > kNoAllocMaxDqFloats || delta_floats > kNoAllocMaxDeltaFloats) {
    fprintf(stderr,
            "ddb_attn_bwd_noalloc: problem too large for the static scratch: rows*heads*64 = "
            "%ld (max %ld), batch*heads*queries = %ld (max %ld)\n",
            dq_floats, kNoAllocMaxDqFloats, delta_floats, kNoAllocMaxDeltaFloats);
    return kNoAllocTooLarge;
  }
  ScratchPtrs sp;
  if (scratch_for_current_device(&sp) != 0) {
    fprintf(stderr, "ddb_attn_bwd_noalloc: cudaGetSymbolAddress failed on this device\n");
    return kNoAllocSetupFailed;
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
    g.dq_acc = sp.dq_acc; g.ld_dqacc = static_cast<long>(x.H) * 64;
    g.dk = x.dk; g.lddk = x.lddk; g.dk_col = x.dk_col;
    g.dv = x.dv; g.lddv = x.lddv; g.dv_col = x.dv_col;
    if (cudaMemsetAsync(sp.dq_acc, 0, dq_floats * sizeof(float), stream) != cudaSuccess)
      return kNoAllocLaunchFailed;
    ddb::attn_bwd_delta(x.o, x.ldo, x.o_col, x.dout, x.lddo, x.do_col, sp.delta, x.B, x.H,
                        x.Tq, x.q_rows_per_b, stream);
    ddb::attn_bwd_with_status(g, sp.status, stream);
    ddb::attn_dq_finalize(sp.dq_acc, g.ld_dqacc, x.dq, x.lddq, x.dq_col,
                          static_cast<int>(q_rows), x.H, nullptr, 1, 0, stream);
    if (cudaGetLastError() != cudaSuccess) return kNoAllocLaunchFailed;
  } catch (const std::exception& e) {
    fprintf(stderr, "ddb_attn_bwd_noalloc: %s\n", e.what());
    return kNoAllocLaunchFailed;
  }
  return kNoAllocOk;
}

}  // extern "C"
