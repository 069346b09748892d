/* Allocation-free attention backward: the public C interface of ddb_attn_bwd_noalloc.
 *
 * This interface has no counterpart in the reference (DriveDiT has no CUDA or C code);
 * it is an addition of this library, exported from the drivedit_b200._C shared object.
 *
 * Who it is for: callers that cannot allocate device memory while they run, such as
 * a runtime that plans every byte of device memory before it starts (a static memory
 * planner, an embedded or serving executor that forbids allocation after start-up),
 * or a host that owns the device allocator and must not let a library grow its own
 * pool. The regular backward needs two scratch buffers (the fp32 dQ accumulator and
 * the per-row delta vector) that its caller allocates; this entry point keeps them in
 * fixed device arrays inside the library instead, so the caller passes only its own
 * inputs and outputs.
 *
 * Limits: rows x heads x 64 <= DDB_NOALLOC_MAX_DQ_FLOATS (16 MiB of fp32 accumulator)
 * and batch x heads x queries <= DDB_NOALLOC_MAX_DELTA_FLOATS (1 MiB); larger problems
 * are rejected with DDB_NOALLOC_TOO_LARGE and nothing is launched. Every GPU that
 * loads the library holds these 17 MiB until the process exits.
 *
 * Rules:
 *  - The first call on a device (with that device current) looks up the device
 *    address of the arrays once with cudaGetSymbolAddress; make that first call
 *    before any stream capture on that device.
 *  - Every call shares the same arrays, and each call overwrites them. Calls that
 *    overlap on the GPU (different streams, or threads without ordering) race on the
 *    scratch and give wrong results: serialise them.
 *  - Kernel-side failures (a bounded pipeline wait that ran out, a bad launch
 *    configuration) are recorded in a device status word that each call clears first.
 *    ddb_attn_bwd_noalloc_status() waits for the stream and reports it.
 *  - No cudaMalloc, cudaFree or allocating library routine is called.
 */
#ifndef DDB_ATTN_NOALLOC_H_
#define DDB_ATTN_NOALLOC_H_

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DDB_NOALLOC_MAX_DQ_FLOATS (4L << 20)
#define DDB_NOALLOC_MAX_DELTA_FLOATS (256L << 10)

/* Return codes. */
enum {
  DDB_NOALLOC_OK = 0,
  DDB_NOALLOC_BAD_ARGUMENT = 1,   /* null pointer, bad shape, Tq not a multiple of 128 */
  DDB_NOALLOC_TOO_LARGE = 2,      /* beyond the static scratch; nothing launched */
  DDB_NOALLOC_SETUP_FAILED = 3,   /* cudaGetSymbolAddress failed on this device */
  DDB_NOALLOC_LAUNCH_FAILED = 4,  /* a CUDA launch or memset returned an error */
  DDB_NOALLOC_DEVICE_ERROR = 5,   /* status query: a kernel recorded an error */
};

/* Arguments. Row strides (ld*) and column offsets (*_col) are in elements; head h of
 * q/k/v/o/dout/dq/dk/dv occupies columns [col + 64 h, col + 64 h + 64) of its rows.
 * Sample b's rows start at row b * q_rows_per_b (q, o, dout, dq) and
 * b * kv_rows_per_b (k, v, dk, dv); only the first Tq (S) rows of each sample are read
 * or written, so rows between samples are left untouched. */
typedef struct {
  int B, H, Tq, S;                 /* batch, heads (d_head = 64), queries, keys per sample */
  long long q_rows_per_b, kv_rows_per_b;
  const void* q; long long ldq; int q_col;        /* bf16 */
  const void* k; long long ldk; int k_col;        /* bf16 */
  const void* v; long long ldv; int v_col;        /* bf16 */
  const void* o; long long ldo; int o_col;        /* bf16 forward output */
  const void* dout; long long lddo; int do_col;   /* bf16 gradient of o */
  const float* lse;                /* [B, H, Tq] from the forward (log2 domain) */
  void* dq; long long lddq; int dq_col;           /* bf16 outputs */
  void* dk; long long lddk; int dk_col;
  void* dv; long long lddv; int dv_col;
  int causal;                      /* 0 none, 1 frame-causal, 2 token-causal */
  int tokens_per_frame;
  int q_pos_offset, kv_pos_offset; /* absolute positions of query 0 and key 0 */
  float scale;                     /* softmax scale (1/sqrt(64) normally) */
} ddb_attn_bwd_noalloc_args;

/* Backward of flash attention (bf16, d_head = 64): writes dq, dk, dv on `stream`
 * (0: the legacy stream) without allocating. Returns DDB_NOALLOC_OK once the work is
 * enqueued, or an error code (nothing, or not all of the work, enqueued). */
int ddb_attn_bwd_noalloc(const ddb_attn_bwd_noalloc_args* args, cudaStream_t stream);

/* Waits for `stream`, copies the current device's status word into *device_status
 * (0: every kernel of the last call finished its work; otherwise the kernel's error
 * code) and returns DDB_NOALLOC_OK or DDB_NOALLOC_DEVICE_ERROR. Allocates nothing. */
int ddb_attn_bwd_noalloc_status(cudaStream_t stream, int* device_status);

/* sizeof(ddb_attn_bwd_noalloc_args) as compiled into the library, so bindings written
 * in other languages can check their copy of the layout. */
unsigned long long ddb_attn_bwd_noalloc_args_size(void);

#ifdef __cplusplus
}
#endif

#endif /* DDB_ATTN_NOALLOC_H_ */
