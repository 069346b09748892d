// Host-side helpers: TMA tensor-map encoding (driver entry point resolved at run time,
// so the extension needs no link against libcuda), SM count, status word.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace ddb {

// 2-D tensor map over a row-major matrix with `rows` rows of `cols` elements,
// `row_stride_bytes` apart. The box is {box_cols, box_rows}; 128-byte swizzle when
// box_cols * elem_size == 128.
CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         uint64_t cols, uint64_t rows, uint64_t row_stride_bytes,
                         uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

// 3-D tensor map: dims {d0 (contiguous), d1, d2}, strides in bytes for d1 and d2.
CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                         uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2,
                         CUtensorMapSwizzle swizzle);

// Tensor map of rank 1..5: dims[0] contiguous, strides_bytes[i] is the byte stride of
// dims[i+1]. Out-of-range box elements read as zero.
CUtensorMap make_tmap_nd(const void* base, CUtensorMapDataType dtype, int elem_bytes, int rank,
                         const uint64_t* dims, const uint64_t* strides_bytes,
                         const uint32_t* box, CUtensorMapSwizzle swizzle);

int num_sms(int device);

// Number of kernels this extension has launched in the process (for launch accounting).
void count_launch(long n = 1);
long launch_count();

// Per-device status word written by kernels whose bounded waits ran out (and, in the
// bounds-checking mode, by kernels that met an out-of-range index).
int* device_status(int device);

// Process-wide debug switches (off by default; read by the kernels' host launchers).
//  deterministic: index-driven permutations (the MoE dispatch) assign rows in a fixed
//                 order instead of by atomic arrival, so every reduction over them is
//                 bit-reproducible run to run;
//  check_bounds:  index-driven kernels check every table-derived index against the
//                 extent of the buffer it addresses; an index out of range is recorded
//                 in the status word (kStatusBadIndex, and the index in word 1) and the
//                 access is skipped instead of faulting.
void set_deterministic(bool on);
bool deterministic();
void set_check_bounds(bool on);
bool check_bounds();

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace ddb
