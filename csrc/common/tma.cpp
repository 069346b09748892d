#include "tma.h"

#include <atomic>
#include <mutex>
#include <unordered_map>

namespace ddb {

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
               "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled not available from the driver");
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}
}  // namespace

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         uint64_t cols, uint64_t rows, uint64_t row_stride_bytes,
                         uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (row_stride_bytes % 16 != 0)
    throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  if ((box_cols * elem_bytes) % 16 != 0)
    throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled (2d) failed with code " +
                             std::to_string(static_cast<int>(r)));
  return m;
}

CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                         uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                         uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2,
                         CUtensorMapSwizzle swizzle) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  if ((box0 * elem_bytes) % 16 != 0)
    throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled (3d) failed with code " +
                             std::to_string(static_cast<int>(r)));
  return m;
}

CUtensorMap make_tmap_nd(const void* base, CUtensorMapDataType dtype, int elem_bytes, int rank,
                         const uint64_t* dims, const uint64_t* strides_bytes,
                         const uint32_t* box, CUtensorMapSwizzle swizzle) {
  if (rank < 1 || rank > 5) throw std::runtime_error("TMA rank must be 1..5");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0)
      throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  if ((box[0] * elem_bytes) % 16 != 0)
    throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t b[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    estr[i] = 1;
    if (box[i] < 1 || box[i] > 256) throw std::runtime_error("TMA box dims must be 1..256");
  }
  for (int i = 0; i + 1 < rank; ++i) st[i] = strides_bytes[i];
  CUresult r = encode_fn()(&m, dtype, rank, const_cast<void*>(base), d, st, b, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled (rank " + std::to_string(rank) +
                             ") failed with code " + std::to_string(static_cast<int>(r)));
  return m;
}

namespace {
std::atomic<long> g_launches{0};
std::atomic<bool> g_deterministic{false};
std::atomic<bool> g_check_bounds{false};
}
void set_deterministic(bool on) { g_deterministic.store(on); }
bool deterministic() { return g_deterministic.load(); }
void set_check_bounds(bool on) { g_check_bounds.store(on); }
bool check_bounds() { return g_check_bounds.load(); }
void count_launch(long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long launch_count() { return g_launches.load(std::memory_order_relaxed); }

int num_sms(int device) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device),
             "cudaDeviceGetAttribute(SM count)");
  cache[device] = n;
  return n;
}

int* device_status(int device) {
  static std::mutex mu;
  static std::unordered_map<int, int*> words;
  std::lock_guard<std::mutex> g(mu);
  auto it = words.find(device);
  if (it != words.end()) return it->second;
  int prev = 0;
  check_cuda(cudaGetDevice(&prev), "cudaGetDevice");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  int* p = nullptr;
  check_cuda(cudaMalloc(&p, sizeof(int) * 8), "cudaMalloc(status)");
  check_cuda(cudaMemset(p, 0, sizeof(int) * 8), "cudaMemset(status)");
  check_cuda(cudaSetDevice(prev), "cudaSetDevice");
  words[device] = p;
  return p;
}

}  // namespace ddb
