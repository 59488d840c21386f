// Host-side helpers shared by the extension's .cu files.
#pragma once

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <atomic>
#include <mutex>
#include <stdexcept>
#include <string>

#define NS_CHECK(cond, msg)                                                   \
  do {                                                                        \
    if (!(cond)) throw std::runtime_error(std::string("nanospec_b200: ") + (msg)); \
  } while (0)

#define NS_CUDA(call)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) +   \
                               " at " __FILE__ ":" + std::to_string(__LINE__));         \
  } while (0)

namespace ns {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    NS_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    NS_CHECK(p != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled not found");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [rows, cols] with row stride `ld`
// elements; box = [box_rows, box_cols]; 128-byte swizzle (box_cols * 2 == 128).
inline CUtensorMap make_tmap_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld,
                                  int box_rows, int box_cols) {
  NS_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  NS_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NS_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return map;
}

// 3-D bf16 tensor map over [d2][d1][d0] (d0 innermost, contiguous) with element
// strides s1 (between d1 entries) and s2 (between d2 entries); box = [b2][b1][b0];
// 128-byte swizzle (b0 * 2 == 128). Used for per-head tiles of [tokens][heads][dim]
// activations without a transposed copy.
inline CUtensorMap make_tmap_bf16_3d(const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t s1, int64_t s2,
                                     int b0, int b1, int b2) {
  NS_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  NS_CHECK((s1 * 2) % 16 == 0 && (s2 * 2) % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)(s1 * 2), (cuuint64_t)(s2 * 2)};
  cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, (cuuint32_t)b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NS_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed (" + std::to_string((int)r) + ")");
  return map;
}

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    NS_CUDA(cudaGetDevice(&dev));
    NS_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

// Runs `set` once per device: function attributes (cudaFuncSetAttribute) belong to
// one device's context, so a process that launches on several devices sets them on
// each. `mask` is a per-call-site bit set indexed by device ordinal.
template <class F>
inline void once_per_device(std::atomic<unsigned long long>& mask, F&& set) {
  int dev;
  NS_CUDA(cudaGetDevice(&dev));
  const unsigned long long bit = 1ull << (dev & 63);
  if (mask.load(std::memory_order_acquire) & bit) return;
  set();
  mask.fetch_or(bit, std::memory_order_acq_rel);
}

// Device-side error word shared by the kernels' bounded waits: a kernel whose
// wait times out stores 1 here and exits; `check_device_error` raises on the host.
int* device_error_flag();
void check_device_error();

inline void check_bf16(const at::Tensor& t, const char* name) {
  NS_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  NS_CHECK(t.scalar_type() == at::kBFloat16, std::string(name) + " must be bfloat16");
}

}  // namespace ns
