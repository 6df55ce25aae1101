// Host-side helpers shared by the CUDA sources: TMA tensor-map encoding through the driver entry
// point (no link against libcuda), SM counts, and argument checks.
#pragma once

#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>

namespace rc {

#define RC_CHECK(cond, msg)                                            \
  do {                                                                 \
    if (!(cond)) throw std::runtime_error(std::string("reelcache_b200: ") + (msg)); \
  } while (0)

#define RC_CUDA(expr)                                                                              \
  do {                                                                                             \
    cudaError_t err__ = (expr);                                                                    \
    if (err__ != cudaSuccess)                                                                      \
      throw std::runtime_error(std::string("reelcache_b200: CUDA error: ") + cudaGetErrorString(err__) + \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__));                \
  } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult query;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &query);
    if (err == cudaSuccess && query == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  RC_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// 2-D tiled tensor map over a row-major matrix [outer, inner] with `row_bytes` between rows.
// The box is [box_outer, box_inner]; with the 128-byte swizzle box_inner * elem_bytes must be 128.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                                uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                                CUtensorMapSwizzle swizzle) {
  RC_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  RC_CHECK(row_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  RC_CHECK((box_inner * elem_bytes) % 16 == 0, "TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult res = encode_tiled_fn()(&map, dtype, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RC_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(res)) + ")");
  return map;
}

// 3-D tiled tensor map over [d2, d1, d0] (d0 innermost) with byte strides s1 (between d1 rows) and
// s2 (between d2 slabs).
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0, uint64_t d1,
                                uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                                CUtensorMapSwizzle swizzle) {
  RC_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base address must be 16-byte aligned");
  RC_CHECK(s1 % 16 == 0 && s2 % 16 == 0, "TMA strides must be multiples of 16 bytes");
  RC_CHECK((b0 * elem_bytes) % 16 == 0, "TMA box inner extent must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t elem_strides[3] = {1, 1, 1};
  CUresult res = encode_tiled_fn()(&map, dtype, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RC_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed (code " + std::to_string(static_cast<int>(res)) + ")");
  return map;
}

inline int sm_count(int device) {
  static int counts[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (counts[device] == 0) {
    int value = 0;
    RC_CUDA(cudaDeviceGetAttribute(&value, cudaDevAttrMultiProcessorCount, device));
    counts[device] = value;
  }
  return counts[device];
}

inline void check_cuda_tensor(const at::Tensor& t, const char* name) {
  RC_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
}

inline int* status_ptr(const c10::optional<at::Tensor>& status) {
  if (!status.has_value() || !status->defined()) return nullptr;
  RC_CHECK(status->is_cuda() && status->scalar_type() == at::kInt && status->numel() >= 1,
           "status must be an int32 CUDA tensor");
  return status->data_ptr<int>();
}

}  // namespace rc
