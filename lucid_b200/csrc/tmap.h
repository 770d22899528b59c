// Host-side TMA descriptor creation.  cuTensorMapEncodeTiled is fetched
// from the driver at run time (cudaGetDriverEntryPoint), so the library
// does not link libcuda directly.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace lb {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// cuTensorMapEncodeTiled needs the device's context current in the calling
// thread.  A thread that has only set the device (e.g. the autograd engine's
// worker thread) has no current context until its first runtime call, so
// bind the primary context once per (thread, device).
inline void bind_current_context() {
  thread_local int bound_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  if (dev != bound_dev) {
    cudaFree(nullptr);
    bound_dev = dev;
  }
}

// bf16 [c3][c2][rows][cols] view with element strides (s_row, s_c2, s_c3);
// box = 64 columns x 128 rows, 128-byte swizzle.  Rows beyond `rows` read
// as zero.
inline bool make_tmap_bf16(CUtensorMap* m, const void* ptr, int cols, int rows, int n2, int n3,
                           long long s_row, long long s_c2, long long s_c3) {
  bind_current_context();
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)n2, (cuuint64_t)n3};
  cuuint64_t strides[3] = {(cuuint64_t)(s_row * 2), (cuuint64_t)(s_c2 * 2), (cuuint64_t)(s_c3 * 2)};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp32 [rows][128] matrix, box = 32 columns (128 bytes) x 128 rows,
// 128-byte swizzle: the target of the bulk reduce-adds of the backward.
inline bool make_tmap_f32_rows(CUtensorMap* m, const void* ptr, long long rows) {
  bind_current_context();
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {128, (cuuint64_t)rows};
  cuuint64_t strides[1] = {128 * 4};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace lb
