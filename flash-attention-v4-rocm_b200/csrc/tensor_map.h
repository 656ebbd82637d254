// Host-side TMA descriptor encoding for BSHD tensors, shared by the library
// and the probe library. cuTensorMapEncodeTiled is fetched through the runtime
// (cudaGetDriverEntryPoint) so the libraries do not link libcuda directly.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace fav4 {

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// BSHD bf16 tensor [B, S, H, 128] as a 4-D TMA map {128, H, S, B} with a
// {64, 1, box_rows, 1} box (box_rows <= 256) and 128-byte swizzle; rows past S
// read as zero.
inline bool encode_bshd(CUtensorMap* map, const void* base, int b, int s, int h, int box_rows = 128) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(s),
                              static_cast<cuuint64_t>(b)};
  const cuuint64_t strides[3] = {256, static_cast<cuuint64_t>(h) * 256, static_cast<cuuint64_t>(s) * h * 256};
  const cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(box_rows), 1};
  const cuuint32_t elem[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace fav4
