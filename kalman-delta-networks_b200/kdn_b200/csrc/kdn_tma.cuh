// Host-side tensor maps for the [B,T,H,D] boundary tensors.
//
// A 4-D map with dims {D, H, T, B} (innermost first) and a box of
// {inner, 1, rows, 1} moves `rows` consecutive tokens of one (b, h) stream
// with one TMA instruction; tokens past T are outside the tensor: loads fill
// them with zeros, stores skip them.  The map encoder is reached through the
// runtime's driver entry point, so the library does not link libcuda directly.
#pragma once

#include <cuda.h>

#include "kdn_common.cuh"

namespace kdn {

// Warp roles of the tensor-core sequential passes: 8 data warps + 1 producer.
constexpr int kTcWarps = 8;
constexpr int kTcThreads = 32 * (kTcWarps + 1);

// Tensor maps handed to those kernels as __grid_constant__ parameters.
struct alignas(64) TcMaps {
  CUtensorMap in;   // value rows (forward) / output cotangent rows (reverse)
  CUtensorMap out;  // output rows (forward)
};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// Map of a contiguous [B,T,H,D] tensor (bf16 or fp32) with boxes of
// `inner` channels x `rows` tokens of one (b, h) stream; `swizzle128` selects
// the 128-byte swizzle (inner * element size must then be 128).
inline int encode_bthd(CUtensorMap* map, const void* base, bool is_bf16, int64_t B, int64_t T, int64_t H, int64_t D,
                       int inner, int rows, bool swizzle128) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return set_error(KDN_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t es = is_bf16 ? 2 : 4;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[3] = {D * es, H * D * es, T * H * D * es};
  const cuuint32_t box[4] = {(cuuint32_t)inner, 1, (cuuint32_t)rows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult rc = fn(map, is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return set_error(KDN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)rc);
  return KDN_OK;
}

}  // namespace kdn
