// Host-side TMA tensor-map construction (driver entry point fetched at run time; no -lcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

namespace ccq {
namespace tc {

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// A [rows, H, K] 16-bit token tensor (row = flattened b*T + t) viewed as 3-D for TMA:
// dims {K, H, rows}; one box = 64 columns x 1 head x box_rows rows, 128-byte swizzle.
// The x coordinate of every load is a multiple of 64 elements (128 bytes), as TMA requires.
inline cudaError_t make_token_map(CUtensorMap* map, const void* base, int64_t rows, int H, int K, int box_rows,
                                  bool is_bf16) {
  auto fn = encode_fn();
  if (fn == nullptr) return cudaErrorNotSupported;
  if (((uintptr_t)base & 15) != 0 || (K * 2) % 16 != 0) return cudaErrorInvalidValue;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)H, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)H * K * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace tc
}  // namespace ccq
