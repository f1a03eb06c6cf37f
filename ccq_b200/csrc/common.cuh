// Shared device/host helpers for the CCQ cleaning kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ccq {

// ------------------------------------------------------------------------------------------
// activation dtypes
// ------------------------------------------------------------------------------------------
template <typename T> struct Act;
template <> struct Act<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct Act<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct Act<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float v) { *p = __float2half_rn(v); }
};

// ------------------------------------------------------------------------------------------
// documents: dense rows (cu_seqlens == nullptr) or varlen segments of a B == 1 batch
// ------------------------------------------------------------------------------------------
struct Seq {
  int64_t bos;   // first token row (in units of tokens of the flattened [B*T] axis)
  int len;       // tokens in the document
};

// In the varlen form (B == 1, T = total tokens) every offset is clamped into [0, T] and each end to
// at least its start, so a malformed cu_seqlens (not starting at 0, decreasing, past the end) gives
// wrong documents but never an index outside the token tensors or the per-chunk workspaces.
__device__ __forceinline__ Seq seq_of(int n, int T, const int64_t* cu_seqlens) {
  Seq s;
  if (cu_seqlens == nullptr) {
    s.bos = (int64_t)n * T;
    s.len = T;
  } else {
    int64_t a = cu_seqlens[n], b = cu_seqlens[n + 1];
    a = a < 0 ? 0 : (a > T ? T : a);
    b = b < a ? a : (b > T ? T : b);
    s.bos = a;
    s.len = (int)(b - a);
  }
  return s;
}

// Varlen launch order: document index of launch slot r, longest document first (LPT), so that a
// long document does not start in a late wave of CTAs and set the kernel's tail.  `order` is
// written by lpt_order() (tc.cu); nullptr means launch order = document order.
__device__ __forceinline__ int doc_of_slot(int r, const int* order) { return order ? order[r] : r; }

// Chunk slot of a document's first chunk in per-chunk workspaces: floor(bos / BT) + n.
// Slots of consecutive documents never overlap (floor(a) + ceil(b) <= floor(a + b) + 1), and
// the total is at most floor(B*T / BT) + n_seqs + 1.
__device__ __forceinline__ int64_t chunk_slot0(int n, int64_t bos, int BT) { return bos / BT + n; }

__host__ __device__ inline int64_t chunk_slots_total(int64_t total_tokens, int n_seqs, int BT) {
  return total_tokens / BT + n_seqs + 1;
}

__device__ __forceinline__ float position_of(int t_local, int position_offset) {
  float p = (float)(t_local + 1 + position_offset);
  return p < 1.0f ? 1.0f : p;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace ccq
