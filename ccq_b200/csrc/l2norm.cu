// Per-row L2 normalisation of q and k, forward and backward, as streaming kernels.
//
// fla's l2norm (fla/modules/l2norm.py:266, kernels at :26-76), which both fused_chunk orchestrators
// apply to q and k right before the cleaning operator (ccq/ops/ccq_gdn/fused_chunk.py:42-44,
// ccq/ops/ccq_gla/fused_chunk.py:31-32):
//   forward   r = 1 / sqrt(sum(x^2) + eps),  y = x * r        (fp32 math, y in the activation dtype)
//   backward  dx = r * (dy - y * sum(dy * y))                 (y the stored, rounded output)
// The tensor-core kernels fold the normalisation (and its backward) into their tiles; these kernels
// serve the exact fp32 / general-K path, whose gradient on the normalised keys (the operator's own
// plus the one arriving from the backbone) is mapped back here.
//
// One warp per row of K elements (K <= 256, K % 2 == 0); a row is a (token, head) vector.
#include "args.h"
#include "common.cuh"

namespace ccq {
namespace {

constexpr int NW = 8;  // warps (rows) per CTA
constexpr float kEps = 1e-6f;

template <typename Tin>
__device__ __forceinline__ float ld(const Tin* p, int64_t i) { return Act<Tin>::load(p + i); }
template <typename Tin>
__device__ __forceinline__ float rnd(float x) {  // the value after a store in the activation dtype
  Tin t;
  Act<Tin>::store(&t, x);
  return Act<Tin>::load(&t);
}

// y = x * r, r = 1 / sqrt(sum x^2 + eps); r written to r_out[2 * row + slot] when r_out is given.
template <typename Tin>
__global__ void __launch_bounds__(32 * NW) l2norm_fwd_kernel(const Tin* x, Tin* y, float* r_out, int slot, int64_t rows,
                                                           int K) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NW + (threadIdx.x >> 5);
  if (row >= rows) return;
  const Tin* xr = x + row * K;
  float ss = 0.f;
  for (int i = lane; i < K; i += 32) {
    const float v = ld(xr, i);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss + kEps);
  Tin* yr = y + row * K;
  for (int i = lane; i < K; i += 32) Act<Tin>::store(yr + i, ld(xr, i) * r);
  if (r_out && lane == 0) r_out[2 * row + slot] = r;
}

// y = x * r with r read from r_in[2 * row + slot] (recomputes a normalised tensor bit for bit)
template <typename Tin>
__global__ void __launch_bounds__(32 * NW) l2norm_scale_kernel(const Tin* x, Tin* y, const float* r_in, int slot,
                                                             int64_t rows, int K) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NW + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float r = r_in[2 * row + slot];
  const Tin* xr = x + row * K;
  Tin* yr = y + row * K;
  for (int i = lane; i < K; i += 32) Act<Tin>::store(yr + i, ld(xr, i) * r);
}

// d <- r * (s - y * sum(s * y)), s = d + d_ext rounded to the activation dtype (the sum autograd
// forms of the two gradients of the normalised tensor), in place on d.
template <typename Tin>
__global__ void __launch_bounds__(32 * NW) l2norm_bwd_kernel(Tin* d, const Tin* d_ext, const Tin* y, const float* r_in,
                                                           int slot, int64_t rows, int K) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * NW + (threadIdx.x >> 5);
  if (row >= rows) return;
  Tin* dr = d + row * K;
  const Tin* yr = y + row * K;
  const Tin* er = d_ext ? d_ext + row * K : nullptr;
  float dot = 0.f;
  for (int i = lane; i < K; i += 32) {
    float s = ld(dr, i);
    if (er) s = rnd<Tin>(s + ld(er, i));
    dot = fmaf(s, ld(yr, i), dot);
  }
  dot = warp_sum(dot);
  const float r = r_in[2 * row + slot];
  for (int i = lane; i < K; i += 32) {
    float s = ld(dr, i);
    if (er) s = rnd<Tin>(s + ld(er, i));
    Act<Tin>::store(dr + i, r * (s - ld(yr, i) * dot));
  }
}

// 16-bit rows of K = 128: sixteen lanes per row, eight elements (16 bytes) per lane and tensor, two
// rows per warp; the same arithmetic as l2norm_bwd_kernel.
template <typename Tin>
__global__ void __launch_bounds__(32 * NW) l2norm_bwd128_kernel(Tin* d, const Tin* d_ext, const Tin* y,
                                                              const float* r_in, int slot, int64_t rows) {
  const int lane = threadIdx.x & 31, sub = lane & 15;
  const int64_t row = ((int64_t)blockIdx.x * NW + (threadIdx.x >> 5)) * 2 + (lane >> 4);
  const bool ok = row < rows;
  const int64_t off = (ok ? row : 0) * 128 + sub * 8;
  float s[8], yv[8];
  uint4 dv = make_uint4(0, 0, 0, 0), ev = make_uint4(0, 0, 0, 0), yy = make_uint4(0, 0, 0, 0);
  if (ok) {
    dv = *reinterpret_cast<const uint4*>(d + off);
    yy = *reinterpret_cast<const uint4*>(y + off);
    if (d_ext) ev = *reinterpret_cast<const uint4*>(d_ext + off);
  }
  const Tin* dp = reinterpret_cast<const Tin*>(&dv);
  const Tin* ep = reinterpret_cast<const Tin*>(&ev);
  const Tin* yp = reinterpret_cast<const Tin*>(&yy);
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s[i] = Act<Tin>::load(dp + i);
    if (d_ext) s[i] = rnd<Tin>(s[i] + Act<Tin>::load(ep + i));
    yv[i] = Act<Tin>::load(yp + i);
    dot = fmaf(s[i], yv[i], dot);
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (!ok) return;
  const float r = r_in[2 * row + slot];
  uint4 out;
  Tin* op = reinterpret_cast<Tin*>(&out);
#pragma unroll
  for (int i = 0; i < 8; ++i) Act<Tin>::store(op + i, r * (s[i] - yv[i] * dot));
  *reinterpret_cast<uint4*>(d + off) = out;
}

template <typename Tin>
cudaError_t launch_fwd(const void* x, void* y, float* r_out, int slot, int64_t rows, int K, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + NW - 1) / NW);
  l2norm_fwd_kernel<Tin><<<grid, 32 * NW, 0, st>>>((const Tin*)x, (Tin*)y, r_out, slot, rows, K);
  return cudaGetLastError();
}
template <typename Tin>
cudaError_t launch_scale(const void* x, void* y, const float* r_in, int slot, int64_t rows, int K, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + NW - 1) / NW);
  l2norm_scale_kernel<Tin><<<grid, 32 * NW, 0, st>>>((const Tin*)x, (Tin*)y, r_in, slot, rows, K);
  return cudaGetLastError();
}
template <typename Tin>
cudaError_t launch_bwd(void* d, const void* d_ext, const void* y, const float* r_in, int slot, int64_t rows, int K,
                       cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const bool vec = sizeof(Tin) == 2 && K == 128 && ((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(y) |
                                                     reinterpret_cast<uintptr_t>(d_ext)) & 15) == 0;
  if (vec) {
    const unsigned grid = (unsigned)((rows + 2 * NW - 1) / (2 * NW));
    l2norm_bwd128_kernel<Tin><<<grid, 32 * NW, 0, st>>>((Tin*)d, (const Tin*)d_ext, (const Tin*)y, r_in, slot, rows);
    return cudaGetLastError();
  }
  const unsigned grid = (unsigned)((rows + NW - 1) / NW);
  l2norm_bwd_kernel<Tin><<<grid, 32 * NW, 0, st>>>((Tin*)d, (const Tin*)d_ext, (const Tin*)y, r_in, slot, rows, K);
  return cudaGetLastError();
}

}  // namespace

cudaError_t l2norm_rows_fwd(int dtype, const void* x, void* y, float* r_out, int slot, int64_t rows, int K,
                            cudaStream_t st) {
  if (dtype == DT_F32) return launch_fwd<float>(x, y, r_out, slot, rows, K, st);
  if (dtype == DT_BF16) return launch_fwd<__nv_bfloat16>(x, y, r_out, slot, rows, K, st);
  return launch_fwd<__half>(x, y, r_out, slot, rows, K, st);
}

cudaError_t l2norm_rows_scale(int dtype, const void* x, void* y, const float* r_in, int slot, int64_t rows, int K,
                              cudaStream_t st) {
  if (dtype == DT_F32) return launch_scale<float>(x, y, r_in, slot, rows, K, st);
  if (dtype == DT_BF16) return launch_scale<__nv_bfloat16>(x, y, r_in, slot, rows, K, st);
  return launch_scale<__half>(x, y, r_in, slot, rows, K, st);
}

cudaError_t l2norm_rows_bwd(int dtype, void* d, const void* d_ext, const void* y, const float* r_in, int slot,
                            int64_t rows, int K, cudaStream_t st) {
  if (dtype == DT_F32) return launch_bwd<float>(d, d_ext, y, r_in, slot, rows, K, st);
  if (dtype == DT_BF16) return launch_bwd<__nv_bfloat16>(d, d_ext, y, r_in, slot, rows, K, st);
  return launch_bwd<__half>(d, d_ext, y, r_in, slot, rows, K, st);
}

}  // namespace ccq
