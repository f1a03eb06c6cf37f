// Recurrent (decode / short prefill) cleaning step over the generation cache.
//
// Per (document, head) and token t, with the fp32 cache state (C, m):
//   C <- C + k_t k_t^T ; m <- m + k_t ; z[v] = sum_k q_t[k] C[k, v]   (inclusive read)
//   q_clean_t = q_t - lambda_t (z / pos_t - (m . q_t) m / pos_t^2)
// This is fla fused_recurrent_gla(q, k, v=k, scale=1) followed by _CCQCleanQ at the cache's
// position offset, as fused_ccq_clean(use_chunk=False) runs it (ccq/ops/ccq_gdn/fused_clean.py:34-83).
//
// The step is bound by the fp32 state traffic (2 * K^2 * 4 bytes per head and token at T=1), so
// the kernel is a streaming pass: one CTA per (column tile, head, document); each thread keeps
// RPT rows x 4 columns of the state in registers (128-bit loads/stores), accumulates its share of
// z, and the partial sums meet in shared memory.  T > 1 keeps the state in registers across tokens.
#include <cooperative_groups.h>

#include "args.h"
#include "common.cuh"

namespace ccq {
namespace {

constexpr int DT = 256;  // threads per CTA

// VT: state columns per CTA (multiple of 4); NCG = VT / 4 column groups; RG = DT / NCG row groups.
// NORM: q and k arrive raw and are L2-normalised here as fla's l2norm does it (fp32 math, eps 1e-6,
// rounded to the activation dtype; fla/modules/l2norm.py:26-46), and the normalised k is written out.
template <typename Tin, int VT, int KMAX, int NORM>
__global__ void __launch_bounds__(DT) decode_kernel(CleanArgs a) {
  constexpr int NCG = VT / 4;
  constexpr int RG = DT / NCG;
  constexpr int RPT = (KMAX + RG - 1) / RG;  // rows per thread
  const int vt = blockIdx.x, h = blockIdx.y, n = blockIdx.z;
  const int tid = threadIdx.x, cg = tid % NCG, rg = tid / NCG;
  const int H = a.H, K = a.K;
  const int v = vt * VT + cg * 4;  // first column of this thread
  const bool colok = v < K;        // K % 4 == 0, so the whole float4 is in or out
  const Seq sq = seq_of(n, a.T, a.cu_seqlens);
  const int64_t st = ((int64_t)n * H + h) * K;

  __shared__ float s_q[KMAX], s_k[KMAX], s_m[KMAX], s_w[KMAX];
  __shared__ float4 s_z[RG][NCG];
  __shared__ float s_red[DT / 32];
  __shared__ float s_lam, s_s, s_rn[2];

  float4 c[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg + RG * i;
    c[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.cov_in && colok && r < K) c[i] = __ldcs(reinterpret_cast<const float4*>(a.cov_in + (st + r) * K + v));
  }
  for (int i = tid; i < K; i += DT) {
    s_m[i] = (a.subtract_mean && a.mean_in) ? a.mean_in[st + i] : 0.f;
    s_w[i] = a.lambda_mode == LAMBDA_GATE ? a.gate_w[(int64_t)h * K + i] : 0.f;
  }
  const Tin* q = (const Tin*)a.q;
  const Tin* kp = (const Tin*)a.k;
  Tin* out = (Tin*)a.q_clean;
  const int warp = tid >> 5, lane = tid & 31;

  for (int t = 0; t < sq.len; ++t) {
    const int64_t row = ((sq.bos + t) * H + h) * (int64_t)K;
    __syncthreads();  // previous token's readers of s_q/s_k/s_m are done
    if (NORM) {
      for (int i = tid; i < K; i += DT) {
        s_q[i] = Act<Tin>::load(q + row + i);
        s_k[i] = Act<Tin>::load(kp + row + i);
      }
      __syncthreads();
      if (warp < 2) {
        const float* x = warp == 0 ? s_q : s_k;
        float ss = 0.f;
        for (int i = lane; i < K; i += 32) ss = fmaf(x[i], x[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) s_rn[warp] = 1.0f / sqrtf(ss + 1e-6f);
      }
      __syncthreads();
      const float rq = s_rn[0], rk = s_rn[1];
      for (int i = tid; i < K; i += DT) {
        Tin qh, kh;
        Act<Tin>::store(&qh, s_q[i] * rq);
        Act<Tin>::store(&kh, s_k[i] * rk);
        const float kv = Act<Tin>::load(&kh);
        s_q[i] = Act<Tin>::load(&qh);
        s_k[i] = kv;
        s_m[i] += kv;
        if (vt == 0) reinterpret_cast<Tin*>(a.k_norm)[row + i] = kh;
      }
    } else {
      for (int i = tid; i < K; i += DT) {
        const float kv = Act<Tin>::load(kp + row + i);
        s_q[i] = Act<Tin>::load(q + row + i);
        s_k[i] = kv;
        s_m[i] += kv;
      }
    }
    __syncthreads();
    // s = m_t . q_t and (GATE) the lambda pre-activation, one warp each
    if (warp == 0) {
      float d = 0.f;
      for (int i = lane; i < K; i += 32) d = fmaf(s_m[i], s_q[i], d);
      d = warp_sum(d);
      if (lane == 0) s_s = d;
    } else if (warp == 1) {
      float lamv;
      if (a.lambda_mode == LAMBDA_GATE) {
        float d = 0.f;
        for (int i = lane; i < K; i += 32) d = fmaf(s_w[i], s_q[i], d);
        d = warp_sum(d);
        lamv = sigmoidf_(d + a.gate_b[h]);
      } else {
        lamv = Act<Tin>::load((const Tin*)a.lam + (sq.bos + t) * H + h);
      }
      if (lane == 0) s_lam = lamv;
    }
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    if (colok) {
      const float4 kc = *reinterpret_cast<const float4*>(&s_k[v]);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int r = rg + RG * i;
        if (r < K) {
          const float kr = s_k[r], qr = s_q[r];
          c[i].x = fmaf(kr, kc.x, c[i].x);
          c[i].y = fmaf(kr, kc.y, c[i].y);
          c[i].z = fmaf(kr, kc.z, c[i].z);
          c[i].w = fmaf(kr, kc.w, c[i].w);
          z.x = fmaf(qr, c[i].x, z.x);
          z.y = fmaf(qr, c[i].y, z.y);
          z.z = fmaf(qr, c[i].z, z.z);
          z.w = fmaf(qr, c[i].w, z.w);
        }
      }
    }
    s_z[rg][cg] = z;
    __syncthreads();
    if (tid < NCG && colok) {
      float4 acc = s_z[0][tid];
      for (int r = 1; r < RG; ++r) {
        const float4 p = s_z[r][tid];
        acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
      }
      const float ip = 1.f / position_of(t, a.position_offset);
      const float sp = a.subtract_mean ? s_s * ip * ip : 0.f;
      const float l = s_lam;
      const float zz[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int vv = v + e;
        const float corr = zz[e] * ip - sp * s_m[vv];
        Act<Tin>::store(out + row + vv, s_q[vv] - l * corr);
      }
    }
  }
  if (colok) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg + RG * i;
      if (r < K) __stcs(reinterpret_cast<float4*>(a.cov_out + (st + r) * K + v), c[i]);
    }
  }
  // The column tiles of one (document, head) form a thread-block cluster: every tile has read the
  // mean state before tile 0 writes it, so mean_out may alias mean_in.
  if (gridDim.x > 1) cooperative_groups::this_cluster().sync();
  if (a.subtract_mean && a.mean_out && vt == 0) {
    __syncthreads();
    for (int i = tid; i < K; i += DT) a.mean_out[st + i] = s_m[i];
  }
  (void)s_red;
}

// one launch; the column tiles of a (document, head) run as one cluster (gridDim.x CTAs, <= 8)
template <typename Tin, int VT, int KMAX, int NORM>
cudaError_t launch_tiles(const CleanArgs& a) {
  const unsigned tiles = (unsigned)((a.K + VT - 1) / VT);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, a.H, a.n_seqs);
  cfg.blockDim = dim3(DT);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = a.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = tiles;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = tiles > 1 ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, decode_kernel<Tin, VT, KMAX, NORM>, a);
}

template <typename Tin, int NORM>
cudaError_t launch_norm(const CleanArgs& a) {
  if (a.K <= 64) return launch_tiles<Tin, 64, 64, NORM>(a);
  if (a.K <= 128) return launch_tiles<Tin, 128, 128, NORM>(a);
  return launch_tiles<Tin, 64, 256, NORM>(a);
}

template <typename Tin>
cudaError_t launch(const CleanArgs& a, int* launches) {
  cudaError_t e = a.qk_norm ? launch_norm<Tin, 1>(a) : launch_norm<Tin, 0>(a);
  *launches += 1;
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t decode_step(const CleanArgs& a, int* launches) {
  switch (a.dtype) {
    case DT_F32: return launch<float>(a, launches);
    case DT_BF16: return launch<__nv_bfloat16>(a, launches);
    default: return launch<__half>(a, launches);
  }
}

}  // namespace ccq
