// SIMT (CUDA-core, fp32 arithmetic) forward and backward of the CCQ cleaning operator.
//
// This is the exact path: fp32 activations (the 1e-5 parity bar), any head size K <= 256, and
// the fallback for shapes the tcgen05 path does not take.  One CTA owns one (document, head,
// column tile of the state) and walks the document's chunks in order, keeping its slice of the
// covariance state C[:, v0:v0+VT] on chip; nothing but the inputs and outputs touches HBM in the
// forward.  The math is the reference's (ccq/ops/common/fused_read.py:11-25); the chunked
// decomposition is z = q C_prev + tril(q k^T) k within a chunk of BT tokens.
#include "args.h"
#include "common.cuh"

namespace ccq {
namespace {

constexpr int NT = 256;  // threads per CTA, viewed as a 16 x 16 grid (ty, tx)

// acc[i][j] += sum_{kk < KD} A(ty + 16 i, kk) * B(kk, tx + 16 j), operands in shared memory
// addressed through (row, k) strides so that transposed operands need no copy.
template <int MI, int NJ>
__device__ __forceinline__ void mm(float (&acc)[MI][NJ], int KD, const float* A, int a_rs, int a_ks,
                                   const float* B, int b_ks, int b_cs, int ty, int tx) {
#pragma unroll 2
  for (int kk = 0; kk < KD; ++kk) {
    float av[MI], bv[NJ];
#pragma unroll
    for (int i = 0; i < MI; ++i) av[i] = A[(ty + 16 * i) * a_rs + kk * a_ks];
#pragma unroll
    for (int j = 0; j < NJ; ++j) bv[j] = B[kk * b_ks + (tx + 16 * j) * b_cs];
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
      for (int j = 0; j < NJ; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
  }
}

template <int MI, int NJ>
__device__ __forceinline__ void zero(float (&acc)[MI][NJ]) {
#pragma unroll
  for (int i = 0; i < MI; ++i)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[i][j] = 0.f;
}

template <int KP_, int VT_, int BT_>
struct Cfg {
  static constexpr int KP = KP_, VT = VT_, BT = BT_;
  static constexpr int QS = KP + 1, AS = BT + 1, CS = VT + 1, MS = VT + 1;
  static constexpr size_t fwd_floats = 2 * BT * QS + BT * AS + KP * CS + BT * MS + 2 * KP + 4 * BT;
  static constexpr size_t bwd_floats = 3 * BT * QS + 2 * BT * AS + 2 * KP * CS + BT * MS + 2 * KP + VT + 8 * BT;
};

// load a [BT, KP] token tile (rows beyond the document or columns beyond K are zero)
template <typename Tin, int BT, int KP, int QS>
__device__ __forceinline__ void load_tile(float* dst, const Tin* src, const Seq& sq, int t0, int h, int H, int K) {
  for (int i = threadIdx.x; i < BT * KP; i += NT) {
    int t = i / KP, kk = i - t * KP;
    float v = 0.f;
    if (t0 + t < sq.len && kk < K) v = Act<Tin>::load(src + ((sq.bos + t0 + t) * H + h) * (int64_t)K + kk);
    dst[t * QS + kk] = v;
  }
}

// per-token lambda and 1/pos for one chunk; GATE mode computes sigmoid(W[h] . q_t + b[h])
template <typename Tin, int BT, int KP, int QS>
__device__ __forceinline__ void chunk_scalars(const CleanArgs& a, const Seq& sq, int t0, int h, const float* s_q,
                                              const float* s_w, float gate_b, float* s_lam, float* s_ipos,
                                              float* lam_store) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = warp; t < BT; t += NT / 32) {
    const bool valid = t0 + t < sq.len;
    float lamv = 0.f;
    if (a.lambda_mode == LAMBDA_GATE) {
      float d = 0.f;
      for (int kk = lane; kk < KP; kk += 32) d = fmaf(s_w[kk], s_q[t * QS + kk], d);
      d = warp_sum(d);
      lamv = valid ? sigmoidf_(d + gate_b) : 0.f;
      if (lane == 0 && valid && lam_store) lam_store[(sq.bos + t0 + t) * a.H + h] = lamv;
    } else if (valid) {
      lamv = Act<Tin>::load((const Tin*)a.lam + (sq.bos + t0 + t) * a.H + h);
    }
    if (lane == 0) {
      s_lam[t] = lamv;
      s_ipos[t] = 1.f / position_of(t0 + t, a.position_offset);
    }
  }
}

// ------------------------------------------------------------------------------------------
// forward
// ------------------------------------------------------------------------------------------
template <typename Tin, class C>
__global__ void __launch_bounds__(NT) simt_fwd_kernel(CleanArgs a) {
  constexpr int KP = C::KP, VT = C::VT, BT = C::BT, QS = C::QS, AS = C::AS, CS = C::CS, MS = C::MS;
  const int vt = blockIdx.x, h = blockIdx.y, n = blockIdx.z;
  const int v0 = vt * VT;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int H = a.H, K = a.K;
  const Seq sq = seq_of(n, a.T, a.cu_seqlens);

  extern __shared__ float smem[];
  float* s_q = smem;
  float* s_k = s_q + BT * QS;
  float* s_A = s_k + BT * QS;
  float* s_C = s_A + BT * AS;
  float* s_mc = s_C + KP * CS;
  float* s_m = s_mc + BT * MS;
  float* s_w = s_m + KP;
  float* s_lam = s_w + KP;
  float* s_ipos = s_lam + BT;
  float* s_sp = s_ipos + BT;

  const Tin* q = (const Tin*)a.q;
  const Tin* kp = (const Tin*)a.k;
  Tin* out = (Tin*)a.q_clean;
  const int64_t st_base = ((int64_t)n * H + h) * K;

  for (int i = tid; i < KP * VT; i += NT) {
    int r = i / VT, c = i - r * VT, v = v0 + c;
    float val = 0.f;
    if (a.initial_cov && r < K && v < K) val = a.initial_cov[(st_base + r) * K + v];
    s_C[r * CS + c] = val;
  }
  for (int i = tid; i < KP; i += NT) {
    s_m[i] = (a.subtract_mean && a.initial_mean && i < K) ? a.initial_mean[st_base + i] : 0.f;
    s_w[i] = (a.lambda_mode == LAMBDA_GATE && i < K) ? a.gate_w[(int64_t)h * K + i] : 0.f;
  }
  const float gate_b = a.lambda_mode == LAMBDA_GATE ? a.gate_b[h] : 0.f;
  __syncthreads();

  const int nchunks = (sq.len + BT - 1) / BT;
  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * BT;
    load_tile<Tin, BT, KP, QS>(s_q, q, sq, t0, h, H, K);
    load_tile<Tin, BT, KP, QS>(s_k, kp, sq, t0, h, H, K);
    __syncthreads();
    chunk_scalars<Tin, BT, KP, QS>(a, sq, t0, h, s_q, s_w, gate_b, s_lam, s_ipos, nullptr);
    {  // A = tril(q k^T)
      float acc[BT / 16][BT / 16];
      zero(acc);
      mm(acc, KP, s_q, QS, 1, s_k, 1, QS, ty, tx);
#pragma unroll
      for (int i = 0; i < BT / 16; ++i)
#pragma unroll
        for (int j = 0; j < BT / 16; ++j) {
          int t = ty + 16 * i, jj = tx + 16 * j;
          s_A[t * AS + jj] = jj <= t ? acc[i][j] : 0.f;
        }
    }
    __syncthreads();
    if (a.token_aux && vt == 0) {
      for (int t = tid; t < BT; t += NT)
        if (t0 + t < sq.len) {
          float* aux = a.token_aux + ((sq.bos + t0 + t) * H + h) * 2;
          aux[0] = s_lam[t];
          if (!a.subtract_mean) aux[1] = 0.f;
        }
    }
    if (a.subtract_mean) {
      // s_t = m_prev . q_t + sum_{j<=t} A[t][j];  s_sp = s_t / pos_t^2
      const int warp = tid >> 5, lane = tid & 31;
      for (int t = warp; t < BT; t += NT / 32) {
        float d = 0.f;
        for (int kk = lane; kk < KP; kk += 32) d = fmaf(s_m[kk], s_q[t * QS + kk], d);
        for (int j = lane; j < BT; j += 32) d += s_A[t * AS + j];
        d = warp_sum(d);
        if (lane == 0) s_sp[t] = d * s_ipos[t] * s_ipos[t];
        if (lane == 0 && vt == 0 && a.token_aux && t0 + t < sq.len)
          a.token_aux[((sq.bos + t0 + t) * H + h) * 2 + 1] = d;
      }
      // running key sum inside the chunk for this column tile
      for (int cc = tid; cc < VT; cc += NT) {
        float run = (v0 + cc < KP) ? s_m[v0 + cc] : 0.f;
        for (int t = 0; t < BT; ++t) {
          run += (v0 + cc < KP) ? s_k[t * QS + v0 + cc] : 0.f;
          s_mc[t * MS + cc] = run;
        }
      }
    }
    __syncthreads();
    {  // z = q C_prev + A k ; q_clean = q - lam (z / pos - s m / pos^2)
      float acc[BT / 16][VT / 16];
      zero(acc);
      mm(acc, KP, s_q, QS, 1, s_C, CS, 1, ty, tx);
      mm(acc, BT, s_A, AS, 1, s_k + v0, QS, 1, ty, tx);
#pragma unroll
      for (int i = 0; i < BT / 16; ++i)
#pragma unroll
        for (int j = 0; j < VT / 16; ++j) {
          int t = ty + 16 * i, cc = tx + 16 * j, v = v0 + cc;
          if (t0 + t < sq.len && v < K) {
            float corr = acc[i][j] * s_ipos[t];
            if (a.subtract_mean) corr -= s_sp[t] * s_mc[t * MS + cc];
            float o = s_q[t * QS + v] - s_lam[t] * corr;
            Act<Tin>::store(out + ((sq.bos + t0 + t) * H + h) * (int64_t)K + v, o);
          }
        }
    }
    __syncthreads();
    {  // C[:, tile] += k^T k[:, tile] ; m += sum_t k_t
      float acc[KP / 16][VT / 16];
      zero(acc);
      mm(acc, BT, s_k, 1, QS, s_k + v0, QS, 1, ty, tx);
#pragma unroll
      for (int i = 0; i < KP / 16; ++i)
#pragma unroll
        for (int j = 0; j < VT / 16; ++j) s_C[(ty + 16 * i) * CS + tx + 16 * j] += acc[i][j];
      for (int kk = tid; kk < KP; kk += NT) {
        float s = 0.f;
        for (int t = 0; t < BT; ++t) s += s_k[t * QS + kk];
        s_m[kk] += s;
      }
    }
    __syncthreads();
  }
  if (a.final_cov) {
    for (int i = tid; i < KP * VT; i += NT) {
      int r = i / VT, cc = i - r * VT, v = v0 + cc;
      if (r < K && v < K) a.final_cov[(st_base + r) * K + v] = s_C[r * CS + cc];
    }
  }
  if (a.final_mean && vt == 0) {
    for (int i = tid; i < K; i += NT) a.final_mean[st_base + i] = s_m[i];
  }
}

// ------------------------------------------------------------------------------------------
// backward: a forward sweep checkpoints C_prev / m_prev per chunk into the workspace, then a
// reverse sweep carries S = dC + dC^T (for dk) and the dm suffix, chunk by chunk.
// ------------------------------------------------------------------------------------------
struct BwdWs {
  float* C;     // [slots, H, K, K]   C at each chunk start
  float* m;     // [NV, slots, H, K]  m at each chunk start (one copy per column tile)
  float* dlp;   // [NV, B*T*H]        per-tile partials of dlambda
  float* lam;   // [B*T*H]            lambda (GATE mode)
  float* dpre;  // [B*T*H]            dlambda * sigma'(.) (GATE mode)
  float* gpart; // [H, NBG, K + 1]    gate-gradient partials
};
constexpr int NBG = 64;

inline BwdWs carve_bwd(void* base, int B, int T, int H, int K, int n_seqs, int NV, int BT) {
  BwdWs w;
  char* p = (char*)base;
  const int64_t slots = chunk_slots_total((int64_t)B * T, n_seqs, BT);
  const int64_t ntok = (int64_t)B * T * H;
  w.C = (float*)p; p += ws_align(sizeof(float) * slots * H * K * K);
  w.m = (float*)p; p += ws_align(sizeof(float) * NV * slots * H * K);
  w.dlp = (float*)p; p += ws_align(sizeof(float) * NV * ntok);
  w.lam = (float*)p; p += ws_align(sizeof(float) * ntok);
  w.dpre = (float*)p; p += ws_align(sizeof(float) * ntok);
  w.gpart = (float*)p; p += ws_align(sizeof(float) * H * NBG * (K + 1));
  return w;
}

inline size_t bwd_ws_bytes(int B, int T, int H, int K, int n_seqs, int NV, int BT) {
  const int64_t slots = chunk_slots_total((int64_t)B * T, n_seqs, BT);
  const int64_t ntok = (int64_t)B * T * H;
  return ws_align(sizeof(float) * slots * H * K * K) + ws_align(sizeof(float) * NV * slots * H * K) +
         ws_align(sizeof(float) * NV * ntok) + 2 * ws_align(sizeof(float) * ntok) +
         ws_align(sizeof(float) * H * NBG * (K + 1));
}

template <typename Tin, class C>
__global__ void __launch_bounds__(NT) simt_bwd_kernel(CleanArgs a, BwdWs ws) {
  constexpr int KP = C::KP, VT = C::VT, BT = C::BT, QS = C::QS, AS = C::AS, CS = C::CS, MS = C::MS;
  const int vt = blockIdx.x, h = blockIdx.y, n = blockIdx.z, NV = gridDim.x;
  const int v0 = vt * VT;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int H = a.H, K = a.K;
  const Seq sq = seq_of(n, a.T, a.cu_seqlens);
  const int64_t slot0 = chunk_slot0(n, sq.bos, BT);
  const int64_t st_base = ((int64_t)n * H + h) * K;
  const int64_t ntok = (int64_t)a.B * a.T * H;

  extern __shared__ float smem[];
  float* s_q = smem;
  float* s_k = s_q + BT * QS;
  float* s_g = s_k + BT * QS;       // dq_clean
  float* s_A = s_g + BT * QS;
  float* s_D = s_A + BT * AS;
  float* s_C = s_D + BT * AS;
  float* s_S = s_C + KP * CS;
  float* s_mc = s_S + KP * CS;
  float* s_m = s_mc + BT * MS;
  float* s_w = s_m + KP;
  float* s_carry = s_w + KP;        // [VT]
  float* s_lam = s_carry + VT;
  float* s_ipos = s_lam + BT;
  float* s_s = s_ipos + BT;
  float* s_wt = s_s + BT;
  float* s_ds = s_wt + BT;
  float* s_dmg = s_ds + BT;

  const Tin* q = (const Tin*)a.q;
  const Tin* kp = (const Tin*)a.k;
  const Tin* dqc = (const Tin*)a.dq_clean;
  Tin* dq = (Tin*)a.dq;
  Tin* dk = (Tin*)a.dk;
  const int nchunks = (sq.len + BT - 1) / BT;

  // ---- forward sweep: checkpoint C[:, tile] and m at every chunk start
  for (int i = tid; i < KP * VT; i += NT) {
    int r = i / VT, c = i - r * VT, v = v0 + c;
    float val = 0.f;
    if (a.initial_cov && r < K && v < K) val = a.initial_cov[(st_base + r) * K + v];
    s_C[r * CS + c] = val;
  }
  for (int i = tid; i < KP; i += NT) {
    s_m[i] = (a.subtract_mean && a.initial_mean && i < K) ? a.initial_mean[st_base + i] : 0.f;
    s_w[i] = (a.lambda_mode == LAMBDA_GATE && i < K) ? a.gate_w[(int64_t)h * K + i] : 0.f;
  }
  const float gate_b = a.lambda_mode == LAMBDA_GATE ? a.gate_b[h] : 0.f;
  __syncthreads();
  for (int c = 0; c < nchunks; ++c) {
    const int64_t slot = slot0 + c;
    float* wc = ws.C + (slot * H + h) * (int64_t)K * K;
    for (int i = tid; i < KP * VT; i += NT) {
      int r = i / VT, cc = i - r * VT, v = v0 + cc;
      if (r < K && v < K) wc[(int64_t)r * K + v] = s_C[r * CS + cc];
    }
    float* wm = ws.m + (((int64_t)vt * chunk_slots_total((int64_t)a.B * a.T, a.n_seqs, BT) + slot) * H + h) * K;
    for (int i = tid; i < K; i += NT) wm[i] = s_m[i];
    load_tile<Tin, BT, KP, QS>(s_k, kp, sq, c * BT, h, H, K);
    __syncthreads();
    float acc[KP / 16][VT / 16];
    zero(acc);
    mm(acc, BT, s_k, 1, QS, s_k + v0, QS, 1, ty, tx);
#pragma unroll
    for (int i = 0; i < KP / 16; ++i)
#pragma unroll
      for (int j = 0; j < VT / 16; ++j) s_C[(ty + 16 * i) * CS + tx + 16 * j] += acc[i][j];
    for (int kk = tid; kk < KP; kk += NT) {
      float s = 0.f;
      for (int t = 0; t < BT; ++t) s += s_k[t * QS + kk];
      s_m[kk] += s;
    }
    __syncthreads();
  }

  // ---- reverse sweep
  for (int i = tid; i < KP * VT; i += NT) {
    int r = i / VT, c = i - r * VT, v = v0 + c;
    float val = 0.f;
    if (a.dfinal_cov && r < K && v < K)
      val = a.dfinal_cov[(st_base + r) * K + v] + a.dfinal_cov[(st_base + v) * K + r];
    s_S[r * CS + c] = val;
  }
  for (int i = tid; i < VT; i += NT)
    s_carry[i] = (a.dfinal_mean && v0 + i < K) ? a.dfinal_mean[st_base + v0 + i] : 0.f;
  __syncthreads();

  const int64_t slots_total = chunk_slots_total((int64_t)a.B * a.T, a.n_seqs, BT);
  for (int c = nchunks - 1; c >= 0; --c) {
    const int t0 = c * BT;
    const int64_t slot = slot0 + c;
    load_tile<Tin, BT, KP, QS>(s_q, q, sq, t0, h, H, K);
    load_tile<Tin, BT, KP, QS>(s_k, kp, sq, t0, h, H, K);
    load_tile<Tin, BT, KP, QS>(s_g, dqc, sq, t0, h, H, K);
    {
      const float* wc = ws.C + (slot * H + h) * (int64_t)K * K;
      for (int i = tid; i < KP * VT; i += NT) {
        int r = i / VT, cc = i - r * VT, v = v0 + cc;
        s_C[r * CS + cc] = (r < K && v < K) ? wc[(int64_t)r * K + v] : 0.f;
      }
      const float* wm = ws.m + (((int64_t)vt * slots_total + slot) * H + h) * K;
      for (int i = tid; i < KP; i += NT) s_m[i] = i < K ? wm[i] : 0.f;
    }
    __syncthreads();
    chunk_scalars<Tin, BT, KP, QS>(a, sq, t0, h, s_q, s_w, gate_b, s_lam, s_ipos,
                                   (vt == 0 && a.lambda_mode == LAMBDA_GATE) ? ws.lam : nullptr);
    {  // A = tril(q k^T), D = tril(dqc k^T)
      float acc[BT / 16][BT / 16], acc2[BT / 16][BT / 16];
      zero(acc);
      zero(acc2);
      mm(acc, KP, s_q, QS, 1, s_k, 1, QS, ty, tx);
      mm(acc2, KP, s_g, QS, 1, s_k, 1, QS, ty, tx);
#pragma unroll
      for (int i = 0; i < BT / 16; ++i)
#pragma unroll
        for (int j = 0; j < BT / 16; ++j) {
          int t = ty + 16 * i, jj = tx + 16 * j;
          s_A[t * AS + jj] = jj <= t ? acc[i][j] : 0.f;
          s_D[t * AS + jj] = jj <= t ? acc2[i][j] : 0.f;
        }
    }
    __syncthreads();
    {  // s_t = m_t . q_t, w_t = m_t . dqc_t, ds_t, dmg_t
      const int warp = tid >> 5, lane = tid & 31;
      for (int t = warp; t < BT; t += NT / 32) {
        float ds = 0.f, dmg = 0.f, s = 0.f, w = 0.f;
        if (a.subtract_mean) {
          for (int kk = lane; kk < KP; kk += 32) {
            s = fmaf(s_m[kk], s_q[t * QS + kk], s);
            w = fmaf(s_m[kk], s_g[t * QS + kk], w);
          }
          for (int j = lane; j < BT; j += 32) {
            s += s_A[t * AS + j];
            w += s_D[t * AS + j];
          }
          s = warp_sum(s);
          w = warp_sum(w);
          const float ip2 = s_ipos[t] * s_ipos[t];
          ds = s_lam[t] * w * ip2;
          dmg = s_lam[t] * s * ip2;
        }
        if (lane == 0) {
          s_s[t] = s;
          s_wt[t] = w;
          s_ds[t] = ds;
          s_dmg[t] = dmg;
        }
      }
      if (a.subtract_mean) {
        for (int cc = tid; cc < VT; cc += NT) {
          float run = (v0 + cc < KP) ? s_m[v0 + cc] : 0.f;
          for (int t = 0; t < BT; ++t) {
            run += (v0 + cc < KP) ? s_k[t * QS + v0 + cc] : 0.f;
            s_mc[t * MS + cc] = run;
          }
        }
      }
    }
    __syncthreads();
    {  // z tile -> partial dlambda ; dq tile
      float z[BT / 16][VT / 16], g1[BT / 16][VT / 16];
      zero(z);
      zero(g1);
      mm(z, KP, s_q, QS, 1, s_C, CS, 1, ty, tx);
      mm(z, BT, s_A, AS, 1, s_k + v0, QS, 1, ty, tx);
      mm(g1, KP, s_g, QS, 1, s_C, CS, 1, ty, tx);  // dqc C_prev (scaled by -lam/pos below)
#pragma unroll
      for (int i = 0; i < BT / 16; ++i) {
        const int t = ty + 16 * i;
        float u = 0.f;
#pragma unroll
        for (int j = 0; j < VT / 16; ++j) {
          const int v = v0 + tx + 16 * j;
          if (v < K) u = fmaf(s_g[t * QS + v], z[i][j], u);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o);
        if (tx == 0 && t0 + t < sq.len) {
          float dl = -u * s_ipos[t];
          if (a.subtract_mean && vt == 0) dl += s_s[t] * s_wt[t] * s_ipos[t] * s_ipos[t];
          ws.dlp[(int64_t)vt * ntok + (sq.bos + t0 + t) * H + h] = dl;
        }
      }
      __syncthreads();  // every thread is done with the unscaled A and D
      // B = -alpha D ; A' = -alpha A (rows scaled by -lambda_t / pos_t)
      for (int i = tid; i < BT * BT; i += NT) {
        int t = i / BT, jj = i - t * BT;
        const float na = -s_lam[t] * s_ipos[t];
        s_D[t * AS + jj] *= na;
        s_A[t * AS + jj] *= na;
      }
      __syncthreads();
      float g2[BT / 16][VT / 16];
      zero(g2);
      mm(g2, BT, s_D, AS, 1, s_k + v0, QS, 1, ty, tx);
#pragma unroll
      for (int i = 0; i < BT / 16; ++i)
#pragma unroll
        for (int j = 0; j < VT / 16; ++j) {
          const int t = ty + 16 * i, cc = tx + 16 * j, v = v0 + cc;
          if (t0 + t < sq.len && v < K) {
            float r = s_g[t * QS + v] - s_lam[t] * s_ipos[t] * g1[i][j] + g2[i][j];
            if (a.subtract_mean) r += s_ds[t] * s_mc[t * MS + cc];
            Act<Tin>::store(dq + ((sq.bos + t0 + t) * H + h) * (int64_t)K + v, r);
          }
        }
    }
    __syncthreads();  // s_mc is reused for the dm suffix
    {  // dk tile = A'^T dqc + B^T q + k S + suffix(dm) + carry
      for (int cc = tid; cc < VT; cc += NT) {
        float run = s_carry[cc];
        const int v = v0 + cc;
        for (int t = BT - 1; t >= 0; --t) {
          if (a.subtract_mean && v < KP) run += s_dmg[t] * s_g[t * QS + v] + s_ds[t] * s_q[t * QS + v];
          s_mc[t * MS + cc] = run;
        }
        s_carry[cc] = run;
      }
      float acc[BT / 16][VT / 16];
      zero(acc);
      mm(acc, BT, s_A, 1, AS, s_g + v0, QS, 1, ty, tx);
      mm(acc, BT, s_D, 1, AS, s_q + v0, QS, 1, ty, tx);
      mm(acc, KP, s_k, QS, 1, s_S, CS, 1, ty, tx);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < BT / 16; ++i)
#pragma unroll
        for (int j = 0; j < VT / 16; ++j) {
          const int t = ty + 16 * i, cc = tx + 16 * j, v = v0 + cc;
          if (t0 + t < sq.len && v < K)
            Act<Tin>::store(dk + ((sq.bos + t0 + t) * H + h) * (int64_t)K + v, acc[i][j] + s_mc[t * MS + cc]);
        }
    }
    // S[:, tile] += sum_t qa_t dqc_t^T + dqc_t qa_t^T with qa = -alpha q
    for (int i = tid; i < BT * KP; i += NT) {
      int t = i / KP, kk = i - t * KP;
      s_q[t * QS + kk] *= -s_lam[t] * s_ipos[t];
    }
    __syncthreads();
    {
      float acc[KP / 16][VT / 16];
      zero(acc);
      mm(acc, BT, s_q, 1, QS, s_g + v0, QS, 1, ty, tx);
      mm(acc, BT, s_g, 1, QS, s_q + v0, QS, 1, ty, tx);
#pragma unroll
      for (int i = 0; i < KP / 16; ++i)
#pragma unroll
        for (int j = 0; j < VT / 16; ++j) s_S[(ty + 16 * i) * CS + tx + 16 * j] += acc[i][j];
    }
    __syncthreads();
  }
  if (a.dinitial_mean && (a.subtract_mean || a.dfinal_mean)) {
    for (int i = tid; i < VT; i += NT)
      if (v0 + i < K) a.dinitial_mean[st_base + v0 + i] = s_carry[i];
  }
}

// dlambda = sum of the per-tile partials; GATE mode turns it into dpre = dlambda * lam (1 - lam)
__global__ void dlam_reduce_kernel(CleanArgs a, BwdWs ws, int NV) {
  const int64_t ntok = (int64_t)a.B * a.T * a.H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < ntok; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int v = 0; v < NV; ++v) s += ws.dlp[(int64_t)v * ntok + i];
    if (a.lambda_mode == LAMBDA_GATE) {
      const float l = ws.lam[i];
      ws.dpre[i] = s * l * (1.f - l);
    } else if (a.dlam) {
      a.dlam[i] = s;
    }
  }
}

// GATE mode: dq += dpre * W[h]; partial dW/db per (head, block)
template <typename Tin>
__global__ void gate_bwd_kernel(CleanArgs a, BwdWs ws) {
  const int h = blockIdx.y, nb = blockIdx.x, H = a.H, K = a.K;
  const int64_t ntoks = (int64_t)a.B * a.T;
  const int64_t per = (ntoks + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = nb * per, r1 = r0 + per < ntoks ? r0 + per : ntoks;
  const Tin* q = (const Tin*)a.q;
  Tin* dq = (Tin*)a.dq;
  __shared__ float s_db[8];
  float db = 0.f;
  for (int d = threadIdx.x; d < K; d += blockDim.x) {
    const float w = a.gate_w[(int64_t)h * K + d];
    float acc = 0.f;
    for (int64_t r = r0; r < r1; ++r) {
      const float dp = ws.dpre[r * H + h];
      const int64_t off = (r * H + h) * K + d;
      acc = fmaf(dp, Act<Tin>::load(q + off), acc);
      Act<Tin>::store(dq + off, Act<Tin>::load(dq + off) + dp * w);
    }
    ws.gpart[((int64_t)h * NBG + nb) * (K + 1) + d] = acc;
  }
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) db += ws.dpre[r * H + h];
  db = warp_sum(db);
  if ((threadIdx.x & 31) == 0) s_db[threadIdx.x >> 5] = db;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += s_db[i];
    ws.gpart[((int64_t)h * NBG + nb) * (K + 1) + K] = s;
  }
}

__global__ void gate_reduce_kernel(CleanArgs a, BwdWs ws, int nblocks) {
  const int h = blockIdx.x, K = a.K;
  for (int d = threadIdx.x; d <= K; d += blockDim.x) {
    float s = 0.f;
    for (int nb = 0; nb < nblocks; ++nb) s += ws.gpart[((int64_t)h * NBG + nb) * (K + 1) + d];
    if (d < K) a.dgate_w[(int64_t)h * K + d] = s;
    else a.dgate_b[h] = s;
  }
}

// dC_0 = dC_T + sum_t q_t dz_t^T, dz_t = -lam_t dqc_t / pos_t ; one 32x32 tile per CTA
template <typename Tin>
__global__ void __launch_bounds__(256) dh0_kernel(CleanArgs a, BwdWs ws) {
  const int kt = blockIdx.x / ((a.K + 31) / 32), vtile = blockIdx.x % ((a.K + 31) / 32);
  const int nh = blockIdx.y, n = nh / a.H, h = nh % a.H, H = a.H, K = a.K;
  const Seq sq = seq_of(n, a.T, a.cu_seqlens);
  const Tin* q = (const Tin*)a.q;
  const Tin* g = (const Tin*)a.dq_clean;
  __shared__ float s_q[32][33], s_z[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t0 = 0; t0 < sq.len; t0 += 32) {
    for (int i = threadIdx.x; i < 32 * 32; i += 256) {
      const int t = i >> 5, d = i & 31;
      float qv = 0.f, zv = 0.f;
      if (t0 + t < sq.len) {
        const int64_t row = sq.bos + t0 + t;
        const float lamv = a.lambda_mode == LAMBDA_GATE ? ws.lam[row * H + h]
                                                        : Act<Tin>::load((const Tin*)a.lam + row * H + h);
        const float na = -lamv / position_of(t0 + t, a.position_offset);
        if (kt * 32 + d < K) qv = Act<Tin>::load(q + (row * H + h) * K + kt * 32 + d);
        if (vtile * 32 + d < K) zv = na * Act<Tin>::load(g + (row * H + h) * K + vtile * 32 + d);
      }
      s_q[t][d] = qv;
      s_z[t][d] = zv;
    }
    __syncthreads();
    for (int t = 0; t < 32; ++t) {
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = fmaf(s_q[t][ty + 8 * i], s_z[t][tx], acc[i]);
    }
    __syncthreads();
  }
  const int64_t base = ((int64_t)n * H + h) * K;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = kt * 32 + ty + 8 * i, v = vtile * 32 + tx;
    if (r < K && v < K) {
      float val = acc[i];
      if (a.dfinal_cov) val += a.dfinal_cov[(base + r) * K + v];
      a.dinitial_cov[(base + r) * K + v] = val;
    }
  }
}

template <typename Tin, class C>
cudaError_t launch_fwd(const CleanArgs& a, int* launches) {
  const size_t smem = C::fwd_floats * sizeof(float);
  auto kern = simt_fwd_kernel<Tin, C>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((a.K + C::VT - 1) / C::VT, a.H, a.n_seqs);
  kern<<<grid, NT, smem, a.stream>>>(a);
  *launches += 1;
  return cudaGetLastError();
}

template <typename Tin, class C>
cudaError_t launch_bwd(const CleanArgs& a, int* launches) {
  const int NV = (a.K + C::VT - 1) / C::VT;
  BwdWs ws = carve_bwd(a.workspace, a.B, a.T, a.H, a.K, a.n_seqs, NV, C::BT);
  const size_t smem = C::bwd_floats * sizeof(float);
  auto kern = simt_bwd_kernel<Tin, C>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(NV, a.H, a.n_seqs);
  kern<<<grid, NT, smem, a.stream>>>(a, ws);
  *launches += 1;
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int64_t ntok = (int64_t)a.B * a.T * a.H;
  const int rb = (int)((ntok + 255) / 256 < 4096 ? (ntok + 255) / 256 : 4096);
  if (a.dlam || a.lambda_mode == LAMBDA_GATE) {
    dlam_reduce_kernel<<<rb > 0 ? rb : 1, 256, 0, a.stream>>>(a, ws, NV);
    *launches += 1;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (a.lambda_mode == LAMBDA_GATE) {
    const int64_t ntoks = (int64_t)a.B * a.T;
    const int nb = (int)(ntoks < NBG ? (ntoks > 0 ? ntoks : 1) : NBG);
    gate_bwd_kernel<Tin><<<dim3(nb, a.H), 128, 0, a.stream>>>(a, ws);
    gate_reduce_kernel<<<a.H, 128, 0, a.stream>>>(a, ws, nb);
    *launches += 2;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (a.dinitial_cov) {
    const int kt = (a.K + 31) / 32;
    dh0_kernel<Tin><<<dim3(kt * kt, a.n_seqs * a.H), 256, 0, a.stream>>>(a, ws);
    *launches += 1;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

template <typename Tin>
cudaError_t fwd_by_k(const CleanArgs& a, int* l) {
  if (a.K <= 16) return launch_fwd<Tin, Cfg<16, 16, 64>>(a, l);
  if (a.K <= 32) return launch_fwd<Tin, Cfg<32, 32, 64>>(a, l);
  if (a.K <= 64) return launch_fwd<Tin, Cfg<64, 64, 64>>(a, l);
  if (a.K <= 128) return launch_fwd<Tin, Cfg<128, 64, 64>>(a, l);
  return launch_fwd<Tin, Cfg<256, 32, 32>>(a, l);
}

template <typename Tin>
cudaError_t bwd_by_k(const CleanArgs& a, int* l) {
  if (a.K <= 16) return launch_bwd<Tin, Cfg<16, 16, 64>>(a, l);
  if (a.K <= 32) return launch_bwd<Tin, Cfg<32, 32, 64>>(a, l);
  if (a.K <= 64) return launch_bwd<Tin, Cfg<64, 64, 64>>(a, l);
  if (a.K <= 128) return launch_bwd<Tin, Cfg<128, 64, 64>>(a, l);
  return launch_bwd<Tin, Cfg<256, 32, 32>>(a, l);
}

inline void k_cfg(int K, int* VT, int* BT) {
  if (K <= 16) { *VT = 16; *BT = 64; }
  else if (K <= 32) { *VT = 32; *BT = 64; }
  else if (K <= 64) { *VT = 64; *BT = 64; }
  else if (K <= 128) { *VT = 64; *BT = 64; }
  else { *VT = 32; *BT = 32; }
}

}  // namespace

size_t simt_bwd_workspace(int B, int T, int H, int K, int n_seqs) {
  int VT, BT;
  k_cfg(K, &VT, &BT);
  return bwd_ws_bytes(B, T, H, K, n_seqs, (K + VT - 1) / VT, BT);
}

cudaError_t simt_fwd(const CleanArgs& a, int* launches) {
  switch (a.dtype) {
    case DT_F32: return fwd_by_k<float>(a, launches);
    case DT_BF16: return fwd_by_k<__nv_bfloat16>(a, launches);
    default: return fwd_by_k<__half>(a, launches);
  }
}

cudaError_t simt_bwd(const CleanArgs& a, int* launches) {
  switch (a.dtype) {
    case DT_F32: return bwd_by_k<float>(a, launches);
    case DT_BF16: return bwd_by_k<__nv_bfloat16>(a, launches);
    default: return bwd_by_k<__half>(a, launches);
  }
}

}  // namespace ccq
