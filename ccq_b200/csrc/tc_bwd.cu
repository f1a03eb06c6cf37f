// Tensor-core (tcgen05 / TMEM / TMA) backward of the CCQ cleaning operator, bf16 or fp16, K = 128.
//
// One CTA per (document, head) walks the document's chunks of BT = 64 tokens in REVERSE order.
// The forward's final state (C_T, m_T) and its per-token side outputs (lambda_t, s_t) are inputs,
// so the state before each chunk is recovered in TMEM (C -= K^T K, an MMA with negated A), and the
// reverse-scan gradient G = dL/dC (after the chunk) is accumulated in TMEM as well; neither state
// ever goes to HBM.  Per chunk, with Q, K, dQc = 64 x 128 tiles, alpha_t = lambda_t / pos_t:
//   B1  [D ; A]  = [dQc ; Q] K^T                           (M = 128 stacked, N = 64)
//   B5  C       -= K^T K                                   (-> C_prev)
//   B2  [z ; dq] = [0 ; dQc] + [Q ; dZ] bf16(C_prev)        dZ = -alpha dQc (TMEM starts from [0 ; dQc])
//   B2b [z ; dq] += [tril(A) ; P2] K                        P2 = (ds_t - alpha_t D)[j <= t]
//   B3  dk^T     = Q^T P2 + dQc^T P4 + G K^T + G^T K^T      P4 = (beta_t - alpha_t A)[j <= t]
//   B4  G       += Q^T dZ
//   CW  X += Q^T R,  Y += dQc^T R,  R = [ds | dpre | beta | 0]  (persistent 2 x 16 columns: carry =
//       X[0] + Y[2], dW = X[1]; R is double-buffered by chunk parity so CW of a chunk runs after B1 of
//       the next one)
// with ds_t = lambda w_t / pos^2, beta_t = lambda s_t / pos^2, w_t = m_t . dqc_t, and
//   dq_t = [dq]_t + ds_t m_prev (+ dpre_t W_h),  dlambda_t = -dqc_t . z_t / pos + s w / pos^2,
//   dk_j = [dk^T]_j + carry  (the in-chunk dm suffix is folded into P2 and P4).
// These are the reference's gradients (ccq/ops/common/fused_read.py:18-25, kernel :177-307,
// carry :355-376, dC0 / dm0 :420-450).
//
// NORM = 1 (the *_l2norm entry points): q is the raw input and k the forward's normalised keys; the
// aux warps rescale each chunk's Q rows in shared memory by the forward's 1/|q_t| (the same rounded
// products the forward formed), and the dq epilogue maps the gradient on the normalised q back
// through the normalisation, dq = (dq_hat - q_hat (q_hat . dq_hat)) / |q| (fla/modules/l2norm.py:49-72).
// The gradient on the normalised keys, plus the backbone's share of it (an input), is mapped back
// the same way in E3, against the normalised keys the stage's K tile still holds.
//
// Warp roles (384 threads): warp 0 TMA loads, warp 1 TMEM + MMA issue, warps 2-3 aux (partial-chunk
// key zeroing and the running key sum m walked backwards), warps 4-11 epilogue.  The epilogue writes
// dq straight from registers (a thread holds a full 128-byte row segment of it) and stages dk in the
// stage's K tile, which the TMA thread writes out with a bulk store before it reloads the stage.
#include "args.h"
#include "common.cuh"
#include "tc_common.cuh"
#include "tma_host.h"

namespace ccq {

namespace {
using namespace tc;

constexpr int B_THREADS = 384;
constexpr int B_BT = 64;
constexpr uint32_t B_QDPANEL = 24576;            // 192 rows: dQc (0-63), Q (64-127), dZ (128-191)
constexpr uint32_t B_QDTILE = 2 * B_QDPANEL;
constexpr uint32_t B_KPANEL = 8192;              // 64 rows
constexpr uint32_t B_KTILE = 2 * B_KPANEL;
constexpr uint32_t B_STAGE = B_QDTILE + B_KTILE; // 65536
constexpr uint32_t B_OFF_K = B_QDTILE;           // inside a stage
constexpr uint32_t B_OFF_C = 2 * B_STAGE;        // bf16 C_prev, 2 panels of 128 rows
constexpr uint32_t B_OFF_G = B_OFF_C + 32768;    // bf16 G, 2 panels of 128 rows
constexpr uint32_t B_OFF_AP = B_OFF_G + 32768;   // [tril(A) ; P2], 128 rows x 64
constexpr uint32_t B_OFF_P4 = B_OFF_AP + 16384;  // P4, 64 rows x 64
constexpr uint32_t B_OFF_R = B_OFF_P4 + 8192;    // R[2]: 16 rows x 64 each (K-major, rows = columns)
constexpr uint32_t B_OFF_SMALL = B_OFF_R + 4096; // 225280
constexpr uint32_t T_C = 0, T_G = 128, T_ZQ = 256, T_DA = 384, T_CW = 448;

struct BwdSmall {
  float m_buf[2][128];
  float wh[128];
  float wpart[2][64], upart[2][64];
  float w[64], ds[64], dpre[64];
  float qdot[2][64];  // NORM: [column half][token] partial q_hat . dq_hat
  uint64_t full[2], kready[2], empty[2], m_ready[2], m_free[2];
  uint64_t tinit, da_full, c_full, cconv, g_full, zq_full, dk_full, dk_read, cw_done, mma_done, ap_free;
  float db;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t B_SMEM = B_OFF_SMALL + sizeof(BwdSmall) + 1024;
static_assert(B_SMEM <= 232448, "backward kernel shared memory");
constexpr int EPI_WARPS = 8;

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"((unsigned short)v) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
// the first two of 4 consecutive fp32 TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld2f(uint32_t taddr, float* x) {
  uint32_t r0, r1, r2, r3;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(taddr));
  x[0] = __uint_as_float(r0);
  x[1] = __uint_as_float(r1);
  (void)r2;
  (void)r3;
}

// 16 TMEM lanes x 32 columns in the mma-fragment layout (shape 16x256b, 4 repeats): thread t holds
// lanes t/4 and t/4 + 8 of the 16, columns 8k + 2(t%4) and 8k + 2(t%4) + 1 for k = 0..3, as
// v[4k], v[4k+1] (lane t/4) and v[4k+2], v[4k+3] (lane t/4 + 8).
__device__ __forceinline__ void tmem_ld_frag(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// four 8x8 16-bit matrices in the mma-fragment layout stored transposed: thread 8m + i gives the
// address of stored row i of matrix m, which receives column i of that matrix
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};"
               ::"r"(addr), "r"(a0), "r"(a1), "r"(a2), "r"(a3) : "memory");
}

// the dm carry of this thread's lane: column 0 (Q^T ds) + column 18 (dQc^T beta) of the CW region
__device__ __forceinline__ float tmem_carry(uint32_t taddr) {
  uint32_t r0, r1, r2, r3, s0, s1, s2, s3;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%8];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%4, %5, %6, %7}, [%9];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(s0), "=r"(s1), "=r"(s2), "=r"(s3)
      : "r"(taddr), "r"(taddr + 16));
  (void)r1; (void)r2; (void)r3; (void)s0; (void)s1; (void)s3;
  return __uint_as_float(r0) + __uint_as_float(s2);
}

template <int AB16>
__device__ __forceinline__ uint32_t to16(float x) {
  if (AB16) return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
  return (uint32_t)__half_as_ushort(__float2half_rn(x));
}

// 8 packed 16-bit values as fp32
template <int AB16>
__device__ __forceinline__ void unpack8(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = unpack2<AB16>(w[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

// 8 consecutive 16-bit values of a swizzled panel row, as fp32
template <int AB16>
__device__ __forceinline__ void ld_row8(uint32_t panel, int row, int cc, float* f) {
  const uint4 v = ld_shared_v4(panel + sw128(row, cc));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = unpack2<AB16>(w[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

template <int AB16>
__device__ __forceinline__ void store_panel_row(uint32_t panel, int row, const float* v) {
#pragma unroll
  for (int cc = 0; cc < 8; ++cc)
    st_shared_v4(panel + sw128(row, cc), pack2<AB16>(v[8 * cc], v[8 * cc + 1]), pack2<AB16>(v[8 * cc + 2], v[8 * cc + 3]),
                 pack2<AB16>(v[8 * cc + 4], v[8 * cc + 5]), pack2<AB16>(v[8 * cc + 6], v[8 * cc + 7]));
}

template <int AB16, int NORM>
__global__ void __launch_bounds__(B_THREADS, 1)
    tc_bwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmg, const __grid_constant__ CUtensorMap tmdq,
                  const __grid_constant__ CUtensorMap tmdk, CleanArgs a, int* err, float* gate_part) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BwdSmall& S = *reinterpret_cast<BwdSmall*>(sm + B_OFF_SMALL);
  const uint32_t sbase = smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H;
  const int h = blockIdx.x % H, n = doc_of_slot(blockIdx.x / H, a.doc_order);
  const Seq sq = seq_of(n, a.T, a.cu_seqlens);
  const int nchunks = (sq.len + B_BT - 1) / B_BT;
  const int64_t st_base = ((int64_t)n * H + h) * 128;
  const bool sub_mean = a.subtract_mean != 0;
  const bool gate = a.lambda_mode == LAMBDA_GATE;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.kready[i], 1);
      mbar_init(&S.empty[i], 2 + EPI_WARPS);
      mbar_init(&S.m_ready[i], 1);
      mbar_init(&S.m_free[i], EPI_WARPS);
    }
    uint64_t* ones[] = {&S.da_full, &S.c_full, &S.g_full, &S.zq_full, &S.dk_full, &S.cw_done,
                        &S.mma_done};
    for (uint64_t* b : ones) mbar_init(b, 1);
    uint64_t* epis[] = {&S.tinit, &S.cconv, &S.dk_read, &S.ap_free};
    for (uint64_t* b : epis) mbar_init(b, EPI_WARPS);
    S.abort = 0;
    S.db = 0.f;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&S.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = S.tmem_base;
  volatile int* ab = &S.abort;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (chunks in reverse)
    // A stage is reloaded once every reader released it; by then the epilogue has staged that chunk's
    // dk in the stage's K tile, and this thread writes it out first (full chunks only).
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmg);
      tma_prefetch_desc(&tmdk);
      auto store_dk = [&](int j) {
        const int cj = nchunks - 1 - j;
        if (sq.len - cj * B_BT >= B_BT) {
          const int row = (int)(sq.bos + (int64_t)cj * B_BT);
          uint8_t* kt = sm + (j & 1) * B_STAGE + B_OFF_K;
          tma_store_3d(&tmdk, kt, 0, h, row);
          tma_store_3d(&tmdk, kt + B_KPANEL, 64, h, row);
          bulk_commit();
          bulk_wait_read();
        }
      };
      int issued = 0;
      for (int i = 0; i < nchunks; ++i) {
        const int s = i & 1, c = nchunks - 1 - i;
        if (i >= 2) {
          if (!pipe_wait(&S.empty[s], ((i - 2) >> 1) & 1, ab, err, 1)) break;
          store_dk(i - 2);
        }
        if (*ab) break;
        mbar_arrive_expect_tx(&S.full[s], 6 * 8192);
        const int row = (int)(sq.bos + (int64_t)c * B_BT);
        uint8_t* st = sm + s * B_STAGE;
        tma_load_3d(st, &tmg, &S.full[s], 0, h, row);
        tma_load_3d(st + B_QDPANEL, &tmg, &S.full[s], 64, h, row);
        tma_load_3d(st + 8192, &tmq, &S.full[s], 0, h, row);
        tma_load_3d(st + B_QDPANEL + 8192, &tmq, &S.full[s], 64, h, row);
        tma_load_3d(st + B_OFF_K, &tmk, &S.full[s], 0, h, row);
        tma_load_3d(st + B_OFF_K + B_KPANEL, &tmk, &S.full[s], 64, h, row);
        ++issued;
      }
      for (int i = (issued > 2 ? issued - 2 : 0); i < issued; ++i) mbar_wait(&S.full[i & 1], (i >> 1) & 1);
      if (issued == nchunks) {  // the last one or two chunks: write their dk once released
        for (int i = (nchunks > 2 ? nchunks - 2 : 0); i < nchunks; ++i)
          if (pipe_wait(&S.empty[i & 1], (i >> 1) & 1, ab, err, 1)) store_dk(i);
      }
      bulk_wait_all();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_b1 = idesc_f16(128, 64, AB16, 0, 0);
      const uint32_t id_b5 = idesc_f16(128, 128, AB16, 1, 1, 1);
      const uint32_t id_b2 = idesc_f16(128, 128, AB16, 0, 1);
      const uint32_t id_b3mm = idesc_f16(128, 64, AB16, 1, 1);
      const uint32_t id_b3kk = idesc_f16(128, 64, AB16, 0, 0);
      const uint32_t id_b3mk = idesc_f16(128, 64, AB16, 1, 0);
      const uint32_t id_b4 = idesc_f16(128, 128, AB16, 1, 1);
      const uint32_t id_cw = idesc_f16(128, 16, AB16, 1, 0);
      const uint32_t sC = sbase + B_OFF_C, sG = sbase + B_OFF_G, sAP = sbase + B_OFF_AP, sP4 = sbase + B_OFF_P4,
                     sR = sbase + B_OFF_R;
      auto cw = [&](int i) {  // carry / dW accumulation of iteration i
        const uint32_t st = sbase + (i & 1) * B_STAGE, rb = sR + (i & 1) * 2048;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma(tbase + T_CW, sdesc(st + 8192 + ks * 2048, B_QDPANEL, 1024), sdesc(rb + ks * 32, 16, 1024), id_cw, 1);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma(tbase + T_CW + 16, sdesc(st + ks * 2048, B_QDPANEL, 1024), sdesc(rb + ks * 32, 16, 1024), id_cw, 1);
        umma_commit(&S.cw_done);
        umma_commit(&S.empty[i & 1]);
      };
      bool ok = pipe_wait(&S.tinit, 0, ab, err, 2);
      for (int i = 0; i < nchunks && ok; ++i) {
        const int s = i & 1;
        const uint32_t st = sbase + s * B_STAGE, sK = st + B_OFF_K;
        // Every epilogue warp arrives on its barriers in program order (G read, E1 operands stored,
        // C read, C_prev stored = cconv; ZQ read, dpre stored, dk^T and carry read = dk_read), and a
        // commit covers every earlier MMA of this thread, so one wait stands for all earlier steps.
        if (i >= 1) {
          // dk_read: the previous chunk's dpre is stored and its dk^T (B1 overwrites those columns)
          // and carry (CW updates it) are read
          ok = pipe_wait(&S.dk_read, (i - 1) & 1, ab, err, 2);
          if (!ok) break;
        }
        ok = pipe_wait(&S.kready[s], (i >> 1) & 1, ab, err, 2);
        if (!ok) break;
        tc_fence_after();
        // B1: [D ; A] = [dQc ; Q] K^T
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma(tbase + T_DA, sdesc(st + (ks >> 2) * B_QDPANEL + (ks & 3) * 32, 16, 1024),
               sdesc(sK + (ks >> 2) * B_KPANEL + (ks & 3) * 32, 16, 1024), id_b1, ks > 0);
        umma_commit(&S.da_full);
        // B5: C -= K^T K  (C_prev of this chunk; the epilogue read C before the cconv waited on last chunk)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma(tbase + T_C, sdesc(sK + ks * 2048, B_KPANEL, 1024), sdesc(sK + ks * 2048, B_KPANEL, 1024), id_b5, 1);
        umma_commit(&S.c_full);
        if (i >= 1) cw(i - 1);  // carry / dW of the previous chunk (its own R buffer)
        // cconv: bf16 G, [tril(A) ; P2], P4, dZ and bf16 C_prev are in shared memory, and ZQ and G are read
        ok = pipe_wait(&S.cconv, i & 1, ab, err, 2);
        if (!ok) break;
        tc_fence_after();
        // B2 / B2b: [z ; dq] = [Q ; dZ] C_prev + [tril(A) ; P2] K
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma(tbase + T_ZQ, sdesc(st + (ks >> 2) * B_QDPANEL + 8192 + (ks & 3) * 32, 16, 1024),
               sdesc(sC + ks * 2048, 16384, 1024), id_b2, 1);  // onto the dq_clean / zero start
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma(tbase + T_ZQ, sdesc(sAP + ks * 32, 16, 1024), sdesc(sK + ks * 2048, B_KPANEL, 1024), id_b2, 1);
        umma_commit(&S.zq_full);
        // B3: dk^T = Q^T P2 + dQc^T P4 + G K^T + G^T K^T   (columns shared with [D ; A])
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma(tbase + T_DA, sdesc(st + 8192 + ks * 2048, B_QDPANEL, 1024), sdesc(sAP + 8192 + ks * 2048, 8192, 1024),
               id_b3mm, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma(tbase + T_DA, sdesc(st + ks * 2048, B_QDPANEL, 1024), sdesc(sP4 + ks * 2048, 8192, 1024), id_b3mm, 1);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma(tbase + T_DA, sdesc(sG + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024),
               sdesc(sK + (ks >> 2) * B_KPANEL + (ks & 3) * 32, 16, 1024), id_b3kk, 1);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma(tbase + T_DA, sdesc(sG + ks * 2048, 16384, 1024),
               sdesc(sK + (ks >> 2) * B_KPANEL + (ks & 3) * 32, 16, 1024), id_b3mk, 1);
        umma_commit(&S.dk_full);
        // B4: G += Q^T dZ  (the bf16 copy B3 just read was taken before)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma(tbase + T_G, sdesc(st + 8192 + ks * 2048, B_QDPANEL, 1024),
               sdesc(st + 16384 + ks * 2048, B_QDPANEL, 1024), id_b4, 1);
        umma_commit(&S.g_full);
      }
      if (ok && nchunks > 0) {
        ok = pipe_wait(&S.dk_read, (nchunks - 1) & 1, ab, err, 2);
        if (ok) {
          tc_fence_after();
          cw(nchunks - 1);
        }
      }
      umma_commit(&S.mma_done);
      mbar_wait(&S.mma_done, 0);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------------ aux: zero ragged keys, walk m backwards
    const int at = threadIdx.x - 64;
    const uint32_t p = at >> 5;
    const uint32_t e = (2 * at) & 63;
    const uint32_t ch = e >> 3, cb = (e & 7) * 2;
    float m0v = 0.f, m1v = 0.f;
    if (sub_mean && a.state_mean) {
      m0v = a.state_mean[st_base + 2 * at];
      m1v = a.state_mean[st_base + 2 * at + 1];
    }
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1, c = nchunks - 1 - i;
      const int valid = min(B_BT, sq.len - c * B_BT);
      float rq = 0.f;  // NORM: 1/|q| of token `at` of this chunk, fetched while the loads land
      if (NORM && at < valid) rq = a.norm_aux_in[((sq.bos + (int64_t)c * B_BT + at) * H + h) * 2];
      pipe_wait(&S.full[s], (i >> 1) & 1, ab, err, 4);
      const uint32_t kt = sbase + s * B_STAGE + B_OFF_K;
      if (NORM) {  // Q rows (64 + token) of both panels: q_hat = q * (1/|q|), rounded like the forward
#pragma unroll
        for (int pn = 0; pn < 2; ++pn) {
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            const uint32_t ad = sbase + s * B_STAGE + pn * B_QDPANEL + sw128(64 + at, cc);
            const uint4 v4 = ld_shared_v4(ad);
            uint32_t u[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = unpack2<AB16>(u[j]);
              u[j] = pack2<AB16>(f.x * rq, f.y * rq);
            }
            st_shared_v4(ad, u[0], u[1], u[2], u[3]);
          }
        }
        fence_async_smem();
      }
      if (valid < B_BT) {
        const uint32_t wp = at >> 5, wi = at & 31;
        for (int rr = valid; rr < B_BT; ++rr) st_shared_u32(kt + wp * B_KPANEL + sw128(rr, wi >> 2) + (wi & 3) * 4, 0u);
        fence_async_smem();
      }
      bar_sync<2, 64>();
      if (at == 0) mbar_arrive(&S.kready[s]);
      if (sub_mean) {
        float acc0 = 0.f, acc1 = 0.f;
        const uint32_t kb = kt + p * B_KPANEL + cb;
#pragma unroll 8
        for (int tt = 0; tt < B_BT; ++tt) {
          const float2 f = unpack2<AB16>(ld_shared_u32(kb + sw128(tt, ch)));
          acc0 += f.x;
          acc1 += f.y;
        }
        m0v -= acc0;
        m1v -= acc1;
      }
      if (i >= 2) pipe_wait(&S.m_free[s], ((i - 2) >> 1) & 1, ab, err, 8);
      S.m_buf[s][2 * at] = m0v;
      S.m_buf[s][2 * at + 1] = m1v;
      bar_sync<2, 64>();
      if (at == 0) {
        mbar_arrive(&S.m_ready[s]);
        mbar_arrive(&S.empty[s]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (256 threads)
    const int et = threadIdx.x - 128;
    const int g = et >> 7;
    const int qd = warp & 3;
    const int r = 32 * qd + lane;
    const uint32_t lrow = tbase + ((uint32_t)(32 * qd) << 16);
    const uint32_t sC = sbase + B_OFF_C, sG = sbase + B_OFF_G, sAP = sbase + B_OFF_AP, sP4 = sbase + B_OFF_P4,
                   sR = sbase + B_OFF_R;
    const bool dside = r < 64;                        // lanes 0-63: D / z rows, 64-127: A / dq rows
    const int t = dside ? r : r - 64;
    // relation of this warp's 32 rows t with this half's 32 columns j of [D ; A]
    const bool cols_below = 32 * g + 31 < (t & ~31);
    const bool cols_above = 32 * g > (t | 31);
    float v[64];
    // initial TMEM: C = C_T, G = dC_T, [carry | dW] = [dm_T | 0]
    {
      const float4* src = reinterpret_cast<const float4*>(a.state_cov + (st_base + r) * 128 + 64 * g);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 f = src[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      }
      tmem_st32(lrow + T_C + 64 * g, v);
      tmem_st32(lrow + T_C + 64 * g + 32, v + 32);
      if (a.dfinal_cov) {
        const float4* d4 = reinterpret_cast<const float4*>(a.dfinal_cov + (st_base + r) * 128 + 64 * g);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 f = d4[i];
          v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = 0.f;
      }
      tmem_st32(lrow + T_G + 64 * g, v);
      tmem_st32(lrow + T_G + 64 * g + 32, v + 32);
    }
    if (g == 0) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = 0.f;
      if (a.dfinal_mean) v[0] = a.dfinal_mean[st_base + r];
      tmem_st32(lrow + T_CW, v);
    }
    if (gate && et < 128) S.wh[et] = a.gate_w[(int64_t)h * 128 + et];
    st_shared_v4(sR + 16 * et, 0u, 0u, 0u, 0u);  // R[0], R[1]: rows 3-15 stay zero
    fence_async_smem();
    tmem_st_wait();
    tc_fence_before();
    warp_arrive(&S.tinit);
    float db_acc = 0.f;
    // this token's (lambda, s) from the forward (and NORM: 1/|q|) are loaded one chunk ahead, so the
    // load's latency is hidden behind a whole chunk period instead of sitting before E1; chunks after
    // the first one processed (the document's last, possibly partial chunk) are always full
    float2 ax_nx = make_float2(0.f, 0.f);
    float rqn_nx = 0.f;
    if (nchunks > 0 && t < sq.len - (nchunks - 1) * B_BT) {
      const int64_t tok = sq.bos + (int64_t)(nchunks - 1) * B_BT + t;
      ax_nx = *reinterpret_cast<const float2*>(a.token_aux_in + (tok * H + h) * 2);
      if (NORM && !dside) rqn_nx = a.norm_aux_in[(tok * H + h) * 2];
    }

    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1, c = nchunks - 1 - i;
      const int t0 = c * B_BT;
      const int valid = min(B_BT, sq.len - t0);
      const uint32_t st = sbase + s * B_STAGE;
      const uint32_t rb = sR + s * 2048;              // this chunk's R buffer
      const bool tv = t < valid;
      const float2 ax = ax_nx;
      const float rqn = rqn_nx;
      if (i + 1 < nchunks) {
        const int64_t tok = sq.bos + (int64_t)(t0 - B_BT) + t;
        ax_nx = *reinterpret_cast<const float2*>(a.token_aux_in + (tok * H + h) * 2);
        if (NORM && !dside) rqn_nx = a.norm_aux_in[(tok * H + h) * 2];
      }
      pipe_wait(&S.m_ready[s], (i >> 1) & 1, ab, err, 32);  // long done; checked while B4 still runs
      const float lamv = ax.x, sv = sub_mean ? ax.y : 0.f;
      const float ipos = 1.f / position_of(t0 + t, a.position_offset);
      const float alpha = lamv * ipos;
      const float* mp = S.m_buf[s];

      // ---------------- E1a: the part of E1 that does not need this chunk's scores, done while B1 runs:
      // m_prev . dqc_t (z rows), dZ = -alpha dqc into the stage and the start values of ZQ (zero for
      // the z rows, dq_clean for the dq rows; E2 of the previous chunk has read ZQ)
      pipe_wait(&S.full[s], (i >> 1) & 1, ab, err, 32);  // this chunk's dQc / Q tiles
      float wq_t = 0.f;
      if (dside) {
        if (sub_mean) {
          const float4* mp4 = reinterpret_cast<const float4*>(mp + 64 * g);
          float wq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            float f[8];
            ld_row8<AB16>(st + g * B_QDPANEL, t, cc, f);
            const float4 ma = mp4[2 * cc], mb = mp4[2 * cc + 1];
            wq[0] = fmaf(ma.x, f[0], fmaf(mb.x, f[4], wq[0]));
            wq[1] = fmaf(ma.y, f[1], fmaf(mb.y, f[5], wq[1]));
            wq[2] = fmaf(ma.z, f[2], fmaf(mb.z, f[6], wq[2]));
            wq[3] = fmaf(ma.w, f[3], fmaf(mb.w, f[7], wq[3]));
          }
          wq_t = (wq[0] + wq[1]) + (wq[2] + wq[3]);
        }
#pragma unroll
        for (int cc = 0; cc < 64; ++cc) v[cc] = 0.f;
      } else {
        // dZ = -alpha dqc, packed.  These rows held the previous chunk's dq tile of this warp, staged
        // for its bulk store: wait until that store has read them.
        const float na = tv ? -alpha : 0.f;
        if (lane == 0) bulk_wait_read();
        __syncwarp();
        const uint32_t na2 = pack2<AB16>(na, na);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const uint4 d = ld_shared_v4(st + g * B_QDPANEL + sw128(t, cc));
          st_shared_v4(st + g * B_QDPANEL + 16384 + sw128(t, cc), mul2<AB16>(d.x, na2), mul2<AB16>(d.y, na2),
                       mul2<AB16>(d.z, na2), mul2<AB16>(d.w, na2));
          unpack8<AB16>(d, v + 8 * cc);
        }
      }
      // B2 accumulates onto ZQ: its dq rows start from dq_clean (fp32), its z rows from zero
      tmem_st32(lrow + T_ZQ + 64 * g, v);
      tmem_st32(lrow + T_ZQ + 64 * g + 32, v + 32);
      tmem_st_wait();

      // ---------------- G (after this chunk) -> bf16 operand of B3
      if (i >= 1) pipe_wait(&S.g_full, (i - 1) & 1, ab, err, 16);
      tc_fence_after();
      tmem_ld64(lrow + T_G + 64 * g, v);
      store_panel_row<AB16>(sG + g * 16384, r, v);
      fence_async_smem();
      tc_fence_before();

      // ---------------- E1b: P2, tril(A), P4, R columns (needs [D ; A] of B1)
      pipe_wait(&S.da_full, i & 1, ab, err, 32);
      if (NORM && i >= 1) pipe_wait(&S.ap_free, (i - 1) & 1, ab, err, 32);  // E3 of the last chunk read it
      tc_fence_after();
      tmem_ld32(lrow + T_DA + 32 * g, v);
      if (dside) {
        float wp = wq_t;
        if (!cols_above) {
          float tr[8];
#pragma unroll
          for (int k8 = 0; k8 < 8; ++k8) {
            float x = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int jj = 8 * u + k8;
              x += (cols_below || 32 * g + jj <= t) ? v[jj] : 0.f;
            }
            tr[k8] = x;
          }
          wp += ((tr[0] + tr[1]) + (tr[2] + tr[3])) + ((tr[4] + tr[5]) + (tr[6] + tr[7]));
        }
        S.wpart[g][t] = wp;
        bar_sync_quad<3, 64>(qd);
        const float w = S.wpart[0][t] + S.wpart[1][t];
        const float ds = (sub_mean && tv) ? lamv * w * ipos * ipos : 0.f;
        const float na = tv ? -alpha : 0.f;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t p2[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int jj = 8 * q4 + 2 * e2, j = 32 * g + jj;
            const float p0 = (j <= t) ? fmaf(na, v[jj], ds) : 0.f;
            const float p1 = (j + 1 <= t) ? fmaf(na, v[jj + 1], ds) : 0.f;
            p2[e2] = pack2<AB16>(p0, p1);
          }
          st_shared_v4(sAP + 8192 + sw128(t, 4 * g + q4), p2[0], p2[1], p2[2], p2[3]);
        }
        if (g == 0) {
          S.w[t] = w;
          S.ds[t] = ds;
          st_shared_u16(rb + sw128(0, t >> 3) + (t & 7) * 2, to16<AB16>(ds));
        }
      } else {
        const float beta = (sub_mean && tv) ? lamv * sv * ipos * ipos : 0.f;
        const float na = tv ? -alpha : 0.f;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t am[4], p4[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int jj = 8 * q4 + 2 * e2, j = 32 * g + jj;
            am[e2] = pack2<AB16>(j <= t ? v[jj] : 0.f, j + 1 <= t ? v[jj + 1] : 0.f);
            p4[e2] = pack2<AB16>(j <= t ? fmaf(na, v[jj], beta) : 0.f, j + 1 <= t ? fmaf(na, v[jj + 1], beta) : 0.f);
          }
          st_shared_v4(sAP + sw128(t, 4 * g + q4), am[0], am[1], am[2], am[3]);
          st_shared_v4(sP4 + sw128(t, 4 * g + q4), p4[0], p4[1], p4[2], p4[3]);
        }
        if (g == 0) st_shared_u16(rb + sw128(2, t >> 3) + (t & 7) * 2, to16<AB16>(beta));
      }
      fence_async_smem();

      // ---------------- C_prev -> bf16 operand of B2
      pipe_wait(&S.c_full, i & 1, ab, err, 64);
      tc_fence_after();
      tmem_ld64(lrow + T_C + 64 * g, v);
      tc_fence_before();
      // B2 of the previous chunk has read sC: its zq_full was waited on
      store_panel_row<AB16>(sC + g * 16384, r, v);
      fence_async_smem();
      warp_arrive(&S.cconv);

      // ---------------- E2: dlambda (z rows) and dq (dq rows)
      pipe_wait(&S.zq_full, i & 1, ab, err, 128);
      tc_fence_after();
      tmem_ld64(lrow + T_ZQ + 64 * g, v);
      tc_fence_before();
      if (dside) {
        float uq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float f[8];
          ld_row8<AB16>(st + g * B_QDPANEL, t, cc, f);
#pragma unroll
          for (int e2 = 0; e2 < 8; ++e2) uq[e2 & 3] = fmaf(f[e2], v[8 * cc + e2], uq[e2 & 3]);
        }
        const float up = (uq[0] + uq[1]) + (uq[2] + uq[3]);
        S.upart[g][t] = up;
        bar_sync_quad<3, 64>(qd);
        if (g == 0) {
          const float u = S.upart[0][t] + S.upart[1][t];
          float dl = -u * ipos;
          if (sub_mean) dl += sv * S.w[t] * ipos * ipos;
          float dp = 0.f;
          if (gate) dp = tv ? dl * lamv * (1.f - lamv) : 0.f;
          else if (tv && a.dlam) a.dlam[(sq.bos + t0 + t) * H + h] = dl;
          S.dpre[t] = dp;
          st_shared_u16(rb + sw128(1, t >> 3) + (t & 7) * 2, to16<AB16>(dp));
          db_acc += dp;
        }
      }
      if (!dside) {  // dq_t = [dqc_t + dq inter]_t (from ZQ) + ds_t m_prev, before dpre is known
        const float ds = S.ds[t];
        const float4* mp4 = reinterpret_cast<const float4*>(mp + 64 * g);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const float4 ma = mp4[2 * cc], mb = mp4[2 * cc + 1];
          const float mv[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) v[8 * cc + e] = fmaf(ds, mv[e], v[8 * cc + e]);
        }
      }
      if (gate) {  // dpre of these tokens is in S.dpre (z rows t and dq rows t: quadrants qd and qd ^ 2)
        if (qd & 1) bar_sync<8, 128>();
        else bar_sync<7, 128>();
      }
      if (NORM && !dside) {
        // dq_hat = v + dpre_t W_h, then dq = (dq_hat - q_hat (q_hat . dq_hat)) / |q|; the dot product
        // over both column halves meets through shared memory (the two warps of this lane quadrant)
        const float dp = gate ? S.dpre[t] : 0.f;
        if (gate) {
          const float4* wh4 = reinterpret_cast<const float4*>(S.wh + 64 * g);
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            const float4 wa = wh4[2 * cc], wb = wh4[2 * cc + 1];
            const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) v[8 * cc + e] = fmaf(dp, wv[e], v[8 * cc + e]);
          }
        }
        float qd4[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t qrow = st + g * B_QDPANEL + 8192;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float f[8];
          ld_row8<AB16>(qrow, t, cc, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) qd4[e & 3] = fmaf(f[e], v[8 * cc + e], qd4[e & 3]);
        }
        S.qdot[g][t] = (qd4[0] + qd4[1]) + (qd4[2] + qd4[3]);
        bar_sync_quad<3, 64>(qd);  // ids 5 / 6: the dq-side quadrants 2 and 3
        const float dot = S.qdot[0][t] + S.qdot[1][t];
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float f[8];
          ld_row8<AB16>(qrow, t, cc, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[8 * cc + e] = rqn * fmaf(-f[e], dot, v[8 * cc + e]);
        }
        const uint32_t stg = sbase + (s ^ 1) * B_STAGE + g * B_QDPANEL + 16384;
        uint4* orow = reinterpret_cast<uint4*>((uint8_t*)a.dq + (((sq.bos + t0 + t) * H + h) * 128 + 64 * g) * 2);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t o[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) o[e2] = pack2<AB16>(v[8 * cc + 2 * e2], v[8 * cc + 2 * e2 + 1]);
          if (valid == B_BT) st_shared_v4(stg + sw128(t, cc), o[0], o[1], o[2], o[3]);
          else if (tv) orow[cc] = make_uint4(o[0], o[1], o[2], o[3]);
        }
        if (valid == B_BT) {
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int tw = 32 * (qd - 2);
            tma_store_3d(&tmdq, sm + (s ^ 1) * B_STAGE + g * B_QDPANEL + 16384 + tw * 128, 64 * g, h,
                         (int)(sq.bos + (int64_t)t0 + tw));
            bulk_commit();
          }
        }
      } else if (!dside) {  // + dpre_t W_h, then out
        const float dp = gate ? S.dpre[t] : 0.f;
        // A full chunk's dq is staged in the other stage's dZ rows (B4 of the previous chunk has read
        // them; the next chunk's E1, run by this same warp, rewrites them) and each warp writes its
        // 32 x 64 block with one bulk store.
        const uint32_t stg = sbase + (s ^ 1) * B_STAGE + g * B_QDPANEL + 16384;
        uint4* orow = reinterpret_cast<uint4*>((uint8_t*)a.dq + (((sq.bos + t0 + t) * H + h) * 128 + 64 * g) * 2);
        const float4* wh4 = reinterpret_cast<const float4*>(S.wh + 64 * g);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float wv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (gate) {
            const float4 wa = wh4[2 * cc], wb = wh4[2 * cc + 1];
            wv[0] = wa.x; wv[1] = wa.y; wv[2] = wa.z; wv[3] = wa.w;
            wv[4] = wb.x; wv[5] = wb.y; wv[6] = wb.z; wv[7] = wb.w;
          }
          uint32_t o[4];
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const int jj = 8 * cc + 2 * e2;
            o[e2] = pack2<AB16>(fmaf(dp, wv[2 * e2], v[jj]), fmaf(dp, wv[2 * e2 + 1], v[jj + 1]));
          }
          if (valid == B_BT) st_shared_v4(stg + sw128(t, cc), o[0], o[1], o[2], o[3]);
          else if (tv) orow[cc] = make_uint4(o[0], o[1], o[2], o[3]);
        }
        if (valid == B_BT) {
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int tw = 32 * (qd - 2);  // this warp's first token of the chunk
            tma_store_3d(&tmdq, sm + (s ^ 1) * B_STAGE + g * B_QDPANEL + 16384 + tw * 128, 64 * g, h,
                         (int)(sq.bos + (int64_t)t0 + tw));
            bulk_commit();
          }
        }
      }
      fence_async_smem();  // dpre in R is read by the CW MMAs
      warp_arrive(&S.m_free[s]);

      // ---------------- E3: dk = dk^T + carry, staged through the K tile
      pipe_wait(&S.dk_full, i & 1, ab, err, 256);
      tc_fence_after();
      tmem_ld_frag(lrow + T_DA + 32 * g, v);                  // dims 32qd + 0..15
      tmem_ld_frag(lrow + (16u << 16) + T_DA + 32 * g, v + 16);  // dims 32qd + 16..31
      const float carry = tmem_carry(lrow + T_CW);            // of dim 32qd + lane
      tc_fence_before();
      warp_arrive(&S.dk_read);
      // NORM: dk on the normalised keys is staged in [tril(A) ; P2] (free from dk_full until the next
      // chunk's E1) and mapped into the K tile below, which still holds this chunk's normalised keys
      const uint32_t dkst = NORM ? sAP : st + B_OFF_K;
      {  // dk rows (tokens) written as 8 x 8 blocks transposed out of the fragment layout
        const int mi = lane >> 3, ri = lane & 7;  // this thread addresses row ri of matrix mi
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const float* f = v + 16 * b;
          const float cu = __shfl_sync(0xffffffffu, carry, 16 * b + (lane >> 2));
          const float cl = __shfl_sync(0xffffffffu, carry, 16 * b + 8 + (lane >> 2));
          const int dd = 32 * qd + 16 * b + 8 * (mi & 1);   // first dim of matrix mi
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int k0 = 2 * h2, kk = k0 + (mi >> 1);      // matrices: (k0, dims +0), (k0, +8), (k0+1, +0), (k0+1, +8)
            const uint32_t addr = dkst + (dd >> 6) * B_KPANEL + sw128(32 * g + 8 * kk + ri, (dd & 63) >> 3);
            stmatrix_x4_trans(addr, pack2<AB16>(f[4 * k0] + cu, f[4 * k0 + 1] + cu),
                              pack2<AB16>(f[4 * k0 + 2] + cl, f[4 * k0 + 3] + cl),
                              pack2<AB16>(f[4 * k0 + 4] + cu, f[4 * k0 + 5] + cu),
                              pack2<AB16>(f[4 * k0 + 6] + cl, f[4 * k0 + 7] + cl));
          }
        }
      }
      if (NORM) {
        // the gradient on the normalised keys mapped back through the normalisation (fla's l2norm
        // backward, fla/modules/l2norm.py:49-72): dk = (s - k_hat (k_hat . s)) / |k| with
        // s = dk_hat + the backbone's gradient on k_hat, rounded to 16 bits as autograd's sum of the
        // two would be.  Four threads per token row, 32 dims (64 bytes) each; the result replaces
        // k_hat in the K tile, which the TMA thread stores as dk.
        const int row = et >> 2, qq = et & 3, pn = qq >> 1, c0 = 4 * (qq & 1);
        const bool rv = row < valid;
        const int64_t tok = sq.bos + (int64_t)t0 + row;
        uint4 ev[4] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u),
                       make_uint4(0u, 0u, 0u, 0u)};
        if (rv && a.dk_ext) {
          const uint4* ep = reinterpret_cast<const uint4*>((const uint8_t*)a.dk_ext + ((tok * H + h) * 128 + 32 * qq) * 2);
#pragma unroll
          for (int c = 0; c < 4; ++c) ev[c] = ep[c];
        }
        const float rk = rv ? a.norm_aux_in[(tok * H + h) * 2 + 1] : 0.f;
        if (g == 0) bar_sync<9, 128>();  // the four warps of this token half have staged their blocks
        else bar_sync<10, 128>();
        uint4 dv[4], kv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          dv[c] = ld_shared_v4(sAP + pn * B_KPANEL + sw128(row, c0 + c));
          kv[c] = ld_shared_v4(st + B_OFF_K + pn * B_KPANEL + sw128(row, c0 + c));
        }
        warp_arrive(&S.ap_free);  // [tril(A) ; P2] is read: the next chunk's E1b may overwrite it
        uint32_t sp[16];
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t dw[4] = {dv[c].x, dv[c].y, dv[c].z, dv[c].w};
          const uint32_t ew[4] = {ev[c].x, ev[c].y, ev[c].z, ev[c].w};
          const uint32_t kw[4] = {kv[c].x, kv[c].y, kv[c].z, kv[c].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 d2 = unpack2<AB16>(dw[j]), e2 = unpack2<AB16>(ew[j]), k2 = unpack2<AB16>(kw[j]);
            sp[4 * c + j] = pack2<AB16>(d2.x + e2.x, d2.y + e2.y);
            const float2 s2 = unpack2<AB16>(sp[4 * c + j]);
            dot = fmaf(s2.x, k2.x, dot);
            dot = fmaf(s2.y, k2.y, dot);
          }
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t kw[4] = {kv[c].x, kv[c].y, kv[c].z, kv[c].w};
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 s2 = unpack2<AB16>(sp[4 * c + j]), k2 = unpack2<AB16>(kw[j]);
            o[j] = pack2<AB16>(rk * (s2.x - k2.x * dot), rk * (s2.y - k2.y * dot));
          }
          st_shared_v4(st + B_OFF_K + pn * B_KPANEL + sw128(row, c0 + c), o[0], o[1], o[2], o[3]);
        }
      }
      if (valid < B_BT) {  // a document's last, partial chunk: plain stores of its valid rows
        bar_sync<1, 256>();
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int qid = et + 256 * k4;             // 16-byte chunk id: row (64) x panel (2) x chunk (8)
          const int row = qid >> 4, pn = (qid >> 3) & 1, cc = qid & 7;
          if (row < valid) {
            const uint4 val = ld_shared_v4(st + B_OFF_K + pn * B_KPANEL + sw128(row, cc));
            *reinterpret_cast<uint4*>((uint8_t*)a.dk + (((sq.bos + t0 + row) * H + h) * 128 + 64 * pn + 8 * cc) * 2) = val;
          }
        }
      }
      fence_async_smem();  // the staged dk is read by the TMA thread's bulk store
      warp_arrive(&S.empty[s]);
    }
    if (!dside && lane == 0) bulk_wait_all();  // this warp's dq bulk stores
    // ---------------- per-document outputs
    if (nchunks > 0) {
      pipe_wait(&S.g_full, (nchunks - 1) & 1, ab, err, 512);
      pipe_wait(&S.cw_done, (nchunks - 1) & 1, ab, err, 512);
    }
    tc_fence_after();
    if (a.dinitial_cov) {
      tmem_ld64(lrow + T_G + 64 * g, v);
      float4* dst = reinterpret_cast<float4*>(a.dinitial_cov + (st_base + r) * 128 + 64 * g);
#pragma unroll
      for (int k4 = 0; k4 < 16; ++k4) dst[k4] = make_float4(v[4 * k4], v[4 * k4 + 1], v[4 * k4 + 2], v[4 * k4 + 3]);
    }
    {
      float cwv[2];
      tmem_ld2f(lrow + T_CW, cwv);
      const float carry = tmem_carry(lrow + T_CW);
      if (g == 0 && a.dinitial_mean) a.dinitial_mean[st_base + r] = carry;
      if (g == 0 && gate) gate_part[((int64_t)n * H + h) * 129 + r] = cwv[1];
    }
    if (gate) {
      db_acc = warp_sum(db_acc);
      if (lane == 0 && db_acc != 0.f) atomicAdd(&S.db, db_acc);
      bar_sync<1, 256>();
      if (et == 0) gate_part[((int64_t)n * H + h) * 129 + 128] = S.db;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// gate partials: 128 dW entries and db per (document, head)
size_t part_bytes(int H, int n_seqs) { return ws_align(sizeof(float) * (size_t)n_seqs * H * 129); }

// dW[h] = sum over documents of the per-CTA partials, db[h] likewise
__global__ void gate_sum_kernel(const float* part, int n_seqs, int H, float* dW, float* db) {
  const int h = blockIdx.x;
  for (int d = threadIdx.x; d <= 128; d += blockDim.x) {
    float s = 0.f;
    for (int n = 0; n < n_seqs; ++n) s += part[((int64_t)n * H + h) * 129 + d];
    if (d < 128) dW[(int64_t)h * 128 + d] = s;
    else db[h] = s;
  }
}

template <int AB16, int NORM>
cudaError_t launch(const CleanArgs& a, int* launches) {
  CUtensorMap tq, tk, tg, tdq, tdk;
  const int64_t rows = (int64_t)a.B * a.T;
  cudaError_t e = tc::make_token_map(&tq, a.q, rows, a.H, 128, B_BT, AB16 != 0);
  if (e != cudaSuccess) return e;
  if ((e = tc::make_token_map(&tk, a.k, rows, a.H, 128, B_BT, AB16 != 0)) != cudaSuccess) return e;
  if ((e = tc::make_token_map(&tg, a.dq_clean, rows, a.H, 128, B_BT, AB16 != 0)) != cudaSuccess) return e;
  if ((e = tc::make_token_map(&tdk, a.dk, rows, a.H, 128, B_BT, AB16 != 0)) != cudaSuccess) return e;
  if ((e = tc::make_token_map(&tdq, a.dq, rows, a.H, 128, 32, AB16 != 0)) != cudaSuccess) return e;  // per-warp blocks
  int* err = reinterpret_cast<int*>(a.workspace);
  float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.workspace) + 256);
  if ((e = cudaMemsetAsync(err, 0, sizeof(int), a.stream)) != cudaSuccess) return e;
  CleanArgs la = a;
  la.doc_order = nullptr;
  if (lpt_order_bytes(a.n_seqs, a.cu_seqlens != nullptr) > 0) {
    int* order = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(a.workspace) + 256 + part_bytes(a.H, a.n_seqs));
    if ((e = lpt_order(a, order, launches)) != cudaSuccess) return e;
    la.doc_order = order;
  }
  auto kern = tc_bwd_kernel<AB16, NORM>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)B_SMEM)) != cudaSuccess)
    return e;
  kern<<<a.n_seqs * a.H, B_THREADS, B_SMEM, a.stream>>>(tq, tk, tg, tdq, tdk, la, err, part);
  *launches += 1;
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (a.lambda_mode == LAMBDA_GATE) {
    gate_sum_kernel<<<a.H, 128, 0, a.stream>>>(part, a.n_seqs, a.H, a.dgate_w, a.dgate_b);
    *launches += 1;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

// error word (256 bytes), the per-(document, head) gate partials, then the varlen launch order
size_t tc_bwd_workspace(int B, int, int H, int, int n_seqs) {
  return 256 + part_bytes(H, n_seqs) + lpt_order_bytes(n_seqs, B == 1 && n_seqs >= 2);
}

cudaError_t tc_bwd(const CleanArgs& a, int* launches) {
  if (a.qk_norm) return a.dtype == DT_BF16 ? launch<1, 1>(a, launches) : launch<0, 1>(a, launches);
  return a.dtype == DT_BF16 ? launch<1, 0>(a, launches) : launch<0, 0>(a, launches);
}

}  // namespace ccq
