// Tensor-core (tcgen05 / TMEM / TMA) forward of the CCQ cleaning operator, bf16 or fp16, K = 128.
//
// One CTA per (document, head) walks the document in chunks of BT = 128 tokens.  The covariance
// state C (128 x 128 fp32) lives in TMEM for the whole document and is never written to HBM, so
// the kernel reads q and k once and writes q_clean once.  Per chunk (Q, K = 128 x 128 tiles; the K
// tile carries four extra rows m_hi, m_lo, w_hi, w_lo after its 128 keys, then zero rows to 144):
//   F1  A  = Q [K ; m_hi ; m_lo ; w_hi ; w_lo]^T        (N = 144: q k_j^T, q.m_prev, q.w for the gate)
//   F3  C += K^T K                                      (the state update, fp32 accumulate in TMEM)
//   F2a Z  = Q bf16(C_prev)
//   F2b Z += [P' | -sp -sp] [K ; m_hi ; m_lo]           (K-dim 144: the rank-1 mean term rides along)
// with P'[t][j] = (A[t][j] - sp_t)[j <= t], sp_t = s_t / pos_t, s_t = q_t . m_t, so that
//   Z_t = z_t - sp_t m_t   and   q_clean_t = q_t - (lambda_t / pos_t) Z_t,
// the reference's q_t - lambda_t (z_t / pos_t - s_t m_t / pos_t^2) (ccq/ops/common/fused_read.py:11-16,
// kernel at :86-174).  TMEM holds C (128 columns), two 144-column regions and P' (72 columns of
// packed 16-bit values, the A operand of F2b); chunk i uses region i % 2 first for its scores A_i
// and then, once they are read, for Z_i, so the scores of chunk i+1 and the output of chunk i are in
// flight together.  q_clean is staged in shared memory and written by TMA bulk stores; the output
// group reads q for it again (a TMA load that hits L2) into the staging tile, so an input stage is
// released as soon as the chunk's last MMA has read it, and the TMA thread also prefetches the next
// chunk of a stage into L2 while the stage is still busy.
//
// Warp roles (640 threads):
//   warp 0      TMA loads of the Q / K tiles (two stages);
//   warp 1      TMEM allocation and every MMA, from one thread that issues whichever of the four MMA
//               groups has its inputs ready (the groups of neighbouring chunks overlap);
//   warps 2-3   running key sum m: the m rows of the K tile and the fp32 m_prev of each chunk;
//   warps 4-11  "score" group: A -> P' (two warps per TMEM lane quadrant, 64 columns each), lambda;
//   warps 12-19 "output" group: C -> bf16 operand of the next chunk, Z -> q_clean (one thread issues
//               the bulk store of each full chunk; a document's last, partial chunk is written with
//               plain stores so no row of the next document is touched).
// Every mbarrier wait is bounded; on a timeout the CTA records an error in the workspace and unwinds.
//
// NORM = 1 (the *_l2norm entry points) takes raw q and k and applies fla's l2norm (y = x / sqrt(|x|^2
// + 1e-6), fp32 math, rounded to the activation dtype; fla/modules/l2norm.py:26-46) inside the
// kernel.  K: the aux warps normalise each chunk's K tile in place in shared memory before the first
// MMA reads it (the state update and the masked read need the normalised keys as MMA operands), write
// it out as k_norm with one TMA bulk store (the backbone reads it next) and record 1/|k|.  Q is never
// rewritten: with r_t = 1/|q_t| every quantity the kernel forms from q scales by r_t, so the MMAs run
// on the raw Q tile and r_t is applied where it matters: the scores A_t, the mean-term scalar s_t and
// the per-token P' row enter the masked read in raw units (P'' = A_raw - s_raw / pos, whose product
// with r_t is P'), so Z accumulates Z_true / r_t; the gate logit and the token_aux side output take
// r_t explicitly, and the output group forms q_clean = q_hat - (lambda / pos) r_t Z with q_hat the
// re-read q rounded after scaling by r_t, as l2norm's output is.  The score group computes r_t from
// the Q tile (each thread reads its token's full row).
#include <stdlib.h>

#include "args.h"
#include "common.cuh"
#include "tc_common.cuh"
#include "tma_host.h"

namespace ccq {

namespace {
using namespace tc;

constexpr int F_THREADS = 640;
constexpr int F_BT = 128;
constexpr uint32_t F_QPANEL = 16384;                  // 128 rows x 128 B
constexpr uint32_t F_QTILE = 2 * F_QPANEL;            // 128 x 128 bf16
constexpr uint32_t F_KROWS = 144;                     // 128 keys + m_hi, m_lo, w_hi, w_lo, zeros
constexpr uint32_t F_KPANEL = F_KROWS * 128;          // 18432
constexpr uint32_t F_KTILE = 2 * F_KPANEL;
constexpr uint32_t F_OFF_Q = 0;                       // two stages
constexpr uint32_t F_OFF_K = 2 * F_QTILE;             // two stages
constexpr uint32_t F_OFF_C = F_OFF_K + 2 * F_KTILE;   // bf16 C_prev (MN-major B operand)
constexpr uint32_t F_OFF_O = F_OFF_C + F_QTILE;       // q_clean staging (same layout as a Q tile)
constexpr uint32_t F_OFF_SMALL = F_OFF_O + F_QTILE;
constexpr uint32_t T_C = 0, T_R = 128, T_RSTRIDE = 144;  // TMEM columns: C, then regions 0 and 1
constexpr uint32_t T_P = 416;                          // P' (64 + 8 columns of packed pairs)
constexpr int GROUP_WARPS = 8;

struct FwdSmall {
  float xs[2][2][128];     // [chunk parity][column half][row]: partial s_t
  float cf[2][128];        // [chunk parity][row]: lambda_t / pos_t
  float msum[4][128];      // aux: per token-quarter partial key sums
  float rk[2][128];        // NORM: [stage][row] 1/|k| of the stage's chunk
  float rqo[2][128];       // NORM: [chunk parity][row] 1/|q| handed from the score to the output group
  uint64_t full[2], kready[2], empty[2], a_full[2], a_free[2], cf_ready[2], z_full[2], z_free[2];
  uint64_t c_full, c_read, cprev_free, cconv, pready, qo_full, mma_done;
  uint64_t never;          // debug stall: an mbarrier nothing arrives on
  uint32_t tmem_base;
  int abort;
};
constexpr size_t F_SMEM = F_OFF_SMALL + sizeof(FwdSmall) + 1024;
static_assert(F_SMEM <= 232448, "forward kernel shared memory");

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

template <int AB16>
__device__ __forceinline__ float act_load(const void* p, int64_t i) {
  if (AB16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

template <int AB16>
__device__ __forceinline__ uint32_t split_hi(float x, float* rest) {
  if (AB16) {
    __nv_bfloat16 h = __float2bfloat16_rn(x);
    *rest = x - __bfloat162float(h);
    return (uint32_t)__bfloat16_as_ushort(h);
  } else {
    __half h = __float2half_rn(x);
    *rest = x - __half2float(h);
    return (uint32_t)__half_as_ushort(h);
  }
}
template <int AB16>
__device__ __forceinline__ uint32_t to16(float x) {
  if (AB16) return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(x));
  return (uint32_t)__half_as_ushort(__float2half_rn(x));
}

// 4 consecutive fp32 TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
  uint32_t r0, r1, r2, r3;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(taddr));
  v[0] = __uint_as_float(r0);
  v[1] = __uint_as_float(r1);
  v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3);
}

// 64 values of one row -> one 64-column panel row (8 swizzled 16-byte chunks)
template <int AB16>
__device__ __forceinline__ void store_row64(uint32_t panel, int row, const float* x) {
#pragma unroll
  for (int cc = 0; cc < 8; ++cc)
    st_shared_v4(panel + sw128(row, cc), pack2<AB16>(x[8 * cc], x[8 * cc + 1]), pack2<AB16>(x[8 * cc + 2], x[8 * cc + 3]),
                 pack2<AB16>(x[8 * cc + 4], x[8 * cc + 5]), pack2<AB16>(x[8 * cc + 6], x[8 * cc + 7]));
}

template <int AB16, int NORM>
__global__ void __launch_bounds__(F_THREADS, 1)
    tc_fwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmo, const __grid_constant__ CUtensorMap tmkn, CleanArgs a,
                  int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FwdSmall& S = *reinterpret_cast<FwdSmall*>(sm + F_OFF_SMALL);
  const uint32_t sbase = smem_u32(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.H;
  const int h = blockIdx.x % H, n = doc_of_slot(blockIdx.x / H, a.doc_order);
  const Seq sq = seq_of(n, a.T, a.cu_seqlens);
  const int nchunks = (sq.len + F_BT - 1) / F_BT;
  const int64_t st_base = ((int64_t)n * H + h) * 128;
  const bool sub_mean = a.subtract_mean != 0;
  const bool gate = a.lambda_mode == LAMBDA_GATE;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.kready[i], 1);
      mbar_init(&S.empty[i], 2);  // F2b commit, aux
      mbar_init(&S.a_full[i], 1);
      mbar_init(&S.a_free[i], GROUP_WARPS);
      mbar_init(&S.cf_ready[i], GROUP_WARPS / 2);
      mbar_init(&S.z_full[i], 1);
      mbar_init(&S.z_free[i], GROUP_WARPS);
    }
    mbar_init(&S.c_full, 1);
    mbar_init(&S.c_read, GROUP_WARPS);
    mbar_init(&S.cprev_free, 1);
    mbar_init(&S.cconv, GROUP_WARPS);
    mbar_init(&S.pready, GROUP_WARPS);
    mbar_init(&S.qo_full, 1);
    mbar_init(&S.never, 1);
    mbar_init(&S.mma_done, 1);
    S.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&S.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = S.tmem_base;
  volatile int* ab = &S.abort;

  if (a.debug_stall_cycles > 0) {
    // Debug knob (CCQ_B200_DEBUG_STALL_CYCLES): one bounded wait on a barrier nothing arrives on, before
    // any copy or MMA is issued, so the timeout path (error word, abort flag, every role unwinding
    // through its named barriers, TMEM freed) runs without a fault or a hang.
    if (threadIdx.x == 0) {
      const long long t0 = clock64();
      while (!mbar_test(&S.never, 0)) {
        if (clock64() - t0 > a.debug_stall_cycles) {
          S.abort = 1;
          atomicOr(err, 0x100);
          break;
        }
        __nanosleep(256);
      }
    }
    __syncthreads();
  }

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int s = c & 1;
        if (c >= 2 && !pipe_wait(&S.empty[s], ((c - 2) >> 1) & 1, ab, err, 1)) break;
        if (*ab) break;
        mbar_arrive_expect_tx(&S.full[s], 2 * F_QTILE);
        const int row = (int)(sq.bos + (int64_t)c * F_BT);
        uint8_t* q_dst = sm + F_OFF_Q + s * F_QTILE;
        uint8_t* k_dst = sm + F_OFF_K + s * F_KTILE;
        tma_load_3d(q_dst, &tmq, &S.full[s], 0, h, row);
        tma_load_3d(q_dst + F_QPANEL, &tmq, &S.full[s], 64, h, row);
        tma_load_3d(k_dst, &tmk, &S.full[s], 0, h, row);
        tma_load_3d(k_dst + F_KPANEL, &tmk, &S.full[s], 64, h, row);
        ++issued;
        // the load of chunk c+2 waits for this stage to be released: warm L2 for it now
        if (c + 2 < nchunks) {
          const int prow = (int)(sq.bos + (int64_t)(c + 2) * F_BT);
          tma_prefetch_3d(&tmq, 0, h, prow);
          tma_prefetch_3d(&tmq, 64, h, prow);
          tma_prefetch_3d(&tmk, 0, h, prow);
          tma_prefetch_3d(&tmk, 64, h, prow);
        }
      }
      // never leave the CTA with bulk copies in flight
      for (int c = (issued > 2 ? issued - 2 : 0); c < issued; ++c) mbar_wait(&S.full[c & 1], (c >> 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // Four MMA groups per chunk i, each issued once its inputs are ready (checked without
    // blocking, so a group of chunk i+1 can go ahead of a group of chunk i that still waits):
    //   F1_i  needs K/Q tiles of i and region i%2 free (Z of i-2 read);
    //   F3_i  needs C of i-1 read out of TMEM;
    //   F2a_i needs bf16 C_prev in shared memory and the scores A_i read (Z_i overwrites them);
    //   F2b_i needs P'_i; F2b_i's commit also releases the K/Q stage, so F1_i, F3_i and F2a_i of the
    //         same chunk are issued before it.
    if (lane == 0) {
      const uint32_t id_a = idesc_f16(128, 144, AB16, 0, 0);
      const uint32_t id_z = idesc_f16(128, 128, AB16, 0, 1);
      const uint32_t id_c = idesc_f16(128, 128, AB16, 1, 1);
      const uint32_t sC = sbase + F_OFF_C;
      int i1 = 0, i3 = 0, i2a = 0, i2b = 0;
      long long idle0 = clock64();
      while (i2b < nchunks) {
        if (*ab) break;
        bool issued = true;
        if (i2b < i2a && i2b < i3 && mbar_test(&S.pready, i2b & 1)) {
          const int c = i2b, s = c & 1;
          const uint32_t sK = sbase + F_OFF_K + s * F_KTILE;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 9; ++ks)
            umma_ts(tbase + T_R + T_RSTRIDE * s, tbase + T_P + 8 * ks, sdesc(sK + ks * 2048, F_KPANEL, 1024), id_z, 1);
          umma_commit(&S.z_full[s]);
          umma_commit(&S.empty[s]);
          ++i2b;
        } else if (i2a < i1 && mbar_test(&S.cconv, i2a & 1) && mbar_test(&S.a_free[i2a & 1], (i2a >> 1) & 1)) {
          const uint32_t sQ = sbase + F_OFF_Q + (i2a & 1) * F_QTILE;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma(tbase + T_R + T_RSTRIDE * (i2a & 1), sdesc(sQ + (ks >> 2) * F_QPANEL + (ks & 3) * 32, 16, 1024),
                 sdesc(sC + ks * 2048, F_QPANEL, 1024), id_z, ks > 0);
          umma_commit(&S.cprev_free);
          ++i2a;
        } else if (i3 < i1 && mbar_test(&S.c_read, i3 & 1)) {
          const uint32_t sK = sbase + F_OFF_K + (i3 & 1) * F_KTILE;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma(tbase + T_C, sdesc(sK + ks * 2048, F_KPANEL, 1024), sdesc(sK + ks * 2048, F_KPANEL, 1024), id_c, 1);
          umma_commit(&S.c_full);
          ++i3;
        } else if (i1 < nchunks && mbar_test(&S.kready[i1 & 1], (i1 >> 1) & 1) &&
                   (i1 < 2 || mbar_test(&S.z_free[i1 & 1], ((i1 - 2) >> 1) & 1))) {
          const int b = i1 & 1;
          const uint32_t sQ = sbase + F_OFF_Q + b * F_QTILE, sK = sbase + F_OFF_K + b * F_KTILE;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma(tbase + T_R + T_RSTRIDE * b, sdesc(sQ + (ks >> 2) * F_QPANEL + (ks & 3) * 32, 16, 1024),
                 sdesc(sK + (ks >> 2) * F_KPANEL + (ks & 3) * 32, 16, 1024), id_a, ks > 0);
          umma_commit(&S.a_full[b]);
          ++i1;
        } else {
          issued = false;
        }
        if (issued) {
          idle0 = clock64();
        } else {
          __nanosleep(32);  // back off: the polling thread shares its scheduler with epilogue warps
        }
        if (!issued && clock64() - idle0 > (1ll << 31)) {
          *ab = 1;
          atomicOr(err, 2);
          // detail word: how far each MMA group got (chunk counts of F1, F2a, F3, F2b)
          atomicExch(err + 1, (min(i1, 255) << 24) | (min(i2a, 255) << 16) | (min(i3, 255) << 8) | min(i2b, 255));
          break;
        }
      }
      // TMEM is freed only after every issued MMA has completed
      umma_commit(&S.mma_done);
      mbar_wait(&S.mma_done, 0);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------------ aux: running key sum
    const int at = threadIdx.x - 64;           // 0..63
    // m rows: this thread writes dims 2at, 2at+1
    const uint32_t p = at >> 5;
    const uint32_t e = (2 * at) & 63;
    const uint32_t ch = e >> 3, cb = (e & 7) * 2;
    // key sums: this thread adds 16-byte chunk cq (dims 8cq..8cq+7) over tokens 32tq..32tq+31
    const int cq = at & 15, tq = at >> 4;
    float m0v = 0.f, m1v = 0.f;
    if (sub_mean && a.initial_mean) {
      m0v = a.initial_mean[st_base + 2 * at];
      m1v = a.initial_mean[st_base + 2 * at + 1];
    }
    uint32_t wh = 0, wl = 0;
    if (gate) {
      float r0, r1;
      const uint32_t h0 = split_hi<AB16>(a.gate_w[(int64_t)h * 128 + 2 * at], &r0);
      const uint32_t h1 = split_hi<AB16>(a.gate_w[(int64_t)h * 128 + 2 * at + 1], &r1);
      wh = h0 | (h1 << 16);
      wl = to16<AB16>(r0) | (to16<AB16>(r1) << 16);
    }
    for (int s = 0; s < 2; ++s) {
      const uint32_t kb = sbase + F_OFF_K + s * F_KTILE + p * F_KPANEL;
      for (uint32_t row = 130; row < F_KROWS; ++row)
        st_shared_u32(kb + sw128(row, ch) + cb, row == 130 ? wh : (row == 131 ? wl : 0u));
    }
    for (int c = 0; c < nchunks; ++c) {
      const int s = c & 1;
      pipe_wait(&S.full[s], (c >> 1) & 1, ab, err, 4);
      const uint32_t kt = sbase + F_OFF_K + s * F_KTILE;
      const int valid = min(F_BT, sq.len - c * F_BT);
      if (NORM) {
        // the chunk's 128 k rows normalised in place: four threads per row (16-byte chunks
        // 4 sub .. 4 sub + 3 of the row's 16), 16 rows per pass, two passes at a time so their
        // shared-memory loads and reductions overlap (two warps have little else to hide latency
        // with; more at a time spills registers).  1/sqrt is the hardware reciprocal square root:
        // the products are rounded to 16 bits, which absorbs its last-bit difference.
        const int sub = at & 3;
        const uint32_t pan = sub >> 1, cc0 = (sub & 1) * 4;
        const uint32_t base = kt + pan * F_KPANEL;
#pragma unroll 1
        for (int grp = 0; grp < 8; ++grp) {
          uint4 w[1][4];
          float ss[1];
#pragma unroll
          for (int r4 = 0; r4 < 1; ++r4) {
            const int row = (grp + r4) * 16 + (at >> 2);
#pragma unroll
            for (int i = 0; i < 4; ++i) w[r4][i] = ld_shared_v4(base + sw128(row, cc0 + i));
          }
#pragma unroll
          for (int r4 = 0; r4 < 1; ++r4) {
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t u[4] = {w[r4][i].x, w[r4][i].y, w[r4][i].z, w[r4][i].w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = unpack2<AB16>(u[j]);
                a0 = fmaf(f.x, f.x, a0);
                a1 = fmaf(f.y, f.y, a1);
              }
            }
            ss[r4] = a0 + a1;
          }
#pragma unroll
          for (int r4 = 0; r4 < 1; ++r4) ss[r4] += __shfl_xor_sync(0xffffffffu, ss[r4], 1);
#pragma unroll
          for (int r4 = 0; r4 < 1; ++r4) ss[r4] += __shfl_xor_sync(0xffffffffu, ss[r4], 2);
#pragma unroll
          for (int r4 = 0; r4 < 1; ++r4) {
            const int row = (grp + r4) * 16 + (at >> 2);
            const float rinv = rsqrtf(ss[r4] + 1e-6f);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t u[4] = {w[r4][i].x, w[r4][i].y, w[r4][i].z, w[r4][i].w};
              uint32_t o[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = unpack2<AB16>(u[j]);
                o[j] = pack2<AB16>(f.x * rinv, f.y * rinv);
              }
              st_shared_v4(base + sw128(row, cc0 + i), o[0], o[1], o[2], o[3]);
            }
            if (sub == 0) S.rk[s][row] = rinv;
          }
        }
        fence_async_smem();  // the normalised K tile -> the MMAs and the bulk store
        bar_sync<2, 64>();
        const int t0 = c * F_BT;
        if (valid == F_BT) {
          if (at == 0) {
            const int row0 = (int)(sq.bos + (int64_t)t0);
            tma_store_3d(&tmkn, sm + F_OFF_K + s * F_KTILE, 0, h, row0);
            tma_store_3d(&tmkn, sm + F_OFF_K + s * F_KTILE + F_KPANEL, 64, h, row0);
            bulk_commit();
          }
        } else {  // a document's last, partial chunk: plain stores of its valid rows only
          for (int i = at; i < valid * 16; i += 64) {
            const int row = i >> 4, pn = (i >> 3) & 1, cc = i & 7;
            const uint4 val = ld_shared_v4(kt + pn * F_KPANEL + sw128(row, cc));
            *reinterpret_cast<uint4*>((uint8_t*)a.k_norm + (((sq.bos + t0 + row) * H + h) * 128 + 64 * pn + 8 * cc) * 2) =
                val;
          }
        }
        for (int t = at; t < valid; t += 64) a.norm_aux[((sq.bos + t0 + t) * H + h) * 2 + 1] = S.rk[s][t];
      }
      if (valid < F_BT) {  // keys past the end of the document belong to the next one: zero them
        const uint32_t wp = at >> 5, wi = at & 31;
        for (int rr = valid; rr < F_BT; ++rr) st_shared_u32(kt + wp * F_KPANEL + sw128(rr, wi >> 2) + (wi & 3) * 4, 0u);
      }
      {  // rows 128 / 129: m_prev split into two 16-bit parts
        float r0, r1;
        const uint32_t h0 = split_hi<AB16>(sub_mean ? m0v : 0.f, &r0);
        const uint32_t h1 = split_hi<AB16>(sub_mean ? m1v : 0.f, &r1);
        const uint32_t kb = kt + p * F_KPANEL;
        st_shared_u32(kb + sw128(128, ch) + cb, h0 | (h1 << 16));
        st_shared_u32(kb + sw128(129, ch) + cb, to16<AB16>(r0) | (to16<AB16>(r1) << 16));
      }
      fence_async_smem();
      bar_sync<2, 64>();
      if (at == 0) mbar_arrive(&S.kready[s]);
      if (sub_mean) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const uint32_t kb = kt + (cq >> 3) * F_KPANEL;
#pragma unroll 4
        for (int tt = 32 * tq; tt < 32 * tq + 32; ++tt) {
          const uint4 v4 = ld_shared_v4(kb + sw128(tt, cq & 7));
          const uint32_t w4[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = unpack2<AB16>(w4[i]);
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) S.msum[tq][8 * cq + i] = acc[i];
        bar_sync<2, 64>();
        m0v += S.msum[0][2 * at] + S.msum[1][2 * at] + S.msum[2][2 * at] + S.msum[3][2 * at];
        m1v += S.msum[0][2 * at + 1] + S.msum[1][2 * at + 1] + S.msum[2][2 * at + 1] + S.msum[3][2 * at + 1];
      }
      bar_sync<2, 64>();
      if (NORM && at == 0) bulk_wait_read();  // the normalised keys' bulk store has read the stage
      if (at == 0) mbar_arrive(&S.empty[s]);
    }
    if (NORM && at == 0) bulk_wait_all();
    if (sub_mean && a.final_mean) {
      a.final_mean[st_base + 2 * at] = m0v;
      a.final_mean[st_base + 2 * at + 1] = m1v;
    }
  } else if (warp < 4 + GROUP_WARPS) {
    // ------------------------------------------------------------------ score group: A -> P'
    const int qd = warp & 3;                      // TMEM lane quadrant of this warp
    const int hp = (warp - 4) >> 2;               // column half: columns 64hp .. 64hp+63
    const int t = 32 * qd + lane;                 // token of this thread
    const uint32_t lrow = tbase + ((uint32_t)(32 * qd) << 16);
    const float gate_b = gate ? a.gate_b[h] : 0.f;
    const bool cols_below = 64 * hp + 63 < 32 * qd;
    const bool cols_above = 64 * hp > 32 * qd + 31;
    float v[64];
    // P' entries above the diagonal block never change: zero them once; so do mean columns 2..15
    {
      const uint32_t z8[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      if (cols_above)
#pragma unroll
        for (int i = 0; i < 4; ++i) tmem_st8(lrow + T_P + 32 * hp + 8 * i, z8);
      if (hp == 0) tmem_st8(lrow + T_P + 64, z8);
      tmem_st_wait();
    }

    for (int c = 0; c < nchunks; ++c) {
      const int pb = c & 1;
      const int t0 = c * F_BT;
      const int valid = min(F_BT, sq.len - t0);
      pipe_wait(&S.a_full[pb], (c >> 1) & 1, ab, err, 16);
      tc_fence_after();
      float rqv = 1.f;
      if (NORM) {
        // 1/|q_t| from row t of the raw Q tile (the stage holds chunk c until F2b, which waits for
        // this group); both column halves, so no exchange between the warps of a lane quadrant
        const uint32_t qrow = sbase + F_OFF_Q + pb * F_QTILE;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int cc = 0; cc < 16; ++cc) {
          const uint4 w4 = ld_shared_v4(qrow + (cc >> 3) * F_QPANEL + sw128(t, cc & 7));
          const uint32_t u[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack2<AB16>(u[j]);
            a0 = fmaf(f.x, f.x, a0);
            a1 = fmaf(f.y, f.y, a1);
          }
        }
        rqv = rsqrtf(a0 + a1 + 1e-6f);
      }
      float ext[4] = {0.f, 0.f, 0.f, 0.f};
      if (!cols_above) tmem_ld64(lrow + T_R + T_RSTRIDE * pb + 64 * hp, v);
      if (hp == 0) tmem_ld4(lrow + T_R + T_RSTRIDE * pb + 128, ext);
      tc_fence_before();
      warp_arrive(&S.a_free[pb]);
      const float ipos = 1.f / position_of(t0 + t, a.position_offset);
      float part = ext[0] + ext[1];
      if (!cols_above) {
        if (!cols_below) {
          // This warp's 32 tokens t lie in one 32-column half of its 64 columns (tl < 32 for the whole
          // warp or for none of it): the other half is all kept or all zero, so 32 columns get a mask.
          const int tl = t - 64 * hp;
          if (tl < 32) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = (jj <= tl) ? v[jj] : 0.f;
#pragma unroll
            for (int jj = 32; jj < 64; ++jj) v[jj] = 0.f;
          } else {
#pragma unroll
            for (int jj = 32; jj < 64; ++jj) v[jj] = (jj <= tl) ? v[jj] : 0.f;
          }
        }
        float tr[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) tr[i] = (v[i] + v[i + 16]) + (v[i + 32] + v[i + 48]);
#pragma unroll
        for (int i = 0; i < 4; ++i) tr[i] = (tr[i] + tr[i + 4]) + (tr[i + 8] + tr[i + 12]);
        part += (tr[0] + tr[1]) + (tr[2] + tr[3]);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(pack2<AB16>(v[2 * i], v[2 * i + 1]));
      }
      // s_t = sum of both column halves.  For tokens 0-63 the second half lies above the diagonal and
      // adds nothing, so quadrants 0-1 need no exchange (and their half-1 warps no s_t at all).
      float st = 0.f;
      if (qd >= 2) {
        S.xs[pb][hp][t] = part;
        if (qd == 2) bar_sync<5, 64>();
        else bar_sync<6, 64>();
        st = S.xs[pb][0][t] + S.xs[pb][1][t];
      } else {
        st = part;
      }
      if (!sub_mean) st = 0.f;
      const float sp = st * ipos;
      // P' packed now, stored into TMEM once F2b of the previous chunk has read the buffer
      if (!cols_above) {  // minus the mean term, in packed 16-bit arithmetic; zero above the diagonal
        const uint32_t sp2 = pack2<AB16>(sp, sp);
        if (cols_below) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(sub2<AB16>(__float_as_uint(v[i]), sp2));
        } else {
          const int tl = t - 64 * hp;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const uint32_t m = (2 * i + 1 <= tl) ? 0xFFFFFFFFu : ((2 * i <= tl) ? 0x0000FFFFu : 0u);
            v[i] = __uint_as_float(sub2<AB16>(__float_as_uint(v[i]), sp2) & m);
          }
        }
      }
      if (c > 0) pipe_wait(&S.z_full[(c - 1) & 1], ((c - 1) >> 1) & 1, ab, err, 8);
      if (!cols_above) tmem_st32(lrow + T_P + 32 * hp, v);
      if (hp == 0) tmem_st1(lrow + T_P + 64, pack2<AB16>(-sp, -sp));
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(&S.pready);
      // lambda / pos for the output group and the token_aux side output, while F2b runs
      if (hp == 0) {
        // NORM: the gate logit and s_t were formed from the raw q; r_t scales both
        float lamv;
        if (gate) lamv = sigmoidf_(rqv * (ext[2] + ext[3]) + gate_b);
        else lamv = t < valid ? act_load<AB16>(a.lam, (sq.bos + t0 + t) * H + h) : 0.f;
        S.cf[pb][t] = lamv * ipos;
        if (NORM) S.rqo[pb][t] = rqv;
        warp_arrive(&S.cf_ready[pb]);
        if (a.token_aux && t < valid) {
          float2* aux = reinterpret_cast<float2*>(a.token_aux + ((sq.bos + t0 + t) * H + h) * 2);
          *aux = make_float2(lamv, st * rqv);
        }
        if (NORM && t < valid) a.norm_aux[((sq.bos + t0 + t) * H + h) * 2] = rqv;
      }
    }
  } else {
    // ------------------------------------------------------------------ output group: C, q_clean
    const int qd = warp & 3;
    const int ho = (warp - 4 - GROUP_WARPS) >> 2;  // column half: columns 64ho .. 64ho+63
    const int r = 32 * qd + lane;                  // state row (C) or token (Z)
    const uint32_t lrow = tbase + ((uint32_t)(32 * qd) << 16);
    const uint32_t cpan = sbase + F_OFF_C + (uint32_t)ho * F_QPANEL;
    const bool leader = warp == 4 + GROUP_WARPS && lane == 0;  // issues the bulk stores
    float v[64];

    // initial state -> TMEM C and the bf16 operand for chunk 0
    if (a.initial_cov) {
      const float4* src = reinterpret_cast<const float4*>(a.initial_cov + (st_base + r) * 128 + 64 * ho);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 f = src[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = 0.f;
    }
    tmem_st32(lrow + T_C + 64 * ho, v);
    tmem_st32(lrow + T_C + 64 * ho + 32, v + 32);
    if (nchunks == 0 && a.final_cov) {
      float4* dst = reinterpret_cast<float4*>(a.final_cov + (st_base + r) * 128 + 64 * ho);
#pragma unroll
      for (int i = 0; i < 16; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    store_row64<AB16>(cpan, r, v);
    tmem_st_wait();
    fence_async_smem();
    tc_fence_before();
    warp_arrive(&S.c_read);
    warp_arrive(&S.cconv);

    for (int c = 0; c < nchunks; ++c) {
      const int s = c & 1;
      const int t0 = c * F_BT;
      const int valid = min(F_BT, sq.len - t0);
      // ---------------- C after chunk c -> bf16 operand of chunk c+1 (or the final state)
      pipe_wait(&S.c_full, c & 1, ab, err, 32);
      tc_fence_after();
      tmem_ld64(lrow + T_C + 64 * ho, v);
      tc_fence_before();
      warp_arrive(&S.c_read);
      if (c + 1 < nchunks) {
        pipe_wait(&S.cprev_free, c & 1, ab, err, 64);
        store_row64<AB16>(cpan, r, v);
        fence_async_smem();
        // cconv is one barrier whose phases are tested by parity: arrive only for a chunk that
        // exists.  An arrival in the last chunk could complete a second phase before the MMA
        // thread has tested the one for the last chunk's F2a, which then would read as pending.
        warp_arrive(&S.cconv);
      } else if (a.final_cov) {
        float4* dst = reinterpret_cast<float4*>(a.final_cov + (st_base + r) * 128 + 64 * ho);
#pragma unroll
        for (int i = 0; i < 16; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      }
      // ---------------- q_clean of chunk c = q - (lambda / pos) Z
      // The Q tile of the stage was released after the chunk's last MMA; q is read again (from L2)
      // into the staging tile, once the previous bulk store has read that tile.
      if (leader) {
        bulk_wait_read();
        const int row = (int)(sq.bos + (int64_t)t0);
        mbar_arrive_expect_tx(&S.qo_full, F_QTILE);
        tma_load_3d(sm + F_OFF_O, &tmq, &S.qo_full, 0, h, row);
        tma_load_3d(sm + F_OFF_O + F_QPANEL, &tmq, &S.qo_full, 64, h, row);
      }
      pipe_wait(&S.z_full[s], (c >> 1) & 1, ab, err, 128);
      tc_fence_after();
      tmem_ld64(lrow + T_R + T_RSTRIDE * s + 64 * ho, v);
      tc_fence_before();
      warp_arrive(&S.z_free[s]);
      pipe_wait(&S.cf_ready[s], (c >> 1) & 1, ab, err, 0x200);
      const float rq = NORM ? S.rqo[s][r] : 1.f;
      const float cf = NORM ? S.cf[s][r] * rq : S.cf[s][r];  // NORM: Z holds Z_true / r_t
      const uint32_t opan = sbase + F_OFF_O + (uint32_t)ho * F_QPANEL;
      own_copy_wait(&S.qo_full, c & 1, ab, err, 0x400);  // q of this chunk, reloaded into the staging tile
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const uint32_t ad = opan + sw128(r, cc);
        uint4 qv = ld_shared_v4(ad);
        if (NORM) {  // the raw q re-read from memory, normalised and rounded as l2norm's output
          uint32_t u[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack2<AB16>(u[j]);
            u[j] = pack2<AB16>(f.x * rq, f.y * rq);
          }
          qv = make_uint4(u[0], u[1], u[2], u[3]);
        }
        st_shared_v4(ad, sub2<AB16>(qv.x, pack2<AB16>(cf * v[8 * cc], cf * v[8 * cc + 1])),
                     sub2<AB16>(qv.y, pack2<AB16>(cf * v[8 * cc + 2], cf * v[8 * cc + 3])),
                     sub2<AB16>(qv.z, pack2<AB16>(cf * v[8 * cc + 4], cf * v[8 * cc + 5])),
                     sub2<AB16>(qv.w, pack2<AB16>(cf * v[8 * cc + 6], cf * v[8 * cc + 7])));
      }
      if (valid == F_BT) {
        fence_async_smem();
        bar_sync<7, 32 * GROUP_WARPS>();
        if (leader) {
          const int row = (int)(sq.bos + (int64_t)t0);
          tma_store_3d(&tmo, sm + F_OFF_O, 0, h, row);
          tma_store_3d(&tmo, sm + F_OFF_O + F_QPANEL, 64, h, row);
          bulk_commit();
        }
      } else {
        // partial chunk: this warp's 32 rows x 64 columns, four 128-byte row segments per store
        __syncwarp();
        uint8_t* obase = (uint8_t*)a.q_clean + ((sq.bos + t0) * H + h) * 256 + ho * 128 + (lane & 7) * 16;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = 32 * qd + 4 * i + (lane >> 3);
          const uint4 ov = ld_shared_v4(opan + sw128(row, lane & 7));
          if (row < valid) *reinterpret_cast<uint4*>(obase + (int64_t)row * H * 256) = ov;
        }
      }
    }
    if (leader) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// CCQ_B200_DEBUG_STALL_CYCLES=<n> (debug only): the forward kernel's first wait gives up after n
// clock cycles (at most 2^31), exercising the bounded-wait error path; unset or 0 in normal use.
long long debug_stall_cycles() {
  const char* env = getenv("CCQ_B200_DEBUG_STALL_CYCLES");
  if (env == nullptr) return 0;
  long long v = atoll(env);
  if (v < 0) v = 0;
  if (v > (1ll << 31)) v = 1ll << 31;
  return v;
}

template <int AB16, int NORM>
cudaError_t launch(const CleanArgs& a, int* launches) {
  CUtensorMap tq, tk, to, tkn;
  const int64_t rows = (int64_t)a.B * a.T;
  cudaError_t e = tc::make_token_map(&tq, a.q, rows, a.H, 128, F_BT, AB16 != 0);
  if (e != cudaSuccess) return e;
  if ((e = tc::make_token_map(&tk, a.k, rows, a.H, 128, F_BT, AB16 != 0)) != cudaSuccess) return e;
  if ((e = tc::make_token_map(&to, a.q_clean, rows, a.H, 128, F_BT, AB16 != 0)) != cudaSuccess) return e;
  if (NORM) {
    if ((e = tc::make_token_map(&tkn, a.k_norm, rows, a.H, 128, F_BT, AB16 != 0)) != cudaSuccess) return e;
  } else {
    tkn = tk;  // unused
  }
  int* err = reinterpret_cast<int*>(a.workspace);
  if ((e = cudaMemsetAsync(err, 0, 2 * sizeof(int), a.stream)) != cudaSuccess) return e;
  CleanArgs la = a;
  la.doc_order = nullptr;
  if (lpt_order_bytes(a.n_seqs, a.cu_seqlens != nullptr) > 0) {
    int* order = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(a.workspace) + 256);
    if ((e = lpt_order(a, order, launches)) != cudaSuccess) return e;
    la.doc_order = order;
  }
  la.debug_stall_cycles = debug_stall_cycles();
  auto kern = tc_fwd_kernel<AB16, NORM>;
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)F_SMEM)) != cudaSuccess)
    return e;
  kern<<<a.n_seqs * a.H, F_THREADS, F_SMEM, a.stream>>>(tq, tk, to, tkn, la, err);
  *launches += 1;
  return cudaGetLastError();
}

}  // namespace

// error word (256 bytes), then the varlen launch order
size_t tc_fwd_workspace(int B, int, int, int, int n_seqs) {
  return 256 + lpt_order_bytes(n_seqs, B == 1 && n_seqs >= 2);
}

cudaError_t tc_fwd(const CleanArgs& a, int* launches) {
  if (a.qk_norm) return a.dtype == DT_BF16 ? launch<1, 1>(a, launches) : launch<0, 1>(a, launches);
  return a.dtype == DT_BF16 ? launch<1, 0>(a, launches) : launch<0, 0>(a, launches);
}

}  // namespace ccq
