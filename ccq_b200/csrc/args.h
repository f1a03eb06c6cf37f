// Host-side argument bundle shared by the C entry points and the kernel launchers.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ccq {

enum { LAMBDA_TOKEN = 0, LAMBDA_GATE = 1 };
enum { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

struct CleanArgs {
  int dtype, B, T, H, K, n_seqs;
  const void* q;
  const void* k;
  int lambda_mode;
  const void* lam;
  const float* gate_w;
  const float* gate_b;
  float* token_aux;        // fwd output [B,T,H,2]: lambda_t, s_t
  const int64_t* cu_seqlens;
  int position_offset, subtract_mean;
  const float* initial_cov;
  const float* initial_mean;
  // forward outputs
  void* q_clean;
  float* final_cov;
  float* final_mean;
  // backward inputs / outputs
  const float* state_cov;
  const float* state_mean;
  const float* token_aux_in;  // bwd input, as written by the forward
  const void* dq_clean;
  const float* dfinal_cov;
  const float* dfinal_mean;
  void* dq;
  void* dk;
  float* dlam;
  float* dgate_w;
  float* dgate_b;
  float* dinitial_cov;
  float* dinitial_mean;
  // decode states
  const float* cov_in;
  const float* mean_in;
  float* cov_out;
  float* mean_out;
  void* workspace;
  size_t workspace_bytes;
  cudaStream_t stream;
  // tensor-core kernels: varlen launch order (device, [n_seqs]; nullptr = document order), set by
  // the launchers from the workspace
  const int* doc_order;
  // L2 normalisation of q and k inside the operator (the *_l2norm entry points): q and k are the
  // raw inputs; the forward also writes the normalised keys and the two reciprocal norms per
  // (token, head); the backward reads the normalised keys as `k`, the saved norms, and the
  // gradient arriving on the normalised keys from the rest of the model.
  int qk_norm;
  void* k_norm;             // fwd output [B,T,H,K]
  float* norm_aux;          // fwd output [B,T,H,2]: 1/|q|, 1/|k|
  const float* norm_aux_in; // bwd input, as written by the forward
  const void* dk_ext;       // bwd input [B,T,H,K] or nullptr
  // debug only (tensor-core forward): > 0 makes the kernel's first wait give up after that many
  // cycles, to exercise the bounded-wait error path
  long long debug_stall_cycles;
};

// Workspace carving: every region starts on a 256-byte boundary.
inline size_t ws_align(size_t x) { return (x + 255) & ~size_t(255); }

// SIMT path (any K <= 256, fp32/bf16/fp16)
size_t simt_bwd_workspace(int B, int T, int H, int K, int n_seqs);
cudaError_t simt_fwd(const CleanArgs& a, int* launches);
cudaError_t simt_bwd(const CleanArgs& a, int* launches);

// Row-wise L2 normalisation (l2norm.cu): rows of K elements; r arrays hold two floats per row,
// `slot` picks which.
cudaError_t l2norm_rows_fwd(int dtype, const void* x, void* y, float* r_out, int slot, int64_t rows, int K,
                            cudaStream_t st);
cudaError_t l2norm_rows_scale(int dtype, const void* x, void* y, const float* r_in, int slot, int64_t rows, int K,
                              cudaStream_t st);
cudaError_t l2norm_rows_bwd(int dtype, void* d, const void* d_ext, const void* y, const float* r_in, int slot,
                            int64_t rows, int K, cudaStream_t st);

// decode step (K % 4 == 0, K <= 256)
cudaError_t decode_step(const CleanArgs& a, int* launches);

// tensor-core path (bf16/fp16, K == 128)
bool tc_supported(const CleanArgs& a, int op);
// Longest-first launch order of varlen documents: bytes it needs in a workspace (0 when the batch
// gets no reordering) and the kernel that writes it.
size_t lpt_order_bytes(int n_seqs, bool varlen);
cudaError_t lpt_order(const CleanArgs& a, int* order, int* launches);
size_t tc_fwd_workspace(int B, int T, int H, int K, int n_seqs);
size_t tc_bwd_workspace(int B, int T, int H, int K, int n_seqs);
cudaError_t tc_fwd(const CleanArgs& a, int* launches);
cudaError_t tc_bwd(const CleanArgs& a, int* launches);

}  // namespace ccq
