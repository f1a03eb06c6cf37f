/*
 * ccq_b200.h -- C ABI of the B200-native CCQ cleaning operator.
 *
 * The operator (ledong0110/CCQ, ccq/ops/common/fused_read.py:11-25):
 *
 *   C_t = C_0 + sum_{j<=t} k_j k_j^T        m_t = m_0 + sum_{j<=t} k_j
 *   pos_t = t + position_offset (1-based, clamped >= 1, restarting per document)
 *   z_t[v] = sum_k q_t[k] C_t[k,v]          s_t = m_t . q_t
 *   q_clean_t = q_t - lambda_t (z_t / pos_t - s_t m_t / pos_t^2)   (mean term iff subtract_mean)
 *
 * Conventions shared by every entry point:
 *   - All pointers are DEVICE pointers unless stated; all tensors are contiguous.
 *   - Token tensors (q, k, q_clean, dq, dk, ...) are [B, T, H, K] row-major in the activation
 *     dtype.  Varlen batches use B == 1 and cu_seqlens (int64, [n_seqs + 1], device), exactly as
 *     the reference's cu_seqlens argument; dense batches pass cu_seqlens = NULL and n_seqs = B.
 *   - States are fp32: cov [n_seqs, H, K, K] in the fla layout (z = q @ C), mean [n_seqs, H, K].
 *   - lambda is per token [B, T, H] in the activation dtype (CCQ_LAMBDA_TOKEN), or the per-head
 *     gate lambda = sigmoid(W[h] . q_t + b[h]) with W [H, K] fp32 and b [H] fp32 computed inside
 *     the kernels (CCQ_LAMBDA_GATE).
 *   - stream is a cudaStream_t passed as void*; every launch goes to that stream, no entry point
 *     synchronises, and none allocates device memory: the caller owns every buffer, including the
 *     workspace sized by ccq_workspace_size().
 *   - Every entry point returns a ccq_status; on failure ccq_last_error() returns a message for
 *     the calling thread.  Calls on different streams from different threads are independent.
 *   - cu_seqlens must start at 0, never decrease and end at T (the reference's convention).  The
 *     kernels clamp every offset into [0, T], so a malformed array gives wrong documents but no
 *     access outside the tensors; the Python layer validates it when CCQ_B200_CHECK=1.
 *   - Device-side failures: every pipeline wait inside the tensor-core kernels is bounded (about a
 *     second).  A wait that gives up makes the kernel unwind without hanging and OR a non-zero code
 *     into the first 4 bytes (an int) of the workspace it was given; the launcher zeroes that word
 *     first.  The entry points return before the kernels run, so they cannot see it; read it with
 *     ccq_device_status() (ccq_noalloc_status() for ccq_clean_bwd_noalloc), or set the environment
 *     variable CCQ_B200_CHECK=1, which makes every tensor-core call wait for its kernels and return
 *     CCQ_ERR_CUDA with the code in its message.
 */
#ifndef CCQ_B200_H_
#define CCQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  CCQ_OK = 0,
  CCQ_ERR_INVALID = 1,      /* bad pointer, shape, dtype or option */
  CCQ_ERR_UNSUPPORTED = 2,  /* valid request this build does not implement (e.g. K > 256) */
  CCQ_ERR_CUDA = 3,         /* a CUDA runtime or driver call failed */
  CCQ_ERR_WORKSPACE = 4     /* workspace missing or smaller than ccq_workspace_size() */
} ccq_status;

typedef enum { CCQ_F32 = 0, CCQ_BF16 = 1, CCQ_F16 = 2 } ccq_dtype;

typedef enum { CCQ_LAMBDA_TOKEN = 0, CCQ_LAMBDA_GATE = 1 } ccq_lambda_mode;

typedef enum { CCQ_OP_FWD = 0, CCQ_OP_BWD = 1, CCQ_OP_DECODE = 2 } ccq_op;

/* Implementation a call took (for tests and benchmarks): see ccq_last_path(). */
typedef enum { CCQ_PATH_NONE = 0, CCQ_PATH_SIMT = 1, CCQ_PATH_TCGEN05 = 2, CCQ_PATH_DECODE = 3 } ccq_path;

/* Message of the last failed call on this thread ("" if none). */
const char* ccq_last_error(void);

/* Which kernel family the last successful call on this thread launched. */
int ccq_last_path(void);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int ccq_version(void);

/* Number of kernel launches the last successful call on this thread issued. */
int ccq_last_launch_count(void);

/*
 * Bytes of workspace `op` needs for these sizes (0 if none), enough for whichever backward path a
 * call takes (for CCQ_OP_BWD the larger of the two).  total_tokens = B*T.
 * Replaces the temporaries the reference allocates inside _fused_read_fwd/_fused_read_bwd
 * (fused_read.py:385-394, :413-434).
 */
size_t ccq_workspace_size(int op, int dtype, int B, int T, int H, int K, int n_seqs);

/*
 * Bytes of workspace for the path a call with these sizes will take.  flags: CCQ_WS_HAVE_FWD_OUTPUTS
 * when the backward will be given the forward's state_cov / state_mean / token_aux (the tensor-core
 * backward then runs where supported and needs a few hundred bytes per (document, head); without
 * them the exact backward checkpoints a K x K state per chunk).  Same role as ccq_workspace_size.
 */
#define CCQ_WS_HAVE_FWD_OUTPUTS 1
#define CCQ_WS_L2NORM 2  /* the call is a ccq_clean_l2norm_* call */
size_t ccq_workspace_size_for(int op, int dtype, int B, int T, int H, int K, int n_seqs, int flags);

/*
 * Error word of the tensor-core kernels that last used `workspace` on `stream`: waits for the
 * stream, then stores 0 (no wait gave up) or the OR of the codes of the waits that gave up in *code.
 * No counterpart in the reference (its Triton kernels have no bounded waits).
 */
int ccq_device_status(const void* workspace, void* stream, int* code);

/*
 * Forward: q_clean, and optionally the final cov / mean states.
 * Replaces FusedCCQCleanRead.forward / _fused_read_fwd (fused_read.py:379-403, :480-491).
 *   lambda_mode == CCQ_LAMBDA_TOKEN: lam [B,T,H] activation dtype; gate_w/gate_b unused.
 *   lambda_mode == CCQ_LAMBDA_GATE : gate_w [H,K] f32, gate_b [H] f32; lam unused.
 *   token_aux: optional [B,T,H,2] f32 output, per token and head the lambda used and
 *     s_t = m_t . q_t; the tensor-core backward reads it back instead of recomputing both.
 *   initial_cov / initial_mean: optional; initial_mean is ignored unless subtract_mean.
 *   final_cov / final_mean: optional outputs (the backward's tensor-core path reads them back);
 *   they must not alias initial_cov / initial_mean (column tiles of one head read the initial
 *   state while another tile writes the final one).
 */
int ccq_clean_fwd(int dtype, int B, int T, int H, int K,
                  const void* q, const void* k,
                  int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                  float* token_aux,
                  const int64_t* cu_seqlens, int n_seqs,
                  int position_offset, int subtract_mean,
                  const float* initial_cov, const float* initial_mean,
                  void* q_clean, float* final_cov, float* final_mean,
                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward: dq, dk, dlambda (TOKEN mode) or dW/db (GATE mode), and the initial-state gradients.
 * Replaces FusedCCQCleanRead.backward / _fused_read_bwd (fused_read.py:406-460, :496-514).
 *   state_cov / state_mean / token_aux: the final states and per-token side outputs the forward
 *     wrote for these inputs.  The tensor-core backward needs all three (it walks the chunks
 *     backwards from the final state); when any is NULL the exact SIMT backward runs instead.
 *   dq_clean: upstream gradient [B,T,H,K]; dfinal_cov / dfinal_mean: optional state gradients.
 *   dlam: [B,T,H] f32 output (TOKEN mode), may be NULL when lambda needs no gradient.
 *   dgate_w [H,K] / dgate_b [H] f32 outputs (GATE mode; overwritten, summed over the batch).
 *   dinitial_cov [n_seqs,H,K,K], dinitial_mean [n_seqs,H,K]: optional outputs; dinitial_mean is
 *     written only when subtract_mean or dfinal_mean is given (fused_read.py:444-450).
 */
int ccq_clean_bwd(int dtype, int B, int T, int H, int K,
                  const void* q, const void* k,
                  int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                  const int64_t* cu_seqlens, int n_seqs,
                  int position_offset, int subtract_mean,
                  const float* initial_cov, const float* initial_mean,
                  const float* state_cov, const float* state_mean, const float* token_aux,
                  const void* dq_clean, const float* dfinal_cov, const float* dfinal_mean,
                  void* dq, void* dk, float* dlam, float* dgate_w, float* dgate_b,
                  float* dinitial_cov, float* dinitial_mean,
                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Forward with the L2 normalisation of q and k inside the operator.  Replaces the pair
 *   q = l2norm(q, eps=1e-6); k = l2norm(k, eps=1e-6); fused_ccq_clean_read(q, k, ...)
 * that both fused_chunk orchestrators run (ccq/ops/ccq_gdn/fused_chunk.py:42-53 with
 * use_qk_l2norm_in_kernel, ccq/ops/ccq_gla/fused_chunk.py:31-41; fla l2norm at
 * fla/modules/l2norm.py:266): y = x / sqrt(sum(x^2) + 1e-6) per (token, head), fp32 math, rounded to
 * the activation dtype, then the operator on the normalised q and k.
 *   q, k: the raw (un-normalised) inputs.
 *   k_norm: output [B,T,H,K], the normalised keys (the backbone reads them next).
 *   norm_aux: output [B,T,H,2] f32, per token and head 1/|q| and 1/|k|; the backward reads it.
 *   Everything else as ccq_clean_fwd.  The tensor-core path normalises the tiles it loads, so the
 *   normalised q never goes to memory; the exact path keeps it in the workspace
 *   (ccq_workspace_size_for with CCQ_WS_L2NORM).
 */
int ccq_clean_l2norm_fwd(int dtype, int B, int T, int H, int K,
                         const void* q, const void* k,
                         int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                         float* token_aux, float* norm_aux,
                         const int64_t* cu_seqlens, int n_seqs,
                         int position_offset, int subtract_mean,
                         const float* initial_cov, const float* initial_mean,
                         void* q_clean, void* k_norm, float* final_cov, float* final_mean,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward of ccq_clean_l2norm_fwd: gradients on the RAW q and k.  Replaces the backward of the same
 * l2norm + fused_ccq_clean_read pair (fla l2norm_bwd, fla/modules/l2norm.py:49-72, and
 * FusedCCQCleanRead.backward, fused_read.py:496-514), including autograd's sum of the two
 * gradients on the normalised keys (the operator's and the backbone's).
 *   q: the raw queries; k_norm: the forward's k_norm output; norm_aux: the forward's norm_aux.
 *   dk_norm: optional gradient arriving on k_norm from the rest of the model (NULL = none); the
 *     tensor-core path adds it inside its kernel and needs it 16-byte aligned (otherwise the call
 *     takes the exact path, as for the other tensors).
 *   dq, dk: outputs, gradients on the raw q and k.  Everything else as ccq_clean_bwd.
 */
int ccq_clean_l2norm_bwd(int dtype, int B, int T, int H, int K,
                         const void* q, const void* k_norm,
                         int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                         const int64_t* cu_seqlens, int n_seqs,
                         int position_offset, int subtract_mean,
                         const float* initial_cov, const float* initial_mean,
                         const float* state_cov, const float* state_mean, const float* token_aux,
                         const float* norm_aux,
                         const void* dq_clean, const void* dk_norm, const float* dfinal_cov, const float* dfinal_mean,
                         void* dq, void* dk, float* dlam, float* dgate_w, float* dgate_b,
                         float* dinitial_cov, float* dinitial_mean,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward that allocates nothing.  No counterpart in the reference: the reference's backward gets
 * its scratch from PyTorch's allocator.  This entry point is for callers that cannot hand over a
 * device workspace, for instance a host binding without a device allocator of its own, or a
 * serving loop that keeps the allocator out of its steady state.
 *
 * Same arguments, outputs and errors as ccq_clean_bwd, minus workspace / workspace_bytes: the
 * scratch is a fixed array of CCQ_NOALLOC_SCRATCH_BYTES (1 MiB) in the library's device data.
 *   - A call whose scratch need, on the path it takes, exceeds 1 MiB fails with CCQ_ERR_WORKSPACE
 *     before anything is launched.  The tensor-core backward (bf16 / fp16, K = 128) needs about
 *     256 + 516 * n_seqs * H bytes (plus 4 * n_seqs for a varlen batch), so it fits up to
 *     n_seqs * H = 2031 for a dense batch; the exact fp32 backward's need grows with the sequence
 *     length (ccq_workspace_size_for gives either path's need).
 *   - Every call looks the scratch up on the current device (cudaGetSymbolAddress), and the first
 *     call on a device may load the library's device code; make that first call before any stream
 *     capture begins.
 *   - A bounded pipeline wait that gives up writes its code into the scratch's error word, which
 *     ccq_noalloc_status() reads back.
 *   - All calls on one device share the one scratch array: calls that overlap in time (other
 *     streams, other host threads) race and give wrong results.  Calls issued one after the other
 *     on one stream are safe.
 *   - The kernels clear the part of the scratch that must start at zero on every call.
 */
#define CCQ_NOALLOC_SCRATCH_BYTES (1u << 20)
int ccq_clean_bwd_noalloc(int dtype, int B, int T, int H, int K,
                          const void* q, const void* k,
                          int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                          const int64_t* cu_seqlens, int n_seqs,
                          int position_offset, int subtract_mean,
                          const float* initial_cov, const float* initial_mean,
                          const float* state_cov, const float* state_mean, const float* token_aux,
                          const void* dq_clean, const float* dfinal_cov, const float* dfinal_mean,
                          void* dq, void* dk, float* dlam, float* dgate_w, float* dgate_b,
                          float* dinitial_cov, float* dinitial_mean, void* stream);

/*
 * Error word of the last ccq_clean_bwd_noalloc call on the current device (see "Device-side
 * failures" above): waits for `stream`, then stores 0 or the timeout code in *code.  Allocates
 * nothing.  No counterpart in the reference.
 */
int ccq_noalloc_status(void* stream, int* code);

/*
 * Recurrent (decode / short prefill) cleaning with the generation cache.
 * Replaces fla fused_recurrent_gla(q, k, v=k, scale=1) + _CCQCleanQ as called by
 * fused_ccq_clean(use_chunk=False) (ccq/ops/ccq_gdn/fused_clean.py:34-83) and
 * ccq/ops/ccq_gla/fused_recurrent.py:26-38.  The state read is inclusive of the token.
 *   cov_in / mean_in: cache states before the call (NULL = zeros); cov_out / mean_out: states
 *   after the last token (may alias cov_in / mean_in for an in-place cache update).
 *   mean_in/mean_out are used only when subtract_mean.
 */
int ccq_decode_step(int dtype, int B, int T, int H, int K,
                    const void* q, const void* k,
                    int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                    const int64_t* cu_seqlens, int n_seqs,
                    int position_offset, int subtract_mean,
                    const float* cov_in, const float* mean_in,
                    float* cov_out, float* mean_out,
                    void* q_clean, void* stream);

/*
 * The decode step with the L2 normalisation of q and k inside the kernel.  Replaces
 *   fused_ccq_clean(q, k, ..., use_qk_l2norm_in_kernel=True, use_chunk=False)
 * (ccq/ops/ccq_gdn/fused_clean.py:34-83: fla l2norm of both, then the recurrent read and the
 * cleaning), which the GDN layer's fused_recurrent mode calls (ccq/gdn/layer.py:374-390), and the
 * l2norm + cleaning sequence of ccq/ops/ccq_gla/fused_recurrent.py:26-38.
 *   q, k: the raw tokens; k_norm: output [B,T,H,K], the normalised keys (what the cache and the
 *   backbone see); everything else as ccq_decode_step.  With k_norm == NULL this is ccq_decode_step.
 */
int ccq_decode_step_l2norm(int dtype, int B, int T, int H, int K,
                           const void* q, const void* k,
                           int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                           const int64_t* cu_seqlens, int n_seqs,
                           int position_offset, int subtract_mean,
                           const float* cov_in, const float* mean_in,
                           float* cov_out, float* mean_out,
                           void* q_clean, void* k_norm, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CCQ_B200_H_ */
