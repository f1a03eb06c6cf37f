// C ABI of the B200 CCQ cleaning operator: argument validation, dispatch and error reporting.
// Declarations and contracts: include/ccq_b200.h.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/ccq_b200.h"
#include "args.h"

namespace {

thread_local char g_err[512] = "";
thread_local int g_path = CCQ_PATH_NONE;
thread_local int g_launches = 0;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(CCQ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// The tensor-core kernels' error word (word 0 of the workspace they were given): 0, or the OR of
// the codes of the pipeline waits that gave up.  Copied to the host after the stream drains.
int read_device_word(const void* ws, cudaStream_t stream, int* code) {
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, ws, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  *code = v;
  return CCQ_OK;
}

// With CCQ_B200_CHECK=1 in the environment every tensor-core call waits for its kernels and returns
// CCQ_ERR_CUDA if one of their bounded pipeline waits gave up (or the launch failed asynchronously).
bool check_mode() {
  const char* env = getenv("CCQ_B200_CHECK");
  return env && env[0] == '1';
}

int checked_finish(const char* what, const void* ws, cudaStream_t stream) {
  if (!check_mode()) return CCQ_OK;
  int code = 0;
  int st = read_device_word(ws, stream, &code);
  if (st != CCQ_OK) return st;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  if (code != 0) {
    // the words after the code may hold where the pipeline stood (kernel-specific detail)
    int detail = 0;
    read_device_word(reinterpret_cast<const int*>(ws) + 1, stream, &detail);
    return fail(CCQ_ERR_CUDA, "%s: device pipeline timeout, code %#x (detail %#x)", what, code, detail);
  }
  return CCQ_OK;
}

int check_common(int dtype, int B, int T, int H, int K, const void* q, const void* k, int lambda_mode,
                 const void* lam, const float* gw, const float* gb, const int64_t* cu, int n_seqs) {
  if (dtype != CCQ_F32 && dtype != CCQ_BF16 && dtype != CCQ_F16) return fail(CCQ_ERR_INVALID, "unknown dtype %d", dtype);
  if (B < 1 || T < 0 || H < 1 || K < 1) return fail(CCQ_ERR_INVALID, "bad sizes B=%d T=%d H=%d K=%d", B, T, H, K);
  if (K > 256) return fail(CCQ_ERR_UNSUPPORTED, "head size K=%d > 256 is not supported", K);
  if ((int64_t)H * 65535 < 0 || H > 65535) return fail(CCQ_ERR_INVALID, "H=%d too large", H);
  if (T > 0 && (q == nullptr || k == nullptr)) return fail(CCQ_ERR_INVALID, "q and k are required");
  if (lambda_mode == CCQ_LAMBDA_TOKEN) {
    if (T > 0 && lam == nullptr) return fail(CCQ_ERR_INVALID, "lambda (per token) is required");
  } else if (lambda_mode == CCQ_LAMBDA_GATE) {
    if (gw == nullptr || gb == nullptr) return fail(CCQ_ERR_INVALID, "gate_w and gate_b are required in GATE mode");
  } else {
    return fail(CCQ_ERR_INVALID, "unknown lambda_mode %d", lambda_mode);
  }
  if (cu == nullptr) {
    if (n_seqs != B) return fail(CCQ_ERR_INVALID, "dense batch: n_seqs (%d) must equal B (%d)", n_seqs, B);
  } else {
    if (B != 1) return fail(CCQ_ERR_INVALID, "varlen batch (cu_seqlens given) needs B == 1, got %d", B);
    if (n_seqs < 1) return fail(CCQ_ERR_INVALID, "varlen batch needs n_seqs >= 1");
  }
  if (n_seqs > 65535) return fail(CCQ_ERR_UNSUPPORTED, "n_seqs=%d > 65535", n_seqs);
  return CCQ_OK;
}

ccq::CleanArgs base_args(int dtype, int B, int T, int H, int K, const void* q, const void* k, int lambda_mode,
                         const void* lam, const float* gw, const float* gb, const int64_t* cu, int n_seqs,
                         int position_offset, int subtract_mean, void* stream) {
  ccq::CleanArgs a;
  memset(&a, 0, sizeof(a));
  a.dtype = dtype; a.B = B; a.T = T; a.H = H; a.K = K; a.n_seqs = n_seqs;
  a.q = q; a.k = k;
  a.lambda_mode = lambda_mode; a.lam = lam; a.gate_w = gw; a.gate_b = gb;
  a.cu_seqlens = cu;
  a.position_offset = position_offset;
  a.subtract_mean = subtract_mean ? 1 : 0;
  a.stream = (cudaStream_t)stream;
  return a;
}

size_t elem_bytes(int dtype) { return dtype == CCQ_F32 ? 4 : 2; }

// bytes of the normalised-q copy the exact path keeps in the workspace (l2norm entry points only)
size_t qhat_bytes(const ccq::CleanArgs& a) {
  return ccq::ws_align((size_t)a.B * a.T * a.H * a.K * elem_bytes(a.dtype));
}

// Forward dispatch shared by ccq_clean_fwd and ccq_clean_l2norm_fwd.  With qk_norm the tensor-core
// kernel normalises in its tile loads; the exact path normalises q into the workspace and k into
// k_norm first, then runs on those.
int run_fwd(ccq::CleanArgs& a, const char* who) {
  int launches = 0;
  cudaError_t e;
  const bool tc = ccq::tc_supported(a, CCQ_OP_FWD) && (!a.qk_norm || ((uintptr_t)a.k_norm & 15) == 0);
  if (tc) {
    size_t need = ccq::tc_fwd_workspace(a.B, a.T, a.H, a.K, a.n_seqs);
    if (need > 0 && (a.workspace == nullptr || a.workspace_bytes < need))
      return fail(CCQ_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", who, need, a.workspace_bytes);
    e = ccq::tc_fwd(a, &launches);
    g_path = CCQ_PATH_TCGEN05;
  } else if (a.qk_norm) {
    const size_t need = qhat_bytes(a);
    if (a.T > 0 && (a.workspace == nullptr || a.workspace_bytes < need))
      return fail(CCQ_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", who, need, a.workspace_bytes);
    const int64_t rows = (int64_t)a.B * a.T * a.H;
    ccq::CleanArgs b = a;
    b.q = a.workspace;
    b.k = a.k_norm;
    e = ccq::l2norm_rows_fwd(a.dtype, a.q, a.workspace, a.norm_aux, 0, rows, a.K, a.stream);
    if (e == cudaSuccess) e = ccq::l2norm_rows_fwd(a.dtype, a.k, a.k_norm, a.norm_aux, 1, rows, a.K, a.stream);
    launches += 2;
    if (e == cudaSuccess) e = ccq::simt_fwd(b, &launches);
    g_path = CCQ_PATH_SIMT;
  } else {
    e = ccq::simt_fwd(a, &launches);
    g_path = CCQ_PATH_SIMT;
  }
  if (e != cudaSuccess) {
    char what[96];
    snprintf(what, sizeof(what), "%s launch", who);
    return cuda_fail(e, what);
  }
  g_launches = launches;
  if (tc && a.workspace != nullptr) return checked_finish(who, a.workspace, a.stream);
  return CCQ_OK;
}

// Backward dispatch shared by ccq_clean_bwd and ccq_clean_l2norm_bwd.
int run_bwd(ccq::CleanArgs& a, const char* who) {
  const bool tc = ccq::tc_supported(a, CCQ_OP_BWD) && a.state_cov != nullptr && a.token_aux_in != nullptr &&
                  (a.state_mean != nullptr || !a.subtract_mean) &&
                  (!a.qk_norm || (((uintptr_t)a.dk_ext & 15) == 0));
  const int B = a.B, T = a.T, H = a.H, K = a.K, n = a.n_seqs;
  size_t need = tc ? ccq::tc_bwd_workspace(B, T, H, K, n) : ccq::simt_bwd_workspace(B, T, H, K, n);
  const size_t qh = (!tc && a.qk_norm) ? qhat_bytes(a) : 0;
  need += qh;
  if (T > 0 && need > 0 && (a.workspace == nullptr || a.workspace_bytes < need))
    return fail(CCQ_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", who, need, a.workspace_bytes);
  int launches = 0;
  cudaError_t e = cudaSuccess;
  if (tc) {
    e = ccq::tc_bwd(a, &launches);
    g_path = CCQ_PATH_TCGEN05;
  } else if (a.qk_norm) {
    // exact path: q_hat recomputed bit for bit from the saved norms, the operator's backward on
    // (q_hat, k_hat), then both gradients mapped back through the normalisation
    const int64_t rows = (int64_t)B * T * H;
    ccq::CleanArgs b = a;
    b.q = a.workspace;
    b.workspace = (uint8_t*)a.workspace + qh;
    b.workspace_bytes = a.workspace_bytes - qh;
    e = ccq::l2norm_rows_scale(a.dtype, a.q, a.workspace, a.norm_aux_in, 0, rows, K, a.stream);
    launches += 1;
    if (e == cudaSuccess) e = ccq::simt_bwd(b, &launches);
    if (e == cudaSuccess) e = ccq::l2norm_rows_bwd(a.dtype, a.dq, nullptr, a.workspace, a.norm_aux_in, 0, rows, K,
                                                   a.stream);
    if (e == cudaSuccess) e = ccq::l2norm_rows_bwd(a.dtype, a.dk, a.dk_ext, a.k, a.norm_aux_in, 1, rows, K, a.stream);
    launches += 2;
    g_path = CCQ_PATH_SIMT;
  } else {
    e = ccq::simt_bwd(a, &launches);
    g_path = CCQ_PATH_SIMT;
  }
  if (e != cudaSuccess) {
    char what[96];
    snprintf(what, sizeof(what), "%s launch", who);
    return cuda_fail(e, what);
  }
  g_launches = launches;
  if (tc && a.workspace != nullptr) return checked_finish(who, a.workspace, a.stream);
  return CCQ_OK;
}

}  // namespace

extern "C" {

const char* ccq_last_error(void) { return g_err; }
int ccq_last_path(void) { return g_path; }
int ccq_last_launch_count(void) { return g_launches; }
int ccq_version(void) { return 100; }

size_t ccq_workspace_size(int op, int dtype, int B, int T, int H, int K, int n_seqs) {
  if (op == CCQ_OP_BWD) {
    const size_t s = ccq_workspace_size_for(op, dtype, B, T, H, K, n_seqs, 0);
    const size_t t = ccq_workspace_size_for(op, dtype, B, T, H, K, n_seqs, CCQ_WS_HAVE_FWD_OUTPUTS);
    return s > t ? s : t;
  }
  return ccq_workspace_size_for(op, dtype, B, T, H, K, n_seqs, 0);
}


size_t ccq_workspace_size_for(int op, int dtype, int B, int T, int H, int K, int n_seqs, int flags) {
  if (B < 1 || T < 0 || H < 1 || K < 1 || K > 256 || n_seqs < 1) return 0;
  ccq::CleanArgs a;
  memset(&a, 0, sizeof(a));
  a.dtype = dtype; a.B = B; a.T = T; a.H = H; a.K = K; a.n_seqs = n_seqs;
  const size_t qh = (flags & CCQ_WS_L2NORM) ? qhat_bytes(a) : 0;
  if (op == CCQ_OP_FWD) {
    return ccq::tc_supported(a, CCQ_OP_FWD) ? ccq::tc_fwd_workspace(B, T, H, K, n_seqs) : qh;
  }
  if (op == CCQ_OP_BWD) {
    if ((flags & CCQ_WS_HAVE_FWD_OUTPUTS) && ccq::tc_supported(a, CCQ_OP_BWD))
      return ccq::tc_bwd_workspace(B, T, H, K, n_seqs);
    return ccq::simt_bwd_workspace(B, T, H, K, n_seqs) + qh;
  }
  return 0;
}

int ccq_device_status(const void* workspace, void* stream, int* code) {
  g_err[0] = 0;
  if (workspace == nullptr || code == nullptr) return fail(CCQ_ERR_INVALID, "workspace and code are required");
  return read_device_word(workspace, (cudaStream_t)stream, code);
}

int ccq_clean_fwd(int dtype, int B, int T, int H, int K, const void* q, const void* k, int lambda_mode,
                  const void* lam, const float* gate_w, const float* gate_b, float* token_aux,
                  const int64_t* cu_seqlens, int n_seqs, int position_offset, int subtract_mean,
                  const float* initial_cov, const float* initial_mean, void* q_clean, float* final_cov,
                  float* final_mean, void* workspace, size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  int st = check_common(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs);
  if (st != CCQ_OK) return st;
  if (T > 0 && q_clean == nullptr) return fail(CCQ_ERR_INVALID, "q_clean output is required");
  ccq::CleanArgs a = base_args(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs,
                               position_offset, subtract_mean, stream);
  a.token_aux = token_aux;
  a.initial_cov = initial_cov;
  a.initial_mean = initial_mean;
  a.q_clean = q_clean;
  a.final_cov = final_cov;
  a.final_mean = subtract_mean ? final_mean : nullptr;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return run_fwd(a, "ccq_clean_fwd");
}

int ccq_clean_l2norm_fwd(int dtype, int B, int T, int H, int K, const void* q, const void* k, int lambda_mode,
                         const void* lam, const float* gate_w, const float* gate_b, float* token_aux, float* norm_aux,
                         const int64_t* cu_seqlens, int n_seqs, int position_offset, int subtract_mean,
                         const float* initial_cov, const float* initial_mean, void* q_clean, void* k_norm,
                         float* final_cov, float* final_mean, void* workspace, size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  int st = check_common(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs);
  if (st != CCQ_OK) return st;
  if (T > 0 && (q_clean == nullptr || k_norm == nullptr || norm_aux == nullptr))
    return fail(CCQ_ERR_INVALID, "q_clean, k_norm and norm_aux outputs are required");
  ccq::CleanArgs a = base_args(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs,
                               position_offset, subtract_mean, stream);
  a.qk_norm = 1;
  a.k_norm = k_norm;
  a.norm_aux = norm_aux;
  a.token_aux = token_aux;
  a.initial_cov = initial_cov;
  a.initial_mean = initial_mean;
  a.q_clean = q_clean;
  a.final_cov = final_cov;
  a.final_mean = subtract_mean ? final_mean : nullptr;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return run_fwd(a, "ccq_clean_l2norm_fwd");
}

int ccq_clean_bwd(int dtype, int B, int T, int H, int K, const void* q, const void* k, int lambda_mode,
                  const void* lam, const float* gate_w, const float* gate_b, const int64_t* cu_seqlens, int n_seqs,
                  int position_offset, int subtract_mean, const float* initial_cov, const float* initial_mean,
                  const float* state_cov, const float* state_mean, const float* token_aux, const void* dq_clean,
                  const float* dfinal_cov, const float* dfinal_mean, void* dq, void* dk, float* dlam,
                  float* dgate_w, float* dgate_b, float* dinitial_cov, float* dinitial_mean, void* workspace,
                  size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  int st = check_common(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs);
  if (st != CCQ_OK) return st;
  if (T > 0 && (dq_clean == nullptr || dq == nullptr || dk == nullptr))
    return fail(CCQ_ERR_INVALID, "dq_clean, dq and dk are required");
  if (lambda_mode == CCQ_LAMBDA_GATE && (dgate_w == nullptr || dgate_b == nullptr))
    return fail(CCQ_ERR_INVALID, "dgate_w and dgate_b are required in GATE mode");
  ccq::CleanArgs a = base_args(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs,
                               position_offset, subtract_mean, stream);
  a.initial_cov = initial_cov;
  a.initial_mean = initial_mean;
  a.state_cov = state_cov;
  a.state_mean = state_mean;
  a.token_aux_in = token_aux;
  a.dq_clean = dq_clean;
  a.dfinal_cov = dfinal_cov;
  a.dfinal_mean = dfinal_mean;
  a.dq = dq;
  a.dk = dk;
  a.dlam = lambda_mode == CCQ_LAMBDA_TOKEN ? dlam : nullptr;
  a.dgate_w = dgate_w;
  a.dgate_b = dgate_b;
  a.dinitial_cov = initial_cov ? dinitial_cov : nullptr;
  a.dinitial_mean = (initial_mean && (subtract_mean || dfinal_mean)) ? dinitial_mean : nullptr;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return run_bwd(a, "ccq_clean_bwd");
}

int ccq_clean_l2norm_bwd(int dtype, int B, int T, int H, int K, const void* q, const void* k_norm, int lambda_mode,
                         const void* lam, const float* gate_w, const float* gate_b, const int64_t* cu_seqlens,
                         int n_seqs, int position_offset, int subtract_mean, const float* initial_cov,
                         const float* initial_mean, const float* state_cov, const float* state_mean,
                         const float* token_aux, const float* norm_aux, const void* dq_clean, const void* dk_norm,
                         const float* dfinal_cov, const float* dfinal_mean, void* dq, void* dk, float* dlam,
                         float* dgate_w, float* dgate_b, float* dinitial_cov, float* dinitial_mean, void* workspace,
                         size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  int st = check_common(dtype, B, T, H, K, q, k_norm, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs);
  if (st != CCQ_OK) return st;
  if (T > 0 && (dq_clean == nullptr || dq == nullptr || dk == nullptr || norm_aux == nullptr))
    return fail(CCQ_ERR_INVALID, "dq_clean, norm_aux, dq and dk are required");
  if (lambda_mode == CCQ_LAMBDA_GATE && (dgate_w == nullptr || dgate_b == nullptr))
    return fail(CCQ_ERR_INVALID, "dgate_w and dgate_b are required in GATE mode");
  ccq::CleanArgs a = base_args(dtype, B, T, H, K, q, k_norm, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs,
                               position_offset, subtract_mean, stream);
  a.qk_norm = 1;
  a.norm_aux_in = norm_aux;
  a.dk_ext = dk_norm;
  a.initial_cov = initial_cov;
  a.initial_mean = initial_mean;
  a.state_cov = state_cov;
  a.state_mean = state_mean;
  a.token_aux_in = token_aux;
  a.dq_clean = dq_clean;
  a.dfinal_cov = dfinal_cov;
  a.dfinal_mean = dfinal_mean;
  a.dq = dq;
  a.dk = dk;
  a.dlam = lambda_mode == CCQ_LAMBDA_TOKEN ? dlam : nullptr;
  a.dgate_w = dgate_w;
  a.dgate_b = dgate_b;
  a.dinitial_cov = initial_cov ? dinitial_cov : nullptr;
  a.dinitial_mean = (initial_mean && (subtract_mean || dfinal_mean)) ? dinitial_mean : nullptr;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return run_bwd(a, "ccq_clean_l2norm_bwd");
}

int ccq_decode_step(int dtype, int B, int T, int H, int K, const void* q, const void* k, int lambda_mode,
                    const void* lam, const float* gate_w, const float* gate_b, const int64_t* cu_seqlens, int n_seqs,
                    int position_offset, int subtract_mean, const float* cov_in, const float* mean_in,
                    float* cov_out, float* mean_out, void* q_clean, void* stream) {
  return ccq_decode_step_l2norm(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs,
                                position_offset, subtract_mean, cov_in, mean_in, cov_out, mean_out, q_clean, nullptr,
                                stream);
}

int ccq_decode_step_l2norm(int dtype, int B, int T, int H, int K, const void* q, const void* k, int lambda_mode,
                           const void* lam, const float* gate_w, const float* gate_b, const int64_t* cu_seqlens,
                           int n_seqs, int position_offset, int subtract_mean, const float* cov_in,
                           const float* mean_in, float* cov_out, float* mean_out, void* q_clean, void* k_norm,
                           void* stream) {
  g_err[0] = 0;
  int st = check_common(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs);
  if (st != CCQ_OK) return st;
  if (K % 4 != 0) return fail(CCQ_ERR_UNSUPPORTED, "decode step needs K %% 4 == 0, got K=%d", K);
  if (cov_out == nullptr) return fail(CCQ_ERR_INVALID, "cov_out is required");
  if (T > 0 && q_clean == nullptr) return fail(CCQ_ERR_INVALID, "q_clean output is required");
  if (((uintptr_t)cov_out | (uintptr_t)cov_in) & 15)
    return fail(CCQ_ERR_INVALID, "cov_in / cov_out must be 16-byte aligned");
  ccq::CleanArgs a = base_args(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs,
                               position_offset, subtract_mean, stream);
  a.cov_in = cov_in;
  a.mean_in = mean_in;
  a.cov_out = cov_out;
  a.mean_out = mean_out;
  a.q_clean = q_clean;
  a.qk_norm = k_norm != nullptr;
  a.k_norm = k_norm;
  int launches = 0;
  cudaError_t e = ccq::decode_step(a, &launches);
  if (e != cudaSuccess) return cuda_fail(e, "ccq_decode_step launch");
  g_path = CCQ_PATH_DECODE;
  g_launches = launches;
  return CCQ_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Backward without allocation: the scratch is a fixed device array of this library, looked up once
// per device with that device current.  The existing ccq_clean_bwd does the validation, dispatch and
// launches; this wrapper only supplies the scratch.
// ------------------------------------------------------------------------------------------------
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[CCQ_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch on the current device.  Looked up on every call (a cheap runtime
// query) rather than cached, so a call made under another context of the device, or after
// cudaDeviceReset, never uses an address from an earlier context.
int noalloc_scratch(void** out, const char* who) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) {
    char what[128];
    snprintf(what, sizeof(what), "%s: cudaGetSymbolAddress of the scratch", who);
    return cuda_fail(e, what);
  }
  *out = p;
  return CCQ_OK;
}

}  // namespace

extern "C" int ccq_noalloc_status(void* stream, int* code) {
  g_err[0] = 0;
  if (code == nullptr) return fail(CCQ_ERR_INVALID, "code is required");
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch, "ccq_noalloc_status");
  if (st != CCQ_OK) return st;
  return read_device_word(scratch, (cudaStream_t)stream, code);
}

extern "C" int ccq_clean_bwd_noalloc(int dtype, int B, int T, int H, int K, const void* q, const void* k,
                                     int lambda_mode, const void* lam, const float* gate_w, const float* gate_b,
                                     const int64_t* cu_seqlens, int n_seqs, int position_offset, int subtract_mean,
                                     const float* initial_cov, const float* initial_mean, const float* state_cov,
                                     const float* state_mean, const float* token_aux, const void* dq_clean,
                                     const float* dfinal_cov, const float* dfinal_mean, void* dq, void* dk,
                                     float* dlam, float* dgate_w, float* dgate_b, float* dinitial_cov,
                                     float* dinitial_mean, void* stream) {
  g_err[0] = 0;
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch, "ccq_clean_bwd_noalloc");
  if (st != CCQ_OK) return st;
  st = ccq_clean_bwd(dtype, B, T, H, K, q, k, lambda_mode, lam, gate_w, gate_b, cu_seqlens, n_seqs, position_offset,
                     subtract_mean, initial_cov, initial_mean, state_cov, state_mean, token_aux, dq_clean, dfinal_cov,
                     dfinal_mean, dq, dk, dlam, dgate_w, dgate_b, dinitial_cov, dinitial_mean, scratch,
                     CCQ_NOALLOC_SCRATCH_BYTES, stream);
  if (st == CCQ_ERR_WORKSPACE) {
    char detail[512];
    snprintf(detail, sizeof(detail), "%s", g_err);
    return fail(CCQ_ERR_WORKSPACE,
                "ccq_clean_bwd_noalloc: the call needs more scratch than the fixed %u bytes (%s); "
                "use ccq_clean_bwd with a workspace",
                (unsigned)CCQ_NOALLOC_SCRATCH_BYTES, detail);
  }
  return st;
}

