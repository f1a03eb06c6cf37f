// Dispatch predicate of the tcgen05 paths: bf16 / fp16 activations, K == 128, an sm_100 device.
#include <stdlib.h>
#include <string.h>

#include "args.h"

namespace ccq {

namespace {
int device_major() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 0;
  if (cached[dev] == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
    cached[dev] = major;
  }
  return cached[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

bool tc_supported(const CleanArgs& a, int op) {
  const char* env = getenv("CCQ_B200_FORCE_SIMT");
  if (env && env[0] == '1') return false;
  if (a.dtype != DT_BF16 && a.dtype != DT_F16) return false;
  if (a.K != 128) return false;
  if ((int64_t)a.B * a.T >= (1ll << 31)) return false;
  if (a.q && !(aligned16(a.q) && aligned16(a.k))) return false;
  if (a.q_clean && !aligned16(a.q_clean)) return false;
  if (a.initial_cov && !aligned16(a.initial_cov)) return false;
  if (a.final_cov && !aligned16(a.final_cov)) return false;
  if (op == 1 && !(aligned16(a.dq_clean) && aligned16(a.dq) && aligned16(a.dk) &&
                   aligned16(a.state_cov) && (a.dfinal_cov == nullptr || aligned16(a.dfinal_cov)) &&
                   (a.dk_ext == nullptr || aligned16(a.dk_ext))))
    return false;
  return device_major() == 10;
}


namespace {
constexpr int kLptMaxDocs = 4096;
constexpr int kLptThreads = 1024;

// order[rank] = document, ranks by decreasing length (ties: lower index first).  One CTA; each
// thread ranks its documents against all lengths held in shared memory.
__global__ void __launch_bounds__(kLptThreads) lpt_order_kernel(const int64_t* cu, int n_seqs, int T, int* order) {
  __shared__ int len[kLptMaxDocs];
  for (int d = threadIdx.x; d < n_seqs; d += kLptThreads) {
    int64_t a = cu[d], b = cu[d + 1];
    a = a < 0 ? 0 : (a > T ? T : a);
    b = b < a ? a : (b > T ? T : b);
    len[d] = (int)(b - a);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < n_seqs; d += kLptThreads) {
    const int ld = len[d];
    int rank = 0;
    for (int e = 0; e < n_seqs; ++e) {
      const int le = len[e];
      rank += (le > ld) || (le == ld && e < d);
    }
    order[rank] = d;
  }
}
}  // namespace

size_t lpt_order_bytes(int n_seqs, bool varlen) {
  if (!varlen || n_seqs < 2 || n_seqs > kLptMaxDocs) return 0;
  return ws_align(sizeof(int) * (size_t)n_seqs);
}

cudaError_t lpt_order(const CleanArgs& a, int* order, int* launches) {
  lpt_order_kernel<<<1, kLptThreads, 0, a.stream>>>(a.cu_seqlens, a.n_seqs, a.T, order);
  *launches += 1;
  return cudaGetLastError();
}

}  // namespace ccq
