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
                   aligned16(a.state_cov) && (a.dfinal_cov == nullptr || aligned16(a.dfinal_cov))))
    return false;
  return device_major() == 10;
}


}  // namespace ccq
