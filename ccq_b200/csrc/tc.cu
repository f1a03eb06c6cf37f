// tcgen05 / TMA tensor-core path (bf16 / fp16, K == 128): not built yet.
#include "args.h"

namespace ccq {
bool tc_supported(const CleanArgs&, int) { return false; }
size_t tc_fwd_workspace(int, int, int, int, int) { return 0; }
size_t tc_bwd_workspace(int, int, int, int, int) { return 0; }
cudaError_t tc_fwd(const CleanArgs&, int*) { return cudaErrorNotSupported; }
cudaError_t tc_bwd(const CleanArgs&, int*) { return cudaErrorNotSupported; }
}  // namespace ccq
