// hq_prefill.cu -- tensor-core (tcgen05 / TMEM) W4A16 GEMM for M > 16.
// (Placeholder until the tcgen05 kernel lands: larger M is served by the decode
// kernel 16 rows at a time.)
#include "hq_internal.h"

namespace hq {

size_t prefill_workspace_bytes(int, int, int, int, int) { return 0; }
bool prefill_supported(const GemmArgs&) { return false; }
cudaError_t launch_prefill(const GemmArgs&) { return cudaErrorNotSupported; }

}  // namespace hq
