// Tensor-core causal prefill (tcgen05 / TMEM / TMA). Placeholder until the
// kernel lands: every layer takes the generic path.
#include "tla_internal.h"

namespace tla {
cudaError_t prefill_fast_configure(tla_layer* L) {
  L->fast_prefill = false;
  return cudaSuccess;
}
cudaError_t launch_prefill_fast(const tla_layer*, const void*, const int32_t*, int, int, void*, cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace tla
