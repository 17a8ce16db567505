// prefill.cu -- placeholder until the tcgen05 prefill kernel lands.
#include "kernels.h"

namespace tle {
size_t prefill_workspace_bytes(int n_tokens, int pos0) {
    (void)n_tokens;
    (void)pos0;
    return 0;
}
cudaError_t launch_prefill(const PrefillArgs&, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace tle
