// sm_100a decode kernel (score + split-K attention over TMA-staged pages).
// Placeholder until the specialised kernel lands: reports every shape as unsupported so the
// shape-general kernels serve all calls.
#include "rkv_kernels.h"

namespace rkv {

bool fused_supported(int, int, int, int, int64_t, int64_t, int64_t, int64_t, int64_t,
                     const void*, const void*) {
    return false;
}

size_t fused_workspace_bytes(int64_t, int, int) { return 0; }

cudaError_t launch_fused(const FusedParams&, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace rkv
