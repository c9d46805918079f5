// Decode attention for callers that cannot allocate device memory.
//
// rkv_decode_attention needs a caller-provided workspace for its split-K partials.  Some
// callers have no way to provide one at call time: code running inside a host framework
// that owns the whole device heap and forbids allocations outside its arena, or a serving
// loop that must not take the driver's allocation path (which can synchronise the device)
// between two decode steps.  rkv_decode_attention_noalloc serves them from a fixed scratch
// array compiled into this library instead.
//
// The array below is a file-scope device variable: every GPU that loads the library holds
// RKV_NOALLOC_SCRATCH_BYTES of it until the process exits.  Host code cannot use the array's
// name as a device address (on the host it names a host-side stand-in), so the first call on
// each device looks up the real device address with cudaGetSymbolAddress while that device is
// current and keeps it; make that first call before any stream capture.  The array starts
// at zero like every device variable, and the decode kernels leave the cross-CTA counters in
// its header at zero when they finish, so nothing is cleared between calls and consecutive
// calls overlap a launch's start with the previous one's tail exactly as
// rkv_decode_attention with a caller workspace does.  The array is shared by every call on
// the device: calls whose kernels overlap on the GPU (different streams, or different host
// threads) race on it; serialise them.
//
// Device-side errors are not reported here.  The decode kernels record a bounded wait that
// gave up, or a page id outside the storage, in the error flag inside the scratch array,
// which no entry point reads back.  A caller that needs those errors uses
// rkv_decode_attention with a workspace it can read (its first int32, at
// rkv_workspace_error_flag_offset()).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/razorkv_b200.h"

namespace rkv {
int attention_args_status(const rkv_query* q, const rkv_kv_layout* kv, const rkv_output* out);
}

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[RKV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return RKV_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return RKV_ERR_CUDA;
        g_ptr[dev] = p;
    }
    *out = g_ptr[dev];
    return RKV_OK;
}

}  // namespace

extern "C" int rkv_decode_attention_noalloc(const rkv_query* q, const rkv_kv_layout* kv,
                                            float scale, int causal, const rkv_output* out,
                                            void* stream) {
    // reject a bad call before anything is queued
    int st = rkv::attention_args_status(q, kv, out);
    if (st) return st;
    if (kv->batch == 0) return RKV_OK;
    const size_t need = rkv_decode_attention_workspace_size(q, kv);
    if (need > (size_t)RKV_NOALLOC_SCRATCH_BYTES) return RKV_ERR_WORKSPACE_TOO_SMALL;
    void* ws = nullptr;
    st = scratch_address(&ws);
    if (st) return st;
    return rkv_decode_attention(q, kv, scale, causal, out, ws, (size_t)RKV_NOALLOC_SCRATCH_BYTES,
                                stream);
}
