// vcb_quantize_qk_static: the Q/K quantiser with its scratch memory inside
// the library, for callers that cannot allocate device memory.
//
// Who needs it: code that calls this library from a place where device
// allocation is not allowed or not possible, for example an inference
// runtime's plugin enqueue hook (the runtime plans all device memory ahead
// of time, and a cudaMalloc there would synchronise the device and break that
// plan), or a host program that drives the GPU through a fixed memory pool it
// does not let third-party code grow.  vcb_quantize_qk needs a small
// workspace for the per-head K channel mean; this variant takes it from a
// fixed array compiled into libvcb.so instead of from the caller.
//
// The array is kScratchBytes (8 MiB) of device memory on every GPU that
// loads the library, held until the process exits.  A call needs
// vcb_qk_workspace(heads, sk) bytes of it (heads * (1 + ceil(sk / 256)) * 512
// bytes when k_smooth is set, none otherwise); larger calls are rejected with
// VCB_ERR_INVALID_ARGUMENT before any work is queued.  All calls share the
// one array: calls that overlap on the GPU (different streams, or different
// host threads without ordering) race on it.  Nothing in it needs to start at
// zero: every byte a call reads was written earlier by the same call.
//
// The device address of the array is looked up with cudaGetSymbolAddress the
// first time the entry point runs on a device, with that device current; that
// first call on each device should therefore come before any stream capture.
#include <mutex>

#include "vcb_internal.h"

namespace vcb {
namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_qk_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of g_qk_scratch on the current device (looked up once).
int scratch_address(void** out) {
    int dev = 0;
    VCB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(VCB_ERR_INVALID_ARGUMENT, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_qk_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_qk_scratch)");
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return VCB_OK;
}

}  // namespace
}  // namespace vcb

using namespace vcb;

extern "C" VCB_API int vcb_quantize_qk_static(const vcb_qk_args* args, void* stream) {
    VCB_REQUIRE(args, "null argument struct");
    VCB_REQUIRE(args->heads > 0 && args->sk > 0, "heads and sk must be positive");
    const size_t need = args->k_smooth ? qk_workspace_bytes(args->heads, args->sk) : 0;
    VCB_REQUIRE(need <= kScratchBytes,
                "vcb_quantize_qk_static supports at most %zu bytes of scratch; heads=%lld sk=%lld needs %zu "
                "(use vcb_quantize_qk with a caller workspace)",
                kScratchBytes, (long long)args->heads, (long long)args->sk, need);
    vcb_qk_args a = *args;
    int rc = require_sm100(nullptr);
    if (rc) return rc;
    void* scratch = nullptr;
    rc = scratch_address(&scratch);
    if (rc) return rc;
    a.workspace = scratch;
    a.workspace_bytes = kScratchBytes;
    return vcb_quantize_qk(&a, stream);
}
