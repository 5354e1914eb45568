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
// The address is remembered together with the identity of the CUDA context it
// was looked up in.  If the process resets the device (cudaDeviceReset) and a
// new context loads the library's module again, possibly at another address,
// the next call sees a different context and looks the address up again
// instead of handing the kernels a stale pointer.
#include <mutex>

#include "vcb_internal.h"

namespace vcb {
namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_qk_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchEntry {
    void* ptr;
    unsigned long long ctx_id;     // identity of the context the address belongs to
};
ScratchEntry g_scratch[kMaxDevices] = {};
std::mutex g_scratch_mutex;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Process-unique identity of the current CUDA context (cuCtxGetId, CUDA 12.0);
// 0 when the thread has no current context yet.
int current_context_id(unsigned long long* id) {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    if (!get_current || !get_id) {
        void* a = nullptr;
        void* b = nullptr;
        cudaDriverEntryPointQueryResult qa, qb;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa) != cudaSuccess ||
            qa != cudaDriverEntryPointSuccess || !a ||
            cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb) != cudaSuccess ||
            qb != cudaDriverEntryPointSuccess || !b)
            return fail(VCB_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are not available from the driver");
        get_current = reinterpret_cast<CtxGetCurrentFn>(a);
        get_id = reinterpret_cast<CtxGetIdFn>(b);
    }
    CUcontext ctx = nullptr;
    *id = 0;
    if (get_current(&ctx) != CUDA_SUCCESS) return fail(VCB_ERR_CUDA, "cuCtxGetCurrent failed");
    if (ctx && get_id(ctx, id) != CUDA_SUCCESS) return fail(VCB_ERR_CUDA, "cuCtxGetId failed");
    return VCB_OK;
}

// Device address of g_qk_scratch on the current device, looked up once per
// device and context (cudaGetSymbolAddress also makes the device's primary
// context current when the thread has none yet).
int scratch_address(void** out) {
    int dev = 0;
    VCB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(VCB_ERR_INVALID_ARGUMENT, "device ordinal %d out of range", dev);
    unsigned long long ctx = 0;
    int rc = current_context_id(&ctx);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchEntry& e = g_scratch[dev];
    if (!e.ptr || ctx == 0 || e.ctx_id != ctx) {
        void* p = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&p, g_qk_scratch);
        if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(g_qk_scratch)");
        rc = current_context_id(&ctx);
        if (rc) return rc;
        e.ptr = p;
        e.ctx_id = ctx;
    }
    *out = e.ptr;
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
