// extern "C" entry points of libvcb.so (declared in include/vcb.h): argument
// checks, workspace carving, error reporting, and the standalone ExpCast
// kernel.  Every check that guards memory safety runs here, before a launch.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "vcb_internal.h"

#define VCB_XSTR(x) #x
#define VCB_STR(x) VCB_XSTR(x)
#define VCB_STR_CUDART VCB_STR(CUDART_VERSION)

namespace vcb {

namespace {
thread_local char g_error[512] = "";
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(VCB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

int require_sm100(int* device_out) {
    int dev = 0;
    VCB_CUDA(cudaGetDevice(&dev));
    int major = 0, minor = 0;
    VCB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    VCB_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0)
        return fail(VCB_ERR_UNSUPPORTED_DEVICE,
                    "libvcb targets B200 (sm_100a, compute capability 10.0); device %d is %d.%d", dev, major,
                    minor);
    if (device_out) *device_out = dev;
    return VCB_OK;
}

// ExpCast bytes: one FP32 FMA, round to nearest even, clamp to [0, 120]
// (the contract of core.py:60-68; the Hopper kernel is kernels.cu:61-70).
__global__ void expcast_kernel(const float* __restrict__ x, uint8_t* __restrict__ y, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)blockDim.x * gridDim.x) {
        const float u = __fmaf_rn(x[i], 11.541560173034668f, 119.6500015258789f);
        y[i] = (uint8_t)__float2int_rn(fminf(120.0f, fmaxf(0.0f, u)));
    }
}

int expcast_run(const float* x, uint8_t* codes, int64_t n, cudaStream_t st) {
    if (n == 0) return VCB_OK;
    const int64_t blocks = (n + 255) / 256;
    expcast_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, st>>>(x, codes, n);
    VCB_CUDA(cudaGetLastError());
    return VCB_OK;
}

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_qk(const vcb_qk_args* a, bool quantise) {
    VCB_REQUIRE(a, "null argument struct");
    VCB_REQUIRE(a->q && a->k, "q and k must be non-null");
    VCB_REQUIRE(a->dtype >= VCB_F32 && a->dtype <= VCB_BF16, "dtype must be 0 (fp32), 1 (fp16) or 2 (bf16)");
    VCB_REQUIRE(a->heads > 0 && a->sq > 0 && a->sk > 0, "heads, sq and sk must be positive");
    VCB_REQUIRE(a->d >= 1 && a->d <= 128, "head dimension must be in [1, 128]");
    VCB_REQUIRE(a->sq < (1ll << 31) && a->sk < (1ll << 31) && a->heads < 65536, "sizes exceed the int32 grid");
    if (a->d == 128) VCB_REQUIRE(aligned16(a->q) && aligned16(a->k), "q and k must be 16-byte aligned");
    if (a->k_smooth) {
        VCB_REQUIRE(a->workspace, "k_smooth needs a workspace");
        VCB_REQUIRE(a->workspace_bytes >= qk_workspace_bytes(a->heads, a->sk), "workspace too small");
    }
    if (quantise) {
        VCB_REQUIRE(a->q8 && a->k8 && a->q_scale && a->k_scale, "quantised outputs must be non-null");
        VCB_REQUIRE(aligned16(a->q8) && aligned16(a->k8), "q8 and k8 must be 16-byte aligned");
        VCB_REQUIRE(a->q_block >= 1 && a->q_block <= 4096, "q_block must be in [1, 4096]");
        VCB_REQUIRE(a->k_quant_block >= 1 && a->k_quant_block <= 4096, "k_quant_block must be in [1, 4096]");
        VCB_REQUIRE((a->q_block % 32 == 0 || a->q_block < 32) && (a->k_quant_block % 32 == 0 || a->k_quant_block < 32),
                    "quantisation blocks must be multiples of 32");
    } else {
        VCB_REQUIRE(a->q_out && a->k_out, "q_out and k_out must be non-null");
    }
    return VCB_OK;
}

int check_attn(const vcb_attn_args* a) {
    VCB_REQUIRE(a, "null argument struct");
    VCB_REQUIRE(a->q8 && a->k8 && a->v8 && a->q_scale && a->k_scale && a->v_meta && a->out,
                "operands must be non-null");
    VCB_REQUIRE(a->heads > 0 && a->sq > 0 && a->sk > 0 && a->heads < 65536, "invalid sizes");
    VCB_REQUIRE(a->sq < (1ll << 31) && a->sk < (1ll << 31), "sequence too long");
    VCB_REQUIRE(a->dv >= 1 && a->dv <= 128, "value dimension must be in [1, 128]");
    VCB_REQUIRE(a->kv_block == 128, "kv_block must be 128");
    VCB_REQUIRE(a->q_block >= 1 && a->q_block <= 4096, "q_block must be in [1, 4096]");
    VCB_REQUIRE(a->k_quant_block >= 128 && a->k_quant_block <= 4096 && a->k_quant_block % 128 == 0,
                "k_quant_block must be a multiple of kv_block (128), at most 4096");
    VCB_REQUIRE(a->scale > 0.0f && a->scale <= 3.4e38f, "scale must be positive and finite");
    VCB_REQUIRE(a->out_dtype >= VCB_F32 && a->out_dtype <= VCB_BF16, "unknown output dtype");
    VCB_REQUIRE(aligned16(a->q8) && aligned16(a->k8) && aligned16(a->v8) && aligned16(a->v_meta),
                "operands must be 16-byte aligned");
    return VCB_OK;
}

}  // namespace
}  // namespace vcb

using namespace vcb;

namespace vcb {
// SMs of the current device, looked up once per device (148 when the
// lookup fails: the value only sizes persistent grids)
int sm_count() {
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}
}  // namespace vcb

extern "C" {

int vcb_abi_version(void) { return VCB_ABI_VERSION; }

int vcb_numerical_contract_version(void) { return VCB_NUMERICAL_CONTRACT_VERSION; }

const char* vcb_build_info(void) {
    return "{\"target\": \"sm_100a\", \"cuda_headers\": " VCB_STR_CUDART
           ", \"matmul\": \"tcgen05.mma kind::f8f6f4, E4M3 x E4M3 -> F32 in TMEM\""
           ", \"fully_fused_attention\": true, \"numerical_contract_version\": 2"
           ", \"expcast_rounding\": \"FP32 FMA then RNE\""
           ", \"value_mean_storage\": \"mu / per-channel V scale at configured mean dtype\""
           ", \"row_mass\": \"FP32 sum of the row's decoded ExpCast P, or of its exp values\"}";
}

size_t vcb_last_error(char* buf, size_t size) {
    const size_t n = strlen(g_error);
    if (buf && size) {
        const size_t c = n < size - 1 ? n : size - 1;
        memcpy(buf, g_error, c);
        buf[c] = 0;
    }
    return n;
}

int vcb_check_device(int device) {
    int count = 0;
    VCB_CUDA(cudaGetDeviceCount(&count));
    VCB_REQUIRE(device >= 0 && device < count, "device %d does not exist (%d devices)", device, count);
    int major = 0, minor = 0;
    VCB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    VCB_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    if (major != 10 || minor != 0)
        return fail(VCB_ERR_UNSUPPORTED_DEVICE, "device %d is compute capability %d.%d; libvcb needs 10.0 (B200)",
                    device, major, minor);
    return VCB_OK;
}

int vcb_expcast_codes(const float* x, uint8_t* codes, int64_t n, void* stream) {
    VCB_REQUIRE(n >= 0, "n must be non-negative");
    VCB_REQUIRE(n == 0 || (x && codes), "x and codes must be non-null");
    int rc = require_sm100(nullptr);
    if (rc) return rc;
    return expcast_run(x, codes, n, static_cast<cudaStream_t>(stream));
}

int64_t vcb_padded_rows(int64_t rows, int block) {
    int64_t a = block, b = 128;
    while (b) { const int64_t t = a % b; a = b; b = t; }
    const int64_t unit = (int64_t)block / a * 128;
    return (rows + unit - 1) / unit * unit;
}

size_t vcb_qk_workspace(int64_t heads, int64_t sk) { return qk_workspace_bytes(heads, sk); }

int vcb_preprocess_qk(const vcb_qk_args* a, void* stream) {
    int rc = check_qk(a, false);
    if (rc) return rc;
    rc = require_sm100(nullptr);
    if (rc) return rc;
    return qk_run(a, false, static_cast<cudaStream_t>(stream));
}

int vcb_quantize_qk(const vcb_qk_args* a, void* stream) {
    int rc = check_qk(a, true);
    if (rc) return rc;
    rc = require_sm100(nullptr);
    if (rc) return rc;
    return qk_run(a, true, static_cast<cudaStream_t>(stream));
}

size_t vcb_group_workspace(int64_t heads, int64_t s, int d, int clusters) {
    return group_workspace_bytes(heads, s, d, clusters);
}

int vcb_group_values(const vcb_group_args* a, void* stream) {
    VCB_REQUIRE(a, "null argument struct");
    VCB_REQUIRE(a->v && a->centers_out && a->pi, "v, centers_out and pi must be non-null");
    VCB_REQUIRE(a->dtype >= VCB_F32 && a->dtype <= VCB_BF16, "unknown dtype");
    VCB_REQUIRE(a->heads > 0 && a->s > 0 && a->s < (1ll << 31) && a->heads < 65536, "invalid heads / tokens");
    VCB_REQUIRE(a->d >= 1 && a->d <= 128, "head dimension must be in [1, 128]");
    VCB_REQUIRE(a->clusters >= 1 && a->clusters <= 32, "clusters must be in [1, 32]");
    VCB_REQUIRE(a->iterations >= 1 && a->iterations <= 1000, "iterations must be in [1, 1000]");
    if (a->d == 128) VCB_REQUIRE(aligned16(a->v), "v must be 16-byte aligned");
    VCB_REQUIRE(a->workspace && a->workspace_bytes >= group_workspace_bytes(a->heads, a->s, a->d, a->clusters),
                "workspace too small (%zu bytes needed)", group_workspace_bytes(a->heads, a->s, a->d, a->clusters));
    int rc = require_sm100(nullptr);
    if (rc) return rc;
    return group_run(a, static_cast<cudaStream_t>(stream));
}

int vcb_prepare_v(const vcb_v_args* a, void* stream) {
    VCB_REQUIRE(a, "null argument struct");
    VCB_REQUIRE(a->v && a->v8 && a->v_meta, "v, v8 and v_meta must be non-null");
    VCB_REQUIRE(a->dtype >= VCB_F32 && a->dtype <= VCB_BF16, "unknown dtype");
    VCB_REQUIRE(a->heads > 0 && a->s > 0 && a->s < (1ll << 31) && a->heads < 65536, "invalid heads / tokens");
    VCB_REQUIRE(a->dv >= 1 && a->dv <= 128, "value dimension must be in [1, 128]");
    VCB_REQUIRE(a->kv_block == 128, "kv_block must be 128");
    VCB_REQUIRE(a->mean_type >= 0 && a->mean_type <= 2, "mean_type must be 0, 1 or 2");
    VCB_REQUIRE(aligned16(a->v8), "v8 must be 16-byte aligned");
    int rc = require_sm100(nullptr);
    if (rc) return rc;
    return vprep_run(a, static_cast<cudaStream_t>(stream));
}

int vcb_attention_fp8_probe(const vcb_attn_args* a, const vcb_attn_probe* pr, void* stream) {
    VCB_REQUIRE(pr, "null probe struct");
    VCB_REQUIRE(pr->logits && pr->codes && pr->rowstat, "probe buffers must be non-null");
    int rc = check_attn(a);
    if (rc) return rc;
    VCB_REQUIRE(pr->head >= 0 && pr->head < a->heads, "probe head out of range");
    VCB_REQUIRE(pr->q_tile >= 0 && pr->q_tile < (a->sq + 127) / 128, "probe query tile out of range");
    VCB_REQUIRE(pr->tile_begin >= 0 && pr->tile_count >= 1 &&
                    (int64_t)pr->tile_begin + pr->tile_count <= (a->sk + 127) / 128,
                "probe KV tiles out of range");
    VCB_REQUIRE((reinterpret_cast<uintptr_t>(pr->codes) & 3u) == 0, "probe codes must be 4-byte aligned");
    rc = require_sm100(nullptr);
    if (rc) return rc;
    return attn_run(a, pr, static_cast<cudaStream_t>(stream));
}

int vcb_attention_fp8(const vcb_attn_args* a, void* stream) {
    int rc = check_attn(a);
    if (rc) return rc;
    rc = require_sm100(nullptr);
    if (rc) return rc;
    return attn_run(a, nullptr, static_cast<cudaStream_t>(stream));
}

// Workspace of vcb_forward, carved in this order (256-byte aligned pieces):
// q8, k8, q_scale, k_scale, v8, v_meta, the V-mean operand (V-Smooth in the
// exp modes only: the ExpCast kernel reads the means from v_meta), then the
// Q/K-prep scratch.
namespace {
struct ForwardLayout {
    size_t q8, k8, qs, ks, v8, vm, mop, qk, total;
};
ForwardLayout forward_layout(const vcb_forward_args* a) {
    auto r = [](size_t b) { return (b + 255) & ~size_t(255); };
    ForwardLayout L{};
    const int64_t sq_pad = vcb_padded_rows(a->sq, a->q_block);
    const int64_t sk_pad = vcb_padded_rows(a->sk, a->k_quant_block);
    const int64_t T = (a->sk + 127) / 128;
    size_t o = 0;
    L.q8 = o; o += r((size_t)(a->heads * sq_pad * 128));
    L.k8 = o; o += r((size_t)(a->heads * sk_pad * 128));
    L.qs = o; o += r((size_t)(a->heads * ((a->sq + a->q_block - 1) / a->q_block)) * 4);
    L.ks = o; o += r((size_t)(a->heads * ((a->sk + a->k_quant_block - 1) / a->k_quant_block)) * 4);
    L.v8 = o; o += r((size_t)(a->heads * T * 128 * 128));
    L.vm = o; o += r((size_t)(a->heads * T * 256) * 4);
    L.mop = o; o += (a->smooth && !a->expcast) ? r((size_t)(a->heads * T * 128 * 16) * 2) : 0;
    L.qk = o; o += r(qk_workspace_bytes(a->heads, a->sk));
    L.total = o;
    return L;
}
}  // namespace

size_t vcb_forward_workspace(const vcb_forward_args* a) {
    if (!a || a->heads <= 0 || a->sq <= 0 || a->sk <= 0 || a->q_block <= 0 || a->k_quant_block <= 0) return 0;
    return forward_layout(a).total;
}

int vcb_forward(const vcb_forward_args* a, void* stream) {
    VCB_REQUIRE(a, "null argument struct");
    VCB_REQUIRE(a->q && a->k && a->v && a->out, "q, k, v and out must be non-null");
    VCB_REQUIRE(a->dtype >= VCB_F32 && a->dtype <= VCB_BF16, "unknown dtype");
    VCB_REQUIRE(a->q_block >= 32 && a->q_block <= 256 && a->q_block % 32 == 0,
                "q_block must be a multiple of 32 in [32, 256]");
    VCB_REQUIRE(a->kv_block == 128, "kv_block must be 128");
    VCB_REQUIRE(a->k_quant_block >= 128 && a->k_quant_block <= 4096 && a->k_quant_block % 128 == 0,
                "k_quant_block must be a multiple of kv_block (128), at most 4096");
    VCB_REQUIRE(a->mean_type >= 0 && a->mean_type <= 2, "mean_type must be 0, 1 or 2");
    VCB_REQUIRE(a->workspace, "workspace must be non-null");
    const ForwardLayout L = forward_layout(a);
    if (a->workspace_bytes < L.total)
        return fail(VCB_ERR_WORKSPACE, "workspace too small: %zu bytes, need %zu", a->workspace_bytes, L.total);
    VCB_REQUIRE(aligned16(a->workspace), "workspace must be 16-byte aligned");
    int rc = require_sm100(nullptr);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    char* ws = static_cast<char*>(a->workspace);
    if (a->status) VCB_CUDA(cudaMemsetAsync(a->status, 0, sizeof(int32_t), st));

    vcb_qk_args qk{};
    qk.q = a->q; qk.k = a->k; qk.dtype = a->dtype; qk.heads = a->heads; qk.sq = a->sq; qk.sk = a->sk;
    qk.d = a->d; qk.pi = a->pi; qk.k_smooth = a->k_smooth; qk.hadamard = a->hadamard;
    qk.q_block = a->q_block; qk.k_quant_block = a->k_quant_block;
    qk.q8 = reinterpret_cast<uint8_t*>(ws + L.q8); qk.k8 = reinterpret_cast<uint8_t*>(ws + L.k8);
    qk.q_scale = reinterpret_cast<float*>(ws + L.qs); qk.k_scale = reinterpret_cast<float*>(ws + L.ks);
    qk.status = a->status; qk.workspace = ws + L.qk; qk.workspace_bytes = L.total - L.qk;
    rc = check_qk(&qk, true);
    if (rc) return rc;

    vcb_v_args va{};
    va.v = a->v; va.dtype = a->dtype; va.heads = a->heads; va.s = a->sk; va.dv = a->dv; va.pi = a->pi;
    va.active = a->smooth; va.mean_type = a->mean_type; va.kv_block = a->kv_block;
    va.v8 = reinterpret_cast<uint8_t*>(ws + L.v8); va.v_meta = reinterpret_cast<float*>(ws + L.vm);
    va.v_mean_op = (a->smooth && !a->expcast) ? reinterpret_cast<uint16_t*>(ws + L.mop) : nullptr;
    va.status = a->status;
    VCB_REQUIRE(a->dv >= 1 && a->dv <= 128, "value dimension must be in [1, 128]");

    vcb_attn_args at{};
    at.q8 = qk.q8; at.q_scale = qk.q_scale; at.k8 = qk.k8; at.k_scale = qk.k_scale;
    at.v8 = va.v8; at.v_meta = va.v_meta; at.v_mean_op = va.v_mean_op; at.heads = a->heads; at.sq = a->sq; at.sk = a->sk; at.dv = a->dv;
    at.q_block = a->q_block; at.k_quant_block = a->k_quant_block; at.kv_block = a->kv_block;
    at.expcast = a->expcast; at.has_mean = a->smooth; at.scale = a->scale; at.out = a->out;
    at.out_dtype = a->dtype; at.status = a->status;
    VCB_REQUIRE(a->scale > 0.0f && a->scale <= 3.4e38f, "scale must be positive and finite");

    rc = qk_run(&qk, true, st);
    if (rc) return rc;
    rc = vprep_run(&va, st);
    if (rc) return rc;
    return attn_run(&at, nullptr, st);
}

int vcb_wait_selftest(int complete, const void* src, int32_t* status, int32_t* report, void* stream) {
    VCB_REQUIRE(src && report, "src and report must be non-null");
    VCB_REQUIRE(aligned16(src), "src must be 16-byte aligned");
    int rc = require_sm100(nullptr);
    if (rc) return rc;
    return wait_selftest_run(complete, src, status, report, static_cast<cudaStream_t>(stream));
}

// The copy is ordered on the caller's stream only (no legacy default stream,
// no device-wide synchronisation); the host then waits for that stream.
int vcb_read_status(const int32_t* status, void* stream, int32_t* flags) {
    VCB_REQUIRE(status && flags, "status and flags must be non-null");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t word = 0;
    VCB_CUDA(cudaMemcpyAsync(&word, status, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    VCB_CUDA(cudaStreamSynchronize(st));
    *flags = word;
    return VCB_OK;
}

}  // extern "C"
