/*
 * vcb.h - C ABI of the B200 (sm_100a) VC-Attention forward path.
 *
 * This library replaces the pybind11 extension of czfsdg/vc-attention
 * (csrc/bindings.cpp, PYBIND11_MODULE at bindings.cpp:231-248) with plain C
 * entry points: pointers, sizes and a CUDA stream, no torch types.  Every
 * buffer (inputs, outputs, scratch) belongs to the caller; the library
 * allocates no device memory and keeps no per-call state.  All work is
 * enqueued on the stream the caller passes (bindings.cpp:176 uses the
 * current PyTorch stream the same way); nothing synchronises the device,
 * and only vcb_read_status waits for the caller's stream.
 *
 * The kernels are launched with programmatic stream serialisation, and each
 * waits for the stream's previous grid (griddepcontrol.wait) before it reads
 * or writes anything.  Work the caller queues after a call is ordered as
 * usual, except a kernel of the caller's own launched with that attribute:
 * like any dependent grid, it must wait (griddepcontrol.wait or
 * cudaGridDependencySynchronize) before it reads the call's outputs.
 *
 * Tensors are contiguous, batch and heads flattened: [heads, tokens, dim].
 * Functions return VCB_OK or a VCB_ERR_* code; vcb_last_error() gives the
 * message of the last failure on the calling thread.
 */
#ifndef VCB_H
#define VCB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VCB_API __attribute__((visibility("default")))
#else
#define VCB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define VCB_ABI_VERSION 2
#define VCB_NUMERICAL_CONTRACT_VERSION 2   /* bindings.cpp:232 */

enum vcb_status {
    VCB_OK = 0,
    VCB_ERR_INVALID_ARGUMENT = 1,   /* shape, geometry, pointer or alignment */
    VCB_ERR_UNSUPPORTED_DEVICE = 2, /* device is not compute capability 10.0 */
    VCB_ERR_CUDA = 3,               /* a CUDA runtime or driver call failed */
    VCB_ERR_WORKSPACE = 4           /* workspace smaller than required */
};

enum vcb_dtype { VCB_F32 = 0, VCB_F16 = 1, VCB_BF16 = 2 };

/* Bits of the device status word that kernels set (see vcb_read_status). */
enum vcb_device_flags {
    VCB_FLAG_NONFINITE = 1,         /* a Q, K or V element was NaN or Inf */
    VCB_FLAG_TIMEOUT = 2,           /* a bounded wait in the attention kernel (or vcb_wait_selftest) expired */
    VCB_FLAG_INTERNAL = 4           /* a device-side layout check failed; nothing was computed */
};

/* ---- identification --------------------------------------------------- */
VCB_API int vcb_abi_version(void);
/* replaces the module attribute numerical_contract_version (bindings.cpp:232) */
VCB_API int vcb_numerical_contract_version(void);
/* replaces build_info() (bindings.cpp:237-247); returns a static JSON string */
VCB_API const char* vcb_build_info(void);
/* copies the last error message of this thread into buf; returns its length */
VCB_API size_t vcb_last_error(char* buf, size_t size);
/* VCB_OK when `device` is compute capability 10.0 (sm_100), else an error */
VCB_API int vcb_check_device(int device);

/* ---- ExpCast bytes ------------------------------------------------------ */
/* replaces expcast_codes(x) (bindings.cpp:219-227; kernel kernels.cu:61-70):
 * codes[i] = rne(clamp(fmaf(x[i], 11.541560173034668f, 119.6500015258789f), 0, 120)) */
VCB_API int vcb_expcast_codes(const float* x, uint8_t* codes, int64_t n, void* stream);

/* ---- Q/K preprocessing ---------------------------------------------------- */
typedef struct {
    const void* q;          /* [heads, sq, d]  dtype */
    const void* k;          /* [heads, sk, d]  dtype */
    int dtype;              /* vcb_dtype */
    int64_t heads, sq, sk;
    int d;                  /* 1..128 */
    const int32_t* pi;      /* [heads, sk] K row permutation, or NULL */
    int k_smooth;           /* subtract the per-head K channel mean */
    int hadamard;           /* normalised Sylvester transform, width = next pow2 >= d */
    /* transform-only outputs (vcb_preprocess_qk): float [heads, s, width] */
    float* q_out;
    float* k_out;
    /* quantised outputs (vcb_quantize_qk) */
    int q_block, k_quant_block;
    uint8_t* q8;            /* [heads, sq_pad, 128] e4m3, sq_pad = vcb_padded_rows(sq, q_block) */
    uint8_t* k8;            /* [heads, sk_pad, 128] e4m3 */
    float* q_scale;         /* [heads, ceil(sq / q_block)] */
    float* k_scale;         /* [heads, ceil(sk / k_quant_block)] */
    int32_t* status;        /* device status word (nullable) */
    void* workspace;
    size_t workspace_bytes;
} vcb_qk_args;

/* rows of a payload buffer: whole quantisation blocks and whole 128-row tiles */
VCB_API int64_t vcb_padded_rows(int64_t rows, int block);
VCB_API size_t vcb_qk_workspace(int64_t heads, int64_t sk);
/* replaces preprocess_qk(q, k, k_smooth, hadamard) (bindings.cpp:68-98):
 * writes q_out / k_out only */
VCB_API int vcb_preprocess_qk(const vcb_qk_args* args, void* stream);
/* demean + Hadamard + block E4M3 quantisation in one pass (replaces
 * kernels.cu:72-120, launched at kernels.cu:307-310): writes q8/k8/scales */
VCB_API int vcb_quantize_qk(const vcb_qk_args* args, void* stream);

/* Same work and outputs as vcb_quantize_qk, for callers that cannot allocate
 * device memory (for example a runtime's plugin enqueue hook, where the
 * runtime has planned all device memory and a cudaMalloc would synchronise
 * the device).  args->workspace is ignored: the K-mean scratch comes from a
 * fixed 8 MiB array inside libvcb.so, held on every GPU that loads the
 * library.  Calls needing more than 8 MiB (heads * (1 + ceil(sk / 256)) * 512
 * bytes with k_smooth) fail with VCB_ERR_INVALID_ARGUMENT.  All calls share
 * the array, so calls that overlap on the GPU race.  The first call on a
 * device looks up the array's address and should come before any stream
 * capture; after a device reset the first call in the new context looks it
 * up again.  This entry point has no counterpart in the reference. */
VCB_API int vcb_quantize_qk_static(const vcb_qk_args* args, void* stream);

/* ---- V clustering (Lloyd + stable permutation) ---------------------------- */
typedef struct {
    const void* v;          /* [heads, s, d] dtype */
    int dtype;
    int64_t heads, s;
    int d;                  /* 1..128 */
    int clusters;           /* 1..32; count = min(clusters, s) */
    int iterations;         /* >= 1 */
    const float* centers_in;/* [heads, count, d] warm start, or NULL for equispaced init */
    float* centers_out;     /* [heads, count, d] */
    int32_t* pi;            /* [heads, s] stable argsort of the final labels */
    void* workspace;
    size_t workspace_bytes;
} vcb_group_args;

VCB_API size_t vcb_group_workspace(int64_t heads, int64_t s, int d, int clusters);
/* replaces group_values(v, clusters, iterations, centers) (bindings.cpp:182-217) */
VCB_API int vcb_group_values(const vcb_group_args* args, void* stream);

/* ---- V tiles ------------------------------------------------------------- */
typedef struct {
    const void* v;          /* [heads, s, dv] dtype */
    int dtype;
    int64_t heads, s;
    int dv;                 /* 1..128 */
    const int32_t* pi;      /* [heads, s] or NULL */
    int active;             /* subtract the block mean (V-Smooth window) */
    int mean_type;          /* 0 fp32, 1 fp16, 2 bf16 (cuda_backend.py:52 encoding) */
    int kv_block;           /* 128 */
    uint8_t* v8;            /* [heads, T, 128 channels, kv_block tokens] e4m3 residual */
    float* v_meta;          /* [heads, T, 2, 128]: vscale, then mu/vscale at mean_type */
    uint16_t* v_mean_op;    /* [heads, T, 128, 16] bf16, written when active (nullable): per channel the
                               stored mean mu/vscale as bf16 pieces u1 + u2 + u3 (u1 truncated, u2 and u3
                               rounded remainders) in the row [u1, u2, u3, u1, u2, u1, 0 x 10], the B
                               operand of the exp-mode attention kernel's row-mass x mean MMA */
    int32_t* status;        /* device status word (nullable) */
} vcb_v_args;

/* replaces prepare_values (kernels.cu:124-162, launch kernels.cu:311-312) and
 * the V gather of cuda_backend.py:51 */
VCB_API int vcb_prepare_v(const vcb_v_args* args, void* stream);

/* ---- fused attention over prepared operands ------------------------------- */
typedef struct {
    const uint8_t* q8; const float* q_scale;
    const uint8_t* k8; const float* k_scale;
    const uint8_t* v8; const float* v_meta;
    const uint16_t* v_mean_op;  /* vcb_v_args.v_mean_op; required when has_mean and not expcast (the
                                   ExpCast kernel takes mu / vscale from v_meta) */
    int64_t heads, sq, sk;
    int dv;
    int q_block, k_quant_block, kv_block;
    int expcast;
    int has_mean;           /* v_meta carries non-zero block means (V-Smooth active) */
    float scale;            /* softmax scale, positive finite */
    void* out;              /* [heads, sq, dv] */
    int out_dtype;          /* vcb_dtype */
    int32_t* status;        /* device status word (nullable) */
} vcb_attn_args;

/* replaces the host tile loop of kernels.cu:313-330 (two cuBLASLt FP8 GEMMs
 * and four SIMT kernels per tile pair) with one warp-specialised tcgen05
 * kernel: TMA-staged E4M3 tiles, S and PV accumulators in tensor memory,
 * online softmax with ExpCast and V-mean recovery, output in out_dtype */
VCB_API int vcb_attention_fp8(const vcb_attn_args* args, void* stream);

/* Diagnostic dump of the fused kernel's softmax for one (head, 128-row query
 * tile): KV tiles [tile_begin, tile_begin + tile_count) of that CTA write the
 * raw FP32 logits s = q8 . k8 (masked keys of a ragged last tile as -inf),
 * the 128 P bytes per row exactly as the PV MMA reads them (ExpCast codes, or
 * E4M3(exp * 256)), and per row: the running max m after the tile, the
 * encode's slope A and offset B (P = rne(fma(s, A, B) * 2^24) with ExpCast,
 * in units of 2^-24), and the rescale factor alpha.  The attention itself
 * runs in full as in vcb_attention_fp8.  Used by the tests to count the
 * ExpCast bytes that differ from the reference's FP64-intermediate encode of
 * (S - m) (core.py:60-68, :326-328); no reference counterpart. */
typedef struct {
    int64_t head, q_tile;
    int tile_begin, tile_count;
    float* logits;          /* [tile_count, 128, 128] */
    uint8_t* codes;         /* [tile_count, 128, 128] */
    float* rowstat;         /* [tile_count, 128, 4]: m, A, B, alpha */
} vcb_attn_probe;

VCB_API int vcb_attention_fp8_probe(const vcb_attn_args* args, const vcb_attn_probe* probe, void* stream);

/* ---- whole forward ----------------------------------------------------------- */
typedef struct {
    const void* q; const void* k; const void* v;
    int dtype;
    int64_t heads, sq, sk;
    int d, dv;
    const int32_t* pi;      /* [heads, sk] or NULL */
    int q_block, k_quant_block, kv_block;
    int smooth;             /* V-Smooth demean active */
    int expcast;
    int mean_type;
    float scale;
    int k_smooth, hadamard;
    void* out;              /* [heads, sq, dv] dtype */
    void* workspace;
    size_t workspace_bytes;
    int32_t* status;        /* device status word (nullable); zeroed by the call */
} vcb_forward_args;

VCB_API size_t vcb_forward_workspace(const vcb_forward_args* args);
/* replaces forward(q, k, v, bq, k_quant, bk, smooth, expcast, mean_type,
 * scale, k_smooth, hadamard) (bindings.cpp:100-178) */
VCB_API int vcb_forward(const vcb_forward_args* args, void* stream);

/* Reads the device status word into *flags: one device-to-host copy ordered
 * on `stream` (not on the legacy default stream), then a wait for `stream`
 * only.  The one call of this library that blocks the host. */
VCB_API int vcb_read_status(const int32_t* status, void* stream, int32_t* flags);

/* Self-test of the attention kernel's bounded waits; no reference
 * counterpart (the reference's waits are host-side cuBLASLt calls).  One CTA
 * holds tensor memory and a 1 KB bulk copy of src (device, 16-byte aligned)
 * in flight, and four warps wait on a barrier phase that only `complete`
 * finishes.  Without it every wait gives up after the kernels' 2 s limit; the
 * CTA drains its copy, frees its tensor memory and sets VCB_FLAG_TIMEOUT in
 * *status (nullable), as an attention CTA does.  report: device, 4 x int32,
 * zeroed by the call: waits that gave up, waits that completed, 1 when the
 * drained copy equals src, elapsed milliseconds. */
VCB_API int vcb_wait_selftest(int complete, const void* src, int32_t* status, int32_t* report, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VCB_H */
