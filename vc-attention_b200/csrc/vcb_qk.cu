// Q/K preprocessing for sm_100a: post-RoPE K channel demean, normalised
// Sylvester Hadamard and per-block E4M3 quantisation, fused into one pass per
// quantisation block (reference: core.py:71-99 and :118-135; the Hopper
// extension ran these as kernels.cu:72-120 plus an ATen mean).
//
// Reduction orders are fixed and mirrored by the CPU checker:
//   K mean: chunks of kKsumChunk rows; inside a chunk row r goes to lane
//   r % kKsumLanes, lanes sum their rows in increasing order, the chunk sum
//   adds lanes in order, the head total adds chunks in order, then / S.
#include <type_traits>

#include "vcb_internal.h"

namespace vcb {

constexpr int kKsumChunk = 256;
constexpr int kKsumLanes = 16;

template <typename T>
__global__ void __launch_bounds__(256) k_colsum_kernel(const T* __restrict__ k, int64_t S, int D,
                                                       float* __restrict__ partial, int nchunk) {
    pdl_wait();
    pdl_open();
    __shared__ float part[kKsumLanes][128];
    const int64_t h = blockIdx.y;
    const int chunk = blockIdx.x;
    const int t = threadIdx.x, lane = t / 16, g = t % 16;
    const int64_t base = (int64_t)chunk * kKsumChunk;
    const int64_t end = min(base + (int64_t)kKsumChunk, S);
    const T* kh = k + h * S * D;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    if (D == 128) {
        for (int64_t r = base + lane; r < end; r += kKsumLanes) {
            float x[8];
            load8(kh + r * 128 + 8 * g, x);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] += x[i];
        }
    } else {
        for (int64_t r = base + lane; r < end; r += kKsumLanes) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = 8 * g + i;
                if (c < D) acc[i] += Elem<T>::load(kh + r * D + c);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) part[lane][8 * g + i] = acc[i];
    __syncthreads();
    if (t < 128) {
        float s = 0.0f;
#pragma unroll
        for (int l = 0; l < kKsumLanes; ++l) s += part[l][t];
        partial[((int64_t)h * nchunk + chunk) * 128 + t] = s;
    }
}

__global__ void k_mean_kernel(const float* __restrict__ partial, int nchunk, int64_t S,
                              float* __restrict__ mean) {
    pdl_wait();
    pdl_open();
    const int64_t h = blockIdx.x;
    const int c = threadIdx.x;
    float total = 0.0f;
    for (int ch = 0; ch < nchunk; ++ch) total += partial[((int64_t)h * nchunk + ch) * 128 + c];
    mean[h * 128 + c] = total / (float)S;
}

struct RowArgs {
    const void* x;
    int64_t S;
    int D;
    int width;          // output width: next pow2 >= D with the Hadamard, else D
    int hadamard;
    float norm;         // fp32(width^-0.5)
    const int32_t* pi;  // row permutation or null
    const float* mean;  // [heads, 128] or null
    int block;          // quantisation block rows
    int64_t S_pad;
    int nblk;           // ceil(S / block)
    uint8_t* payload;   // [heads, S_pad, 128]
    float* scales;      // [heads, nblk]
    float* out_f32;     // [heads, S, width] (transform-only mode)
    int32_t* status;
};

// Loads row `r` (through the permutation) and applies demean + Hadamard.
template <typename T>
__device__ __forceinline__ bool transform_row(const RowArgs& a, int64_t h, int64_t r, const float* smean,
                                              float (&x)[128]) {
    const int64_t tok = a.pi ? (int64_t)a.pi[h * a.S + r] : r;
    const T* src = static_cast<const T*>(a.x) + (h * a.S + tok) * a.D;
    bool ok = true;
    if (a.D == 128) {
#pragma unroll
        for (int i = 0; i < 16; ++i) load8(src + 8 * i, x + 8 * i);
    } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) x[c] = c < a.D ? Elem<T>::load(src + c) : 0.0f;
    }
#pragma unroll
    for (int c = 0; c < 128; ++c) ok &= finite_f(x[c]);
    if (smean) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
            if (c < a.D) x[c] = x[c] - smean[c];
    }
    if (a.hadamard) {
        // Butterflies with stride 1, 2, 4, ... (core.py:79-84): (l + r, l - r).
        // Running a stage over the zero-padded 128 array leaves [0, width)
        // exactly the width-point transform and the padding at zero.
#pragma unroll
        for (int s = 1; s < 128; s <<= 1) {
            if (s < a.width) {
#pragma unroll
                for (int base = 0; base < 128; base += 2 * s) {
#pragma unroll
                    for (int t = 0; t < s; ++t) {
                        const float l = x[base + t], rr = x[base + s + t];
                        x[base + t] = l + rr;
                        x[base + s + t] = l - rr;
                    }
                }
            }
        }
#pragma unroll
        for (int c = 0; c < 128; ++c)
            if (c < a.width) x[c] = x[c] * a.norm;
    }
    return ok;
}

// Half-row form used by the quantiser: a lane pair (lane, lane ^ 16) holds
// one row, the lower lane channels [0, 64), the upper lane [64, 128).  The
// butterflies with stride 1..32 stay inside a half; the stride-64 stage
// exchanges halves with one shuffle per element and still computes
// (left + right, left - right) on the same operands.  `tok` is the input row
// (row r through the permutation).
template <typename T>
__device__ __forceinline__ void transform_half(const RowArgs& a, int64_t h, int64_t tok, bool valid, int half,
                                               const float* smean, float (&x)[64]) {
    const int c0 = 64 * half;
    const int D = a.D;
    const int width = a.width;
    const bool hadamard = a.hadamard != 0;
    if (valid) {
        const T* src = static_cast<const T*>(a.x) + (h * a.S + tok) * D;
        if (D == 128) {
#pragma unroll
            for (int i = 0; i < 8; ++i) load8(src + c0 + 8 * i, x + 8 * i);
        } else {
#pragma unroll
            for (int c = 0; c < 64; ++c) x[c] = c0 + c < D ? Elem<T>::load(src + c0 + c) : 0.0f;
        }
        if (smean) {
#pragma unroll
            for (int c = 0; c < 64; ++c)
                if (c0 + c < D) x[c] = x[c] - smean[c0 + c];
        }
    } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] = 0.0f;
    }
    if (hadamard) {
#pragma unroll
        for (int s = 1; s < 64; s <<= 1) {
            if (s < width) {
#pragma unroll
                for (int base = 0; base < 64; base += 2 * s) {
#pragma unroll
                    for (int t = 0; t < s; ++t) {
                        const float l = x[base + t], rr = x[base + s + t];
                        x[base + t] = l + rr;
                        x[base + s + t] = l - rr;
                    }
                }
            }
        }
        if (width > 64) {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const float other = __shfl_xor_sync(0xffffffffu, x[c], 16);
                x[c] = half == 0 ? x[c] + other : other - x[c];
            }
        }
#pragma unroll
        for (int c = 0; c < 64; ++c)
            if (c0 + c < width) x[c] = x[c] * a.norm;
    }
}

// transform_half for D == 128 with the 128-point Hadamard, in packed FP32:
// the half row is 32 channel pairs, and the demean, the butterflies from
// stride 2 on, the stride-64 exchange and the normalisation are add / fma /
// mul .f32x2, each lane rounded once like the scalar form.  l - r is computed
// as fma(r, -1, l): the product is exact, so the result is RN(l - r) with the
// same sign of zero.  hadamard_half128 takes the half row already in x
// (zeros for an invalid row); transform_half128 loads it from global memory.
__device__ __forceinline__ void hadamard_half128(bool valid, int half, const float* smean, float2 (&x)[32]) {
    const int c0 = 64 * half;
    const float2 neg1 = make_float2(-1.0f, -1.0f);
    if (valid && smean) {
        const float2* m2 = reinterpret_cast<const float2*>(smean + c0);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = ffma2(m2[i], neg1, x[i]);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {          // stride 1: inside one pair
        const float l = x[i].x, r = x[i].y;
        x[i] = make_float2(l + r, l - r);
    }
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {      // strides 2 .. 32: s pairs apart
#pragma unroll
        for (int base = 0; base < 32; base += 2 * s) {
#pragma unroll
            for (int t = 0; t < s; ++t) {
                const float2 l = x[base + t], r = x[base + s + t];
                x[base + t] = fadd2(l, r);
                x[base + s + t] = ffma2(r, neg1, l);
            }
        }
    }
    // stride 64 across the lane pair: half 0 keeps left + right = fma(x, 1,
    // other), half 1 left - right = fma(x, -1, other)
    const float sg = half ? -1.0f : 1.0f;
    const float2 sg2 = make_float2(sg, sg);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float2 other = make_float2(__shfl_xor_sync(0xffffffffu, x[i].x, 16),
                                         __shfl_xor_sync(0xffffffffu, x[i].y, 16));
        x[i] = ffma2(x[i], sg2, other);
    }
    const float2 norm2 = make_float2(0.08838834764831845f, 0.08838834764831845f);   // fp32(128^-0.5)
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = fmul2(x[i], norm2);
}

template <typename T>
__device__ __forceinline__ void transform_half128(const RowArgs& a, int64_t h, int64_t tok, bool valid, int half,
                                                  const float* smean, float2 (&x)[32]) {
    if (valid) {
        const T* src = static_cast<const T*>(a.x) + (h * a.S + tok) * 128 + 64 * half;
#pragma unroll
        for (int i = 0; i < 8; ++i) load8x2(src + 8 * i, x + 4 * i);
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = make_float2(0.0f, 0.0f);
    }
    hadamard_half128(valid, half, smean, x);
}

// 64 E4M3 bytes of a half row: x / scale as div_by(x * pre, bdiv, rdiv)
// (the correctly rounded quotient), saturated to +-448 by the E4M3 cast.
// PRE: the scale was prescaled (tiny scales); otherwise pre == 1 and the
// multiply by it is skipped, which changes nothing.
template <bool PRE>
__device__ __forceinline__ void encode_half(const float (&x)[64], int c0, int W, float pre, float bdiv,
                                            float rdiv, uint4* dst) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = 16 * q + 4 * k + e;
                v[e] = c0 + c < W ? div_by(PRE ? __fmul_rn(x[c], pre) : x[c], bdiv, rdiv) : 0.0f;
            }
            w[k] = e4m3x2(v[0], v[1]) | (e4m3x2(v[2], v[3]) << 16);
        }
        dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// encode_half over the 32 channel pairs of transform_half128: div_by in
// packed FP32 (fma(q, -b, x) is fma(-q, b, x): the same exact product).
template <bool PRE>
__device__ __forceinline__ void encode_half128(const float2 (&x)[32], float pre, float bdiv, float rdiv,
                                               uint4* dst) {
    const float2 y2 = make_float2(rdiv, rdiv), nb2 = make_float2(-bdiv, -bdiv), p2 = make_float2(pre, pre);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t b[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float2 v = x[8 * q + 2 * k + e];
                if (PRE) v = fmul2(v, p2);
                const float2 qq = fmul2(v, y2);
                const float2 rr = ffma2(qq, nb2, v);
                const float2 d = ffma2(rr, y2, qq);
                b[e] = e4m3x2(d.x, d.y);
            }
            w[k] = b[0] | (b[1] << 16);
        }
        dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// One CTA per quantisation block, two threads per row, 256 rows per pass.
// Blocks of at most 256 rows keep the transformed halves in registers from
// the amax to the encode; larger blocks re-read and re-transform in pass 2.
// FIX: D == 128 with the 128-point Hadamard, on the packed helpers.
template <typename T, bool FIX>
__global__ void __launch_bounds__(512) qk_quant_kernel(RowArgs a) {
    pdl_wait();
    pdl_open();
    __shared__ __align__(16) float smean[128];
    __shared__ int32_t stok[256];
    __shared__ float red[16];
    __shared__ float sdiv[3];
    const int64_t h = blockIdx.y;
    const int b = blockIdx.x;
    const int nthr = blockDim.x;
    if (a.mean)
        for (int c = threadIdx.x; c < 128; c += nthr) smean[c] = a.mean[h * 128 + c];
    const int64_t r0 = (int64_t)b * a.block;
    const bool single = a.block <= nthr / 2;
    if (single && a.pi)      // the block's permuted rows, read once and early
        for (int i = threadIdx.x; i < a.block; i += nthr)
            stok[i] = r0 + i < a.S ? a.pi[h * a.S + r0 + i] : 0;
    __syncthreads();
    const float* sm = a.mean ? smean : nullptr;
    const int W = FIX ? 128 : a.hadamard ? a.width : a.D;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const int rows_per_pass = nthr / 2;
    using Half = std::conditional_t<FIX, float2[32], float[64]>;
    Half x;
    // the input row of block row rl (valid rows only)
    auto token = [&](int rl, int64_t r) -> int64_t {
        if (!a.pi) return r;
        return single ? (int64_t)stok[rl] : (int64_t)a.pi[h * a.S + r];
    };
    auto transform = [&](int64_t tok, bool valid) {
        if constexpr (FIX) transform_half128<T>(a, h, tok, valid, half, sm, x);
        else transform_half<T>(a, h, tok, valid, half, sm, x);
    };
    // max.NaN keeps a NaN (from a NaN or infinite input, or Inf - Inf in the
    // transform) all the way to the block maximum, which is then the
    // finiteness check of every input row of the block
    float amax = 0.0f;
    for (int base = 0; base < a.block; base += rows_per_pass) {
        const int rl = base + warp * 16 + (lane & 15);
        const int64_t r = r0 + rl;
        const bool valid = rl < a.block && r < a.S;
        transform(valid ? token(rl, r) : 0, valid);
        if constexpr (FIX) {
#pragma unroll
            for (int i = 0; i < 32; ++i) amax = fmax3_nan(amax, fabsf(x[i].x), fabsf(x[i].y));
        } else {
#pragma unroll
            for (int c = 0; c < 64; ++c)
                if (64 * half + c < W) amax = fmax_nan(amax, fabsf(x[c]));
        }
    }
    for (int o = 16; o > 0; o >>= 1) amax = fmax_nan(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float bmax = 0.0f;
        for (int w = 0; w < nthr / 32; ++w) bmax = fmax_nan(bmax, red[w]);
        if (!finite_f(bmax)) flag_status(a.status, VCB_FLAG_NONFINITE);
        float scale = bmax / 448.0f;
        if (scale == 0.0f) scale = 1.0f;
        if (b < a.nblk) a.scales[h * a.nblk + b] = scale;
        const float pre = div_prescale(scale);
        sdiv[0] = pre;
        sdiv[1] = scale * pre;
        sdiv[2] = __frcp_rn(scale * pre);
    }
    __syncthreads();
    const float pre = sdiv[0], bdiv = sdiv[1], rdiv = sdiv[2];
    for (int base = 0; base < a.block; base += rows_per_pass) {
        const int rl = base + warp * 16 + (lane & 15);
        const int64_t r = r0 + rl;
        const bool valid = rl < a.block && r < a.S;
        if (!single) transform(valid ? token(rl, r) : 0, valid);   // warp-uniform
        if (rl >= a.block || r >= a.S_pad) continue;
        uint4* dst = reinterpret_cast<uint4*>(a.payload + (h * a.S_pad + r) * 128 + 64 * half);
        if (!valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = make_uint4(0u, 0u, 0u, 0u);
            continue;
        }
        if constexpr (FIX) {
            if (pre == 1.0f) encode_half128<false>(x, pre, bdiv, rdiv, dst);   // block-uniform
            else encode_half128<true>(x, pre, bdiv, rdiv, dst);
        } else {
            if (pre == 1.0f) encode_half<false>(x, 64 * half, W, pre, bdiv, rdiv, dst);
            else encode_half<true>(x, 64 * half, W, pre, bdiv, rdiv, dst);
        }
    }
}

// ------------------------------------------------------------------------
// Persistent, staged form of qk_quant_kernel for 16-bit rows with D == 128,
// the 128-point Hadamard and blocks of 16 to 256 rows that divide 256 (a
// block spans whole warps; every Q block of the b200 configurations and K
// blocks up to 256).  The unstaged kernel holds one block's rows in
// registers from load to encode, so an SM has only one or two blocks' loads
// in flight and HBM idles while they compute.  Here one CTA of 16 warps per
// SM walks 256-row slabs (slab = one K block or several Q blocks), two
// threads per row as in qk_quant_kernel.  Each thread copies its own half
// row of the slab two steps ahead into a 3-slot shared-memory ring with
// 16-byte cp.async copies (through the permutation for K), so two slabs'
// loads are in flight while a third is transformed, and it reads back only
// what it copied itself: no barrier guards the ring.  Transform, block
// maximum and encode are qk_quant_kernel's, bit for bit.  Rows sit 272 bytes
// apart so that the 16 rows a warp reads at one column offset fall in
// different banks.
constexpr int kSlabRows = 256;
constexpr int kSlabStages = 3;
constexpr uint32_t kSlabPitch = 272;                              // bytes per staged row (256 + 16)
constexpr uint32_t kSlabStageBytes = kSlabRows * kSlabPitch;      // 69632
constexpr int kStagedWarps = 16;
constexpr int kStagedThreads = kStagedWarps * 32;
constexpr uint32_t kStagedSmem = kSlabStages * kSlabStageBytes + 2 * kStagedWarps * 4;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// eight 16-bit elements from shared memory as four channel pairs
template <typename T>
__device__ __forceinline__ void lds8x2(uint32_t addr, float2* o) {
    uint32_t w[4];
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "r"(addr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value)
            o[i] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        else
            o[i] = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    }
}

template <typename T>
__global__ void __launch_bounds__(kStagedThreads, 1) qk_quant_staged_kernel(RowArgs a, int64_t slabs_per_head,
                                                                            int64_t nslabs) {
    pdl_wait();
    pdl_open();
    extern __shared__ __align__(128) uint8_t sm[];
    float* partial = reinterpret_cast<float*>(sm + kSlabStages * kSlabStageBytes);   // [2][kStagedWarps]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const int rl = warp * 16 + (lane & 15);               // row in the slab
    const int B = a.block;                                // a multiple of 16 dividing kSlabRows
    const int w0 = (rl / B) * B / 16, w1 = w0 + B / 16;   // the warps of this row's block
    const T* x = static_cast<const T*>(a.x);
    const uint32_t slot0 = smem_u32(sm) + (uint32_t)rl * kSlabPitch + 128u * half;
    // this thread's half row of slab `slab` into ring slot `s` (nothing past S)
    auto fetch = [&](int64_t slab, int s) {
        if (slab < nslabs) {
            const int64_t h = slab / slabs_per_head, r = (slab % slabs_per_head) * kSlabRows + rl;
            if (r < a.S) {
                const int64_t tok = a.pi ? (int64_t)a.pi[h * a.S + r] : r;
                const T* src = x + (h * a.S + tok) * 128 + 64 * half;
                const uint32_t dst = slot0 + (uint32_t)s * kSlabStageBytes;
#pragma unroll
                for (int i = 0; i < 8; ++i) cp_async16(dst + 16u * i, src + 8 * i);
            }
        }
        cp_async_commit();                               // one group per step, empty or not
    };
    fetch(blockIdx.x, 0);
    fetch(blockIdx.x + gridDim.x, 1);
    int it = 0;
    for (int64_t slab = blockIdx.x; slab < nslabs; slab += gridDim.x, ++it) {
        const int s = it % kSlabStages;
        fetch(slab + 2 * (int64_t)gridDim.x, (it + 2) % kSlabStages);
        cp_async_wait<2>();                              // this thread's copies of `slab` have landed
        const int64_t h = slab / slabs_per_head, r0 = (slab % slabs_per_head) * kSlabRows;
        const int64_t r = r0 + rl;
        const bool valid = r < a.S;
        float2 xv[32];
        if (valid) {
            const uint32_t row = slot0 + (uint32_t)s * kSlabStageBytes;
#pragma unroll
            for (int i = 0; i < 8; ++i) lds8x2<T>(row + 16u * i, xv + 4 * i);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) xv[i] = make_float2(0.0f, 0.0f);
        }
        hadamard_half128(valid, half, a.mean ? a.mean + h * 128 : nullptr, xv);
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmax3_nan(amax, fabsf(xv[i].x), fabsf(xv[i].y));
        for (int o = 16; o > 0; o >>= 1) amax = fmax_nan(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) partial[(it & 1) * kStagedWarps + warp] = amax;
        // only the B / 16 warps of this row's block meet, so the blocks of a
        // slab drift apart and overlap their latencies (one warp for B = 16;
        // named barrier 1 + block index, 2 B threads, for B = 32 .. 128)
        if (B == 16) __syncwarp();
        else if (B == kSlabRows) __syncthreads();
        else asm volatile("bar.sync %0, %1;" ::"r"(1 + rl / B), "r"(2 * B) : "memory");
        float bmax = 0.0f;
        for (int w = w0; w < w1; ++w) bmax = fmax_nan(bmax, partial[(it & 1) * kStagedWarps + w]);
        float scale = bmax / 448.0f;
        if (scale == 0.0f) scale = 1.0f;
        const int64_t b = r / B;
        if (rl % B == 0 && half == 0 && r < a.S_pad) {
            if (!finite_f(bmax)) flag_status(a.status, VCB_FLAG_NONFINITE);
            if (b < a.nblk) a.scales[h * a.nblk + b] = scale;
        }
        if (r >= a.S_pad) continue;
        uint4* dst = reinterpret_cast<uint4*>(a.payload + (h * a.S_pad + r) * 128 + 64 * half);
        if (!valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = make_uint4(0u, 0u, 0u, 0u);
            continue;
        }
        const float pre = div_prescale(scale);
        const float bdiv = scale * pre, rdiv = __frcp_rn(scale * pre);
        if (pre == 1.0f) encode_half128<false>(xv, pre, bdiv, rdiv, dst);   // block-uniform
        else encode_half128<true>(xv, pre, bdiv, rdiv, dst);
    }
    cp_async_wait<0>();                                  // nothing lands after the CTA exits
}

// Transform-only rows (the preprocess_qk export): one row per thread.
template <typename T>
__global__ void __launch_bounds__(128) qk_transform_kernel(RowArgs a) {
    pdl_wait();
    pdl_open();
    __shared__ float smean[128];
    const int64_t h = blockIdx.y;
    if (a.mean) smean[threadIdx.x] = a.mean[h * 128 + threadIdx.x];
    __syncthreads();
    const int64_t r = (int64_t)blockIdx.x * 128 + threadIdx.x;
    if (r >= a.S) return;
    float x[128];
    transform_row<T>(a, h, r, a.mean ? smean : nullptr, x);
    const int W = a.hadamard ? a.width : a.D;
    float* dst = a.out_f32 + (h * a.S + r) * W;
#pragma unroll
    for (int c = 0; c < 128; ++c)
        if (c < W) dst[c] = x[c];
}

namespace {

int width_for(int d, int hadamard) {
    if (!hadamard) return d;
    int w = 1;
    while (w < d) w <<= 1;
    return w;
}

template <typename T>
int launch_k_mean(const void* k, int64_t heads, int64_t S, int D, float* partial, float* mean,
                  cudaStream_t st) {
    const int nchunk = (int)((S + kKsumChunk - 1) / kKsumChunk);
    VCB_CUDA(launch_pdl(k_colsum_kernel<T>, dim3(nchunk, (unsigned)heads), dim3(256), 0, st,
                        static_cast<const T*>(k), S, D, partial, nchunk));
    VCB_CUDA(launch_pdl(k_mean_kernel, dim3((unsigned)heads), dim3(128), 0, st, partial, nchunk, S, mean));
    return VCB_OK;
}

template <typename T>
int launch_rows(const RowArgs& a, int64_t heads, bool quantise, cudaStream_t st) {
    constexpr bool k16 = std::is_same<T, __nv_bfloat16>::value || std::is_same<T, __half>::value;
    const bool aligned = (reinterpret_cast<uintptr_t>(a.x) & 15u) == 0 &&
                         (reinterpret_cast<uintptr_t>(a.mean) & 15u) == 0;
    if (k16 && quantise && a.D == 128 && a.hadamard && a.block % 16 == 0 && kSlabRows % a.block == 0 && aligned) {
        const int64_t slabs_per_head = (a.S_pad + kSlabRows - 1) / kSlabRows;
        const int64_t nslabs = heads * slabs_per_head;
        const int64_t grid = nslabs < sm_count() ? nslabs : sm_count();
        auto kernel = qk_quant_staged_kernel<T>;
        VCB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStagedSmem));
        VCB_CUDA(launch_pdl(kernel, dim3((unsigned)grid), dim3(kStagedThreads), kStagedSmem, st, a, slabs_per_head,
                            nslabs));
        return VCB_OK;
    }
    if (quantise) {
        const unsigned grid = (unsigned)(a.S_pad / a.block);
        const int rows = a.block < 256 ? a.block : 256;
        const int nthr = (rows + 15) / 16 * 32;      // two threads per row, whole warps
        if (a.D == 128 && a.hadamard)
            VCB_CUDA(launch_pdl(qk_quant_kernel<T, true>, dim3(grid, (unsigned)heads), dim3(nthr), 0, st, a));
        else
            VCB_CUDA(launch_pdl(qk_quant_kernel<T, false>, dim3(grid, (unsigned)heads), dim3(nthr), 0, st, a));
    } else {
        VCB_CUDA(launch_pdl(qk_transform_kernel<T>, dim3((unsigned)((a.S + 127) / 128), (unsigned)heads), dim3(128), 0,
                            st, a));
    }
    return VCB_OK;
}

template <typename T>
int run_qk(const vcb_qk_args* p, bool quantise, cudaStream_t st) {
    const int width = width_for(p->d, p->hadamard);
    const float norm = (float)pow((double)width, -0.5);
    float* mean = nullptr;
    if (p->k_smooth) {
        float* ws = static_cast<float*>(p->workspace);
        mean = ws;                                   // [heads, 128]
        float* partial = ws + p->heads * 128;        // [heads, nchunk, 128]
        int rc = launch_k_mean<T>(p->k, p->heads, p->sk, p->d, partial, mean, st);
        if (rc) return rc;
    }
    RowArgs q{};
    q.x = p->q; q.S = p->sq; q.D = p->d; q.width = width; q.hadamard = p->hadamard; q.norm = norm;
    q.pi = nullptr; q.mean = nullptr; q.status = p->status;
    RowArgs k = q;
    k.x = p->k; k.S = p->sk; k.pi = p->pi; k.mean = mean;
    if (quantise) {
        q.block = p->q_block; q.S_pad = vcb_padded_rows(p->sq, p->q_block);
        q.nblk = (int)((p->sq + p->q_block - 1) / p->q_block); q.payload = p->q8; q.scales = p->q_scale;
        k.block = p->k_quant_block; k.S_pad = vcb_padded_rows(p->sk, p->k_quant_block);
        k.nblk = (int)((p->sk + p->k_quant_block - 1) / p->k_quant_block); k.payload = p->k8;
        k.scales = p->k_scale;
    } else {
        q.out_f32 = p->q_out;
        k.out_f32 = p->k_out;
    }
    int rc = launch_rows<T>(q, p->heads, quantise, st);
    if (rc) return rc;
    return launch_rows<T>(k, p->heads, quantise, st);
}

}  // namespace

size_t qk_workspace_bytes(int64_t heads, int64_t sk) {
    const int64_t nchunk = (sk + kKsumChunk - 1) / kKsumChunk;
    return (size_t)(heads * 128 + heads * nchunk * 128) * sizeof(float);
}

int qk_run(const vcb_qk_args* p, bool quantise, cudaStream_t st) {
    switch (p->dtype) {
        case VCB_F32: return run_qk<float>(p, quantise, st);
        case VCB_F16: return run_qk<__half>(p, quantise, st);
        case VCB_BF16: return run_qk<__nv_bfloat16>(p, quantise, st);
        default: return fail(VCB_ERR_INVALID_ARGUMENT, "unknown dtype %d", p->dtype);
    }
}

}  // namespace vcb
