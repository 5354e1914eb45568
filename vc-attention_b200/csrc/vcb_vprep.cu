// V tile preparation for sm_100a (reference: core.py:102-115 per kv_block
// tile at core.py:300-304, after the permutation of core.py:288-290; the
// Hopper extension used one CTA per (tile, channel), kernels.cu:124-162, and
// gathered V in PyTorch, cuda_backend.py:51).
//
// One CTA per (head, 128-token tile): the tile's tokens are gathered through
// the permutation with coalesced 16-byte cp.async row copies into shared
// memory (staged in the input type: 32 KB for bf16 / fp16, so more CTAs fit
// per SM), then
// thread c owns channel c: the finiteness check, the block mean (four
// interleaved partial sums in tile order, see below), residual, per-channel
// scale with the mean-dtype finite-storage guard, E4M3 residual written
// channel-major (the K-major B operand of the PV MMA), and the scaled mean
// rounded to the mean dtype.  With smoothing active the kernel also writes
// the mean operand of the attention kernel's row-mass x mean MMA: per channel
// the stored mean as three bf16 pieces (u1 = the value truncated to bf16,
// u2 and u3 the rounded remainders, so u1 + u2 + u3 carries its 24 bits) laid
// out as the K = 16 row [u1, u2, u3, u1, u2, u1, 0 ...] (32 bytes).
#include "vcb_internal.h"

namespace vcb {

constexpr int kTile = 128;

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

// three-input min that returns NaN when any input is NaN (sm_100)
__device__ __forceinline__ float fmin3_nan(float a, float b, float c) {
    float d;
    asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

template <typename T>
__global__ void __launch_bounds__(128) vprep_kernel(const T* __restrict__ v, int64_t S, int dv,
                                                    const int32_t* __restrict__ pi, int active,
                                                    int mean_type, int T_tiles, uint8_t* __restrict__ v8,
                                                    float* __restrict__ meta, uint16_t* __restrict__ mop,
                                                    int32_t* status) {
    pdl_wait();
    pdl_open();
    extern __shared__ __align__(16) uint8_t tile_raw[];
    T* tile = reinterpret_cast<T*>(tile_raw);     // [kTile][128] in the input type
    const int64_t h = blockIdx.y;
    const int t = blockIdx.x;
    const int64_t s0 = (int64_t)t * kTile;
    const int cnt = (int)min((int64_t)kTile, S - s0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    bool ok = true;
    __shared__ int64_t toks[kTile];
    if ((int)threadIdx.x < cnt) toks[threadIdx.x] = pi ? (int64_t)pi[h * S + s0 + threadIdx.x] : s0 + threadIdx.x;
    __syncthreads();
    if (dv == 128 && (reinterpret_cast<uintptr_t>(v) & 15) == 0) {
        // Rows of 16-byte pieces copied straight into shared memory
        // (cp.async, every copy of the tile in flight at once).  Rows past
        // the end of a ragged tile are not copied; nothing reads them.
        constexpr int E = 16 / (int)sizeof(T);        // elements per piece
        constexpr int NP = 128 / E;                   // pieces per row
        constexpr int kPer = kTile * NP / 128;        // pieces per thread
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int g = threadIdx.x + 128 * u, j = g / NP, k = g % NP;
            if (j < cnt) {
                const uint4* src = reinterpret_cast<const uint4*>(v + (h * S + toks[j]) * 128) + k;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                             ::"r"(smem_u32(tile + j * 128 + k * E)), "l"(__cvta_generic_to_global(src))
                             : "memory");
            }
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    } else
    for (int j = warp; j < kTile; j += 4) {
        const T* row = v + (h * S + toks[j < cnt ? j : 0]) * dv;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = 4 * lane + i;
            tile[j * 128 + c] = j < cnt && c < dv ? row[c] : T(0.0f);
        }
    }
    __syncthreads();
    const int c = threadIdx.x;
    const int64_t m = ((int64_t)h * T_tiles + t);
    uint32_t packed[32];
    float scale = 1.0f, stored = 0.0f;
    if (c < dv) {
        // One pass: the sum as four interleaved partial sums (token j into
        // part j % 4, each in token order, then (p0 + p1) + (p2 + p3)), and
        // the channel's min and max.  max |fl(x - mean)| is
        // max(fl(xmax - mean), fl(mean - xmin)), since rounding is monotone
        // and odd, so no second pass is needed for the scale.
        float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        float xmax = -INFINITY, xmin = INFINITY;
        if (cnt == kTile) {
            // tokens in pairs: part j % 4 in packed adds (each lane the same
            // RN add in token order); max.NaN / min.NaN carry a NaN or an
            // infinity to xmax / xmin, which is then the finiteness check
            float2 p01 = make_float2(0.0f, 0.0f), p23 = make_float2(0.0f, 0.0f);
#pragma unroll 8
            for (int j = 0; j < kTile; j += 4) {
                const float x0 = to_float(tile[j * 128 + c]), x1 = to_float(tile[(j + 1) * 128 + c]);
                const float x2 = to_float(tile[(j + 2) * 128 + c]), x3 = to_float(tile[(j + 3) * 128 + c]);
                p01 = fadd2(p01, make_float2(x0, x1));
                p23 = fadd2(p23, make_float2(x2, x3));
                xmax = fmax3_nan(fmax3_nan(xmax, x0, x1), x2, x3);
                xmin = fmin3_nan(fmin3_nan(xmin, x0, x1), x2, x3);
            }
            ok = finite_f(xmax) && finite_f(xmin);
            part[0] = p01.x; part[1] = p01.y; part[2] = p23.x; part[3] = p23.y;
        } else {
            for (int j = 0; j < cnt; ++j) {
                const float x = to_float(tile[j * 128 + c]);
                ok &= finite_f(x);
                part[j & 3] += x;
                xmax = fmaxf(xmax, x);
                xmin = fminf(xmin, x);
            }
        }
        float mean = 0.0f;
        if (active) mean = __fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3])) / (float)cnt;
        if (!ok) flag_status(status, VCB_FLAG_NONFINITE);
        const float amax = fmaxf(fmaxf(0.0f, __fsub_rn(xmax, mean)), __fsub_rn(mean, xmin));
        scale = amax / 448.0f;
        if (scale == 0.0f) scale = 1.0f;
        const float limit = mean_type == 1 ? 65504.0f : mean_type == 2 ? 3.3895313892515355e38f : 3.4028234663852886e38f;
        scale = fmaxf(scale, fabsf(mean) / limit);
        const float pre = div_prescale(scale);
        const float bdiv = scale * pre;
        const float rdiv = __frcp_rn(bdiv);
        if (cnt == kTile) {
            // div_by on token pairs in packed FP32 (fma(q, -b, x) is
            // fma(-q, b, x): the same exact product); a unit prescale is
            // skipped, which changes nothing
            const float2 nm = make_float2(-mean, -mean), p2 = make_float2(pre, pre);
            const float2 y2 = make_float2(rdiv, rdiv), nb2 = make_float2(-bdiv, -bdiv);
#pragma unroll
            for (int w = 0; w < 32; ++w) {
                uint32_t b2[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int j = 4 * w + 2 * e;
                    float2 r = fadd2(make_float2(to_float(tile[j * 128 + c]), to_float(tile[(j + 1) * 128 + c])), nm);
                    if (pre != 1.0f) r = fmul2(r, p2);
                    const float2 qq = fmul2(r, y2);
                    const float2 rr = ffma2(qq, nb2, r);
                    const float2 d = ffma2(rr, y2, qq);
                    b2[e] = e4m3x2(d.x, d.y);
                }
                packed[w] = b2[0] | (b2[1] << 16);
            }
        } else {
#pragma unroll
            for (int w = 0; w < 32; ++w) {
                float q[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * w + e;
                    const float r = to_float(tile[j * 128 + c]) - mean;
                    q[e] = j < cnt ? div_by(__fmul_rn(r, pre), bdiv, rdiv) : 0.0f;
                }
                packed[w] = e4m3x2(q[0], q[1]) | (e4m3x2(q[2], q[3]) << 16);
            }
        }
        const float sm = __fdiv_rn(mean, scale);
        stored = mean_type == 1 ? __half2float(__float2half_rn(sm))
               : mean_type == 2 ? __bfloat162float(__float2bfloat16_rn(sm)) : sm;
    } else {
#pragma unroll
        for (int w = 0; w < 32; ++w) packed[w] = 0u;
    }
    uint4* dst = reinterpret_cast<uint4*>(v8 + (m * 128 + c) * kTile);
#pragma unroll
    for (int q = 0; q < 8; ++q)
        dst[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    meta[m * 256 + c] = scale;
    meta[m * 256 + 128 + c] = stored;
    if (mop) {
        const __nv_bfloat16 u1 = __float2bfloat16_rz(stored);
        const float r1 = __fsub_rn(stored, __bfloat162float(u1));          // exact
        const __nv_bfloat16 u2 = __float2bfloat16_rn(r1);
        const __nv_bfloat16 u3 = __float2bfloat16_rn(__fsub_rn(r1, __bfloat162float(u2)));   // exact difference
        const uint32_t b1 = __bfloat16_as_ushort(u1), b2 = __bfloat16_as_ushort(u2), b3 = __bfloat16_as_ushort(u3);
        uint4* row = reinterpret_cast<uint4*>(mop + (m * 128 + c) * 16);
        row[0] = make_uint4(b1 | (b2 << 16), b3 | (b1 << 16), b2 | (b1 << 16), 0u);
        row[1] = make_uint4(0u, 0u, 0u, 0u);
    }
}

namespace {
template <typename T>
int launch(const vcb_v_args* p, cudaStream_t st) {
    const int T_tiles = (int)((p->s + kTile - 1) / kTile);
    const size_t smem = kTile * 128 * sizeof(T);
    VCB_CUDA(cudaFuncSetAttribute(vprep_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    VCB_CUDA(launch_pdl(vprep_kernel<T>, dim3(T_tiles, (unsigned)p->heads), dim3(128), smem, st,
                        static_cast<const T*>(p->v), p->s, p->dv, p->pi, p->active, p->mean_type, T_tiles, p->v8,
                        p->v_meta, p->active ? p->v_mean_op : nullptr, p->status));
    return VCB_OK;
}
}  // namespace

int vprep_run(const vcb_v_args* p, cudaStream_t st) {
    switch (p->dtype) {
        case VCB_F32: return launch<float>(p, st);
        case VCB_F16: return launch<__half>(p, st);
        case VCB_BF16: return launch<__nv_bfloat16>(p, st);
        default: return fail(VCB_ERR_INVALID_ARGUMENT, "unknown dtype %d", p->dtype);
    }
}

}  // namespace vcb
