// Fused VC-Attention forward for sm_100a.
//
// Replaces the reference's host loop over heads x Q tiles x KV tiles
// (kernels.cu:313-330: a cuBLASLt E4M3 GEMM for S, softmax_update, a second
// GEMM for PV and accumulate, all through HBM scratch) with one CTA per
// (head, 128-row Q tile) that keeps every intermediate on chip:
//
//   warp 0      TMA producer: Q tile once, then K / V / V-metadata tiles into
//               a 4-stage ring (no cluster multicast).
//   warp 1      MMA issuer (one thread): S_j = Q8 K8_j^T into TMEM
//               (tcgen05.mma kind::f8f6f4, E4M3 x E4M3 -> F32), then
//               O_j = P_j R_j with P read from TMEM.  In ExpCast mode V carries
//               16 extra rows of E4M3 ones, so column 128 of O_j is the row
//               mass sum(decode(P_j)) produced by the tensor core itself.
//   warps 4-7   softmax: one thread per query row.  Row max, alpha, and either
//               the ExpCast byte encode (one FMA per score, the f16-subnormal
//               conversion rounds to the integer code and clamps at zero) or
//               exp + E4M3(p * 256); P is written back over S in TMEM.
//   warps 8-15  correction: acc = alpha * acc + (O_j + M_j * mu_j) * vscale_j
//               per row and channel (two threads per row, 64 channels each),
//               den = alpha * den + M_j; epilogue acc / den in the output dtype.
//
// Numerical contract (core.py:307-341): S = (q8 . k8) * qs * ks * scale;
// ExpCast code = rne(clamp(fma(S - m, 8 log2 e, 119.65), 0, 120)) viewed as
// E4M3 with a 1/256 scale and a decoded row mass; non-ExpCast P8 =
// e4m3(exp(S - m) * 256) with an FP32 row mass; V-mean recovery lives inside
// the accumulator and is rescaled with the running max.  Accumulators are
// kept in units of 256 (acc256 = 256 acc, den256 = 256 den), which changes no
// rounding because 256 is a power of two.
//
// TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+N) with N = 144
// (ExpCast) or 128.  All mbarrier waits are bounded (vcb_common.cuh).
#include "vcb_internal.h"

namespace vcb {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kStages = 4;
constexpr int kThreads = 512;
constexpr uint32_t kTile = 128 * 128;            // one E4M3 tile
constexpr uint32_t kVBytes = kTile + 16 * 128;   // + 16 rows of ones
constexpr uint32_t kMetaBytes = 1024;            // vscale[128], mu[128]
constexpr uint32_t kStageBytes = kTile + kVBytes + kMetaBytes;
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffStages = kTile;
constexpr uint32_t kOffStats = kOffStages + kStages * kStageBytes;   // alpha[4][128], mass[4][128]
constexpr uint32_t kOffBars = kOffStats + 2 * 4 * 128 * 4;
constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 1 + 1 + 4 + 4 + 1;
constexpr uint32_t kOffMisc = kOffBars + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 16;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;

constexpr float kC1 = 11.541560173034668f;       // 8 log2(e) in fp32
constexpr float kC2 = 119.6500015258789f;        // 119.65 in fp32
constexpr float kTwoM24 = 5.9604644775390625e-08f;   // 2^-24
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
    CUtensorMap tm_q, tm_k, tm_v;
    const float* q_scale;
    const float* k_scale;
    const float* v_meta;
    void* out;
    int32_t* status;
    int64_t sq, sk;
    int dv, q_block, kq, nqb, nkb, T;
    int expcast, has_mean, out_dtype;
    float scale;
};

struct Bars {
    uint64_t* q_full;
    uint64_t* kv_full;     // [kStages]
    uint64_t* kv_empty;    // [kStages]
    uint64_t* s_full;      // [2]
    uint64_t* p_full;      // [2]
    uint64_t* o_full;
    uint64_t* o_free;
    uint64_t* st_full;     // [4]
    uint64_t* st_free;     // [4]
    uint64_t* drain;
};

__device__ __forceinline__ Bars bars_at(uint8_t* smem) {
    uint64_t* b = reinterpret_cast<uint64_t*>(smem + kOffBars);
    Bars r;
    r.q_full = b; b += 1;
    r.kv_full = b; b += kStages;
    r.kv_empty = b; b += kStages;
    r.s_full = b; b += 2;
    r.p_full = b; b += 2;
    r.o_full = b; b += 1;
    r.o_free = b; b += 1;
    r.st_full = b; b += 4;
    r.st_free = b; b += 4;
    r.drain = b;
    return r;
}

// Bounded wait used while draining after an abort: ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer() - t0 > kWaitLimitNs) return;
    }
}

__device__ __forceinline__ uint32_t cvt_relu_f16x2(float hi, float lo) {
    uint32_t d;
    asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

__device__ void producer(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort, int qtile,
                         int head) {
    prefetch_tmap(&p.tm_q);
    prefetch_tmap(&p.tm_k);
    prefetch_tmap(&p.tm_v);
    mbar_arrive_expect_tx(B.q_full, kTile);
    tma_load_3d(smem + kOffQ, &p.tm_q, B.q_full, 0, qtile * kBM, head);
    int armed[kStages] = {0, 0, 0, 0};
    const float* meta = p.v_meta + (int64_t)head * p.T * 256;
    for (int j = 0; j < p.T; ++j) {
        const int s = j % kStages, u = j / kStages;
        if (u > 0 && !mbar_wait(&B.kv_empty[s], (u - 1) & 1, abort)) break;
        uint8_t* st = smem + kOffStages + s * kStageBytes;
        mbar_arrive_expect_tx(&B.kv_full[s], 2 * kTile + kMetaBytes);
        tma_load_3d(st, &p.tm_k, &B.kv_full[s], 0, j * kBN, head);
        tma_load_3d(st + kTile, &p.tm_v, &B.kv_full[s], 0, j * 128, head);
        bulk_load(st + kTile + kVBytes, meta + (int64_t)j * 256, kMetaBytes, &B.kv_full[s]);
        armed[s] = u + 1;
    }
    if (*abort) {   // no TMA write may land after the CTA exits
        drain_wait(B.q_full, 0);
        for (int s = 0; s < kStages; ++s)
            if (armed[s] > 0) drain_wait(&B.kv_full[s], (armed[s] - 1) & 1);
    }
}

__device__ void mma_issuer(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort, uint32_t tmem) {
    const uint32_t idesc_qk = idesc_e4m3_f32(kBM, kBN);
    const uint32_t idesc_pv = idesc_e4m3_f32(kBM, p.expcast ? 144 : 128);
    const uint64_t qdesc = smem_desc_k128(smem + kOffQ);
    if (mbar_wait(B.q_full, 0, abort)) {
        for (int j = 0; j <= p.T; ++j) {
            if (j < p.T) {
                const int s = j % kStages;
                if (!mbar_wait(&B.kv_full[s], (j / kStages) & 1, abort)) break;
                tc_fence_after();
                const int b = j & 1;
                const uint64_t kdesc = smem_desc_k128(smem + kOffStages + s * kStageBytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f8_ss(tmem + b * kBN, qdesc + 2 * kk, kdesc + 2 * kk, idesc_qk, kk > 0);
                mma_commit(&B.s_full[b]);
            }
            if (j >= 1) {
                const int jp = j - 1, bp = jp & 1, sp = jp % kStages;
                if (!mbar_wait(&B.p_full[bp], (jp >> 1) & 1, abort)) break;
                if (jp >= 1 && !mbar_wait(B.o_free, (jp - 1) & 1, abort)) break;
                tc_fence_after();
                const uint64_t vdesc = smem_desc_k128(smem + kOffStages + sp * kStageBytes + kTile);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_f8_ts(tmem + kColO, tmem + bp * kBN + kk * 8, vdesc + 2 * kk, idesc_pv, kk > 0);
                mma_commit(B.o_full);
                mma_commit(&B.kv_empty[sp]);
            }
        }
    }
    mma_commit(B.drain);
    drain_wait(B.drain, 0);
}

__device__ void softmax_role(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort, uint32_t tmem,
                             int qtile, int head, int quarter, int lane) {
    const int row = quarter * 32 + lane;
    const int64_t grow = (int64_t)qtile * kBM + row;
    int qb = (int)(grow / p.q_block);
    if (qb >= p.nqb) qb = p.nqb - 1;
    const float qs = p.q_scale[(int64_t)head * p.nqb + qb];
    const float* ksp = p.k_scale + (int64_t)head * p.nkb;
    float* st_alpha = reinterpret_cast<float*>(smem + kOffStats);
    float* st_mass = st_alpha + 4 * 128;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    float m = -INFINITY;
    for (int j = 0; j < p.T; ++j) {
        const int b = j & 1;
        if (!mbar_wait(&B.s_full[b], (j >> 1) & 1, abort)) break;
        tc_fence_after();
        const int nvalid = (int)min((int64_t)kBN, p.sk - (int64_t)j * kBN);
        const bool tail = nvalid < kBN;
        const uint32_t ts = trow + b * kBN;
        float mx = -INFINITY;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
            uint32_t r[32];
            tmem_ld32(ts + 32 * ch, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float v = __uint_as_float(r[i]);
                if (tail && 32 * ch + i >= nvalid) v = -INFINITY;
                mx = fmaxf(mx, v);
            }
        }
        const float ks = ksp[((int64_t)j * kBN) / p.kq];
        const float c = __fmul_rn(__fmul_rn(qs, ks), p.scale);
        const float smax = __fmul_rn(mx, c);
        const float m_new = fmaxf(m, smax);
        const float alpha = expf(m - m_new);
        float A, Bc;
        if (p.expcast) {
            A = __fmul_rn(c, kC1);
            Bc = __fsub_rn(kC2, __fmul_rn(m_new, kC1));
            const float umax = fmaf(mx, A, Bc);
            if (umax > 120.25f) Bc = __fsub_rn(Bc, __fsub_rn(umax, kC2));
            A = __fmul_rn(A, kTwoM24);
            Bc = __fmul_rn(Bc, kTwoM24);
        } else {
            A = __fmul_rn(c, kLog2e);
            Bc = __fsub_rn(8.0f, __fmul_rn(m_new, kLog2e));
        }
        float psum = 0.0f;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
            uint32_t r[32];
            tmem_ld32(ts + 32 * ch, r);
            tmem_wait_ld();
            uint32_t pk[8];
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    v[e] = __uint_as_float(r[4 * w + e]);
                    if (tail && 32 * ch + 4 * w + e >= nvalid) v[e] = -INFINITY;
                }
                if (p.expcast) {
                    const uint32_t h01 = cvt_relu_f16x2(fmaf(v[1], A, Bc), fmaf(v[0], A, Bc));
                    const uint32_t h23 = cvt_relu_f16x2(fmaf(v[3], A, Bc), fmaf(v[2], A, Bc));
                    pk[w] = __byte_perm(h01, h23, 0x6420);
                } else {
                    float e[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        e[q] = exp2f(fmaf(v[q], A, Bc));
                        psum = __fadd_rn(psum, e[q]);
                    }
                    pk[w] = e4m3x2(e[0], e[1]) | (e4m3x2(e[2], e[3]) << 16);
                }
            }
            tmem_st8(ts + 8 * ch, pk);
        }
        tmem_wait_st();
        const int slot = j & 3;
        if (j >= 4 && !mbar_wait(&B.st_free[slot], ((j >> 2) - 1) & 1, abort)) break;
        st_alpha[slot * 128 + row] = alpha;
        st_mass[slot * 128 + row] = psum;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&B.p_full[b]);
            mbar_arrive(&B.st_full[slot]);
        }
        m = m_new;
    }
}

__device__ void correction_role(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort,
                                uint32_t tmem, int qtile, int head, int quarter, int half, int lane) {
    const int row = quarter * 32 + lane;
    const float* st_alpha = reinterpret_cast<const float*>(smem + kOffStats);
    const float* st_mass = st_alpha + 4 * 128;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const int c0 = half * 64;
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
    float den = 0.0f;
    bool done = true;
    for (int j = 0; j < p.T; ++j) {
        if (!mbar_wait(B.o_full, j & 1, abort)) { done = false; break; }
        const int slot = j & 3, sp = j % kStages;
        if (!mbar_wait(&B.st_full[slot], (j >> 2) & 1, abort)) { done = false; break; }
        tc_fence_after();
        const float alpha = st_alpha[slot * 128 + row];
        float M = st_mass[slot * 128 + row];
        const float* meta = reinterpret_cast<const float*>(smem + kOffStages + sp * kStageBytes + kTile + kVBytes);
        const bool rescale = __any_sync(0xffffffffu, alpha != 1.0f);
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
            uint32_t r[32];
            tmem_ld32(trow + kColO + c0 + 32 * ch, r);
            if (ch == 0 && p.expcast) {
                uint32_t mu;
                tmem_ld1(trow + kColO + 128, mu);
                tmem_wait_ld();
                M = __uint_as_float(mu);
            } else {
                tmem_wait_ld();
            }
            if (ch == 1) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(B.o_free);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int col = c0 + 32 * ch + i;
                const float o = __uint_as_float(r[i]);
                const float x = p.has_mean ? fmaf(M, meta[128 + col], o) : o;
                const float a = rescale ? __fmul_rn(acc[32 * ch + i], alpha) : acc[32 * ch + i];
                acc[32 * ch + i] = fmaf(x, meta[col], a);
            }
        }
        den = __fadd_rn(__fmul_rn(alpha, den), M);
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&B.st_free[slot]);
            mbar_arrive(&B.kv_empty[sp]);
        }
    }
    if (!done) return;
    const int64_t grow = (int64_t)qtile * kBM + row;
    if (grow >= p.sq) return;
    const int64_t base = ((int64_t)head * p.sq + grow) * p.dv;
    if (p.out_dtype == VCB_BF16 && p.dv == 128) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + base + c0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__fdiv_rn(acc[8 * q + 2 * e], den),
                                                         __fdiv_rn(acc[8 * q + 2 * e + 1], den));
                w[e] = *reinterpret_cast<uint32_t*>(&h);
            }
            dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        const int col = c0 + i;
        if (col >= p.dv) break;
        const float val = __fdiv_rn(acc[i], den);
        if (p.out_dtype == VCB_BF16) static_cast<__nv_bfloat16*>(p.out)[base + col] = __float2bfloat16_rn(val);
        else if (p.out_dtype == VCB_F16) static_cast<__half*>(p.out)[base + col] = __float2half_rn(val);
        else static_cast<float*>(p.out)[base + col] = val;
    }
}

__global__ void __launch_bounds__(kThreads, 1) attn_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Bars B = bars_at(smem);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qtile = blockIdx.x, head = blockIdx.y;

    if (threadIdx.x == 0) {
        mbar_init(B.q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&B.kv_full[s], 1);
            mbar_init(&B.kv_empty[s], 1 + 8);     // MMA commit + 8 correction warps
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&B.s_full[b], 1);
            mbar_init(&B.p_full[b], 4);           // 4 softmax warps
        }
        mbar_init(B.o_full, 1);
        mbar_init(B.o_free, 8);
        for (int s = 0; s < 4; ++s) {
            mbar_init(&B.st_full[s], 4);
            mbar_init(&B.st_free[s], 8);
        }
        mbar_init(B.drain, 1);
        *abort = 0;
        fence_barrier_init();
    }
    // rows 128..143 of every V buffer: E4M3 1.0, the ones that make O[:,128] the row mass
    for (int i = threadIdx.x; i < kStages * 128; i += kThreads) {
        const int s = i / 128, q = i % 128;
        reinterpret_cast<uint4*>(smem + kOffStages + s * kStageBytes + kTile + kTile)[q] =
            make_uint4(0x38383838u, 0x38383838u, 0x38383838u, 0x38383838u);
    }
    fence_proxy_async_smem();
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) producer(p, smem, B, abort, qtile, head);
    } else if (warp == 1) {
        if (lane == 0) mma_issuer(p, smem, B, abort, tmem);
    } else if (warp >= 4 && warp < 8) {
        softmax_role(p, smem, B, abort, tmem, qtile, head, warp - 4, lane);
    } else if (warp >= 8) {
        correction_role(p, smem, B, abort, tmem, qtile, head, warp & 3, (warp - 8) >> 2, lane);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort) flag_status(p.status, VCB_FLAG_TIMEOUT);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encoder(EncodeTiledFn* fn) {
    static EncodeTiledFn cached = nullptr;
    if (!cached) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr)
            return fail(VCB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        cached = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    *fn = cached;
    return VCB_OK;
}

// 3-D byte tensor [z][y][128] with 128-byte rows, tiles of 128 x 128, 128B swizzle.
int make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t planes) {
    EncodeTiledFn enc;
    int rc = get_encoder(&enc);
    if (rc) return rc;
    const cuuint64_t dims[3] = {128, rows, planes};
    const cuuint64_t strides[2] = {128, 128 * rows};
    const cuuint32_t box[3] = {128, 128, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VCB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return VCB_OK;
}

}  // namespace

int attn_run(const vcb_attn_args* a, cudaStream_t st) {
    Params p;
    memset(&p, 0, sizeof(p));
    const int64_t sq_pad = vcb_padded_rows(a->sq, a->q_block);
    const int64_t sk_pad = vcb_padded_rows(a->sk, a->k_quant_block);
    const int T = (int)((a->sk + kBN - 1) / kBN);
    int rc = make_map(&p.tm_q, a->q8, (uint64_t)sq_pad, (uint64_t)a->heads);
    if (!rc) rc = make_map(&p.tm_k, a->k8, (uint64_t)sk_pad, (uint64_t)a->heads);
    if (!rc) rc = make_map(&p.tm_v, a->v8, (uint64_t)T * 128, (uint64_t)a->heads);
    if (rc) return rc;
    p.q_scale = a->q_scale;
    p.k_scale = a->k_scale;
    p.v_meta = a->v_meta;
    p.out = a->out;
    p.status = a->status;
    p.sq = a->sq;
    p.sk = a->sk;
    p.dv = a->dv;
    p.q_block = a->q_block;
    p.kq = a->k_quant_block;
    p.nqb = (int)((a->sq + a->q_block - 1) / a->q_block);
    p.nkb = (int)((a->sk + a->k_quant_block - 1) / a->k_quant_block);
    p.T = T;
    p.expcast = a->expcast;
    p.has_mean = a->has_mean;
    p.out_dtype = a->out_dtype;
    p.scale = a->scale;
    VCB_CUDA(cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemAlloc));
    const dim3 grid((unsigned)((a->sq + kBM - 1) / kBM), (unsigned)a->heads);
    attn_kernel<<<grid, kThreads, kSmemAlloc, st>>>(p);
    VCB_CUDA(cudaGetLastError());
    return VCB_OK;
}

}  // namespace vcb
