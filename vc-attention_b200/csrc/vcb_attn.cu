// Fused VC-Attention forward for sm_100a.
//
// Replaces the reference's host loop over heads x Q tiles x KV tiles
// (kernels.cu:313-330: a cuBLASLt E4M3 GEMM for S, softmax_update, a second
// GEMM for PV and accumulate, all through HBM scratch) with one CTA per
// (head, 128-row Q tile) that keeps every intermediate on chip.
//
// Roles (640 threads, register budgets rebalanced with setmaxnreg):
//   warp 0      TMA producer: the Q tile once, then K / V tiles into a 4-stage
//               ring (no cluster multicast).
//   warp 2      the per-tile V scales and means into a 16-slot ring.
//   warp 1      MMA issuer (one thread): S_j = Q8 K8_j^T into TMEM
//               (tcgen05.mma kind::f8f6f4, E4M3 x E4M3 -> F32) and
//               O_j = P_j R_j with P_j in TMEM and R_j in shared memory.
//   warps 4-11  softmax, two threads of one warp per query row (64 scores
//               each; one shuffle swaps the partial row maxima): row max, alpha,
//               the ExpCast byte encode (one packed FMA per pair of scores;
//               the f16-subnormal conversion rounds to the integer code and
//               clamps it at zero) or exp + E4M3(p * 256); the row mass;
//               P_j written back over the thread's own S_j columns.
//   warps 12-19 correction, two threads per row (64 channels each):
//               acc = alpha acc + (O_j + M_j mu_j) vscale_j,
//               den = alpha den + M_j; epilogue acc / den in the output dtype.
//
// Latency hiding: S and O are double-buffered in TMEM (S0, S1, O0, O1 use all
// 512 columns).  P_j lives in S_j's columns, so the MMA issues PV_j and then
// QK_{j+2} into the same buffer (the tensor pipe keeps issue order); QK_{j+2}
// runs while the softmax works on tile j+1.  PV_j only waits for the
// correction of tile j-2.  The commit that signals PV_j done (o_full) also
// tells the producer that K/V stage j % 4 is free.
//
// Numerical contract (core.py:307-341): S = (q8 . k8) * qs * ks * scale;
// ExpCast code = rne(clamp(fma(S - m, 8 log2 e, 119.65), 0, 120)) viewed as
// E4M3 with a 1/256 scale, row mass = sum of decoded P; non-ExpCast P8 =
// e4m3(exp(S - m) * 256) with an FP32 row mass of exp; V-mean recovery lives
// inside the accumulator and is rescaled with the running max.  The
// accumulators are kept in units of 256 (acc256 = 256 acc, den256 = 256
// den); 256 is a power of two, so no rounding changes.  Every mbarrier wait
// is bounded (vcb_common.cuh).
#include "vcb_internal.h"
#include <type_traits>

namespace vcb {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kStages = 4;
constexpr int kMetaSlots = 16;                   // per-tile vscale / mu ring
constexpr int kThreads = 640;                    // 20 warps: 4 producer/MMA, 8 softmax, 8 correction
constexpr uint32_t kTile = 128 * 128;            // one E4M3 tile (16 KB)
constexpr uint32_t kMetaBytes = 1024;            // vscale[128], mu[128]
constexpr uint32_t kStageBytes = 2 * kTile;      // K tile, V tile
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffStages = kTile;
constexpr uint32_t kOffMeta = kOffStages + kStages * kStageBytes;    // vscale[128], mu[128] per slot
constexpr uint32_t kOffStats = kOffMeta + kMetaSlots * kMetaBytes;   // alpha[4][128], mass[4][2][128]
constexpr uint32_t kOffBars = kOffStats + 3 * 4 * 128 * 4;
constexpr int kNumBars = 1 + kStages + 2 * kMetaSlots + 2 * 4 + 2 * 4 + 1;
constexpr uint32_t kOffMisc = kOffBars + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 16;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                    // S0, S1
constexpr uint32_t kColO = 256;                  // O0, O1

constexpr float kC1 = 11.541560173034668f;       // 8 log2(e) in fp32
constexpr float kC2 = 119.6500015258789f;        // 119.65 in fp32
constexpr float kTwoM24 = 5.9604644775390625e-08f;   // 2^-24
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMinNormal = 1.17549435e-38f;    // 2^-126

struct Params {
    CUtensorMap tm_q, tm_k, tm_v;
    const float* q_scale;
    const float* k_scale;
    const float* v_meta;
    void* out;
    int32_t* status;
    int64_t sq, sk;
    int dv, q_block, kq, nqb, nkb, T;
    int out_dtype;
    float scale;
    // diagnostic dump of one CTA's softmax (vcb_attention_fp8_probe)
    float* pr_logits;      // [pr_count][128][128] raw accumulators q8 . k8 (masked keys -inf)
    uint8_t* pr_codes;     // [pr_count][128][128] P bytes as stored for the PV MMA
    float* pr_rowstat;     // [pr_count][128][4]: running max after the tile, A, B, alpha
    int pr_head, pr_qtile, pr_begin, pr_count;
};

struct Bars {
    uint64_t* q_full;
    uint64_t* kv_full;     // [kStages]
    uint64_t* meta_full;   // [kMetaSlots]
    uint64_t* meta_empty;  // [kMetaSlots]  the 8 correction warps have read the slot
    uint64_t* s_full;      // [2]  QK_j done
    uint64_t* p_full;      // [2]  P_j in TMEM (implies S_j fully read)
    uint64_t* o_full;      // [2]  PV_j done; also frees K/V stage j % kStages
    uint64_t* o_free;      // [2]  correction has read O_j
    uint64_t* st_full;     // [4]  alpha / mass of tile j
    uint64_t* st_free;     // [4]
    uint64_t* drain;
};

__device__ __forceinline__ Bars bars_at(uint8_t* smem) {
    uint64_t* b = reinterpret_cast<uint64_t*>(smem + kOffBars);
    Bars r;
    r.q_full = b; b += 1;
    r.kv_full = b; b += kStages;
    r.meta_full = b; b += kMetaSlots;
    r.meta_empty = b; b += kMetaSlots;
    r.s_full = b; b += 2;
    r.p_full = b; b += 2;
    r.o_full = b; b += 2;
    r.o_free = b; b += 2;
    r.st_full = b; b += 4;
    r.st_free = b; b += 4;
    r.drain = b;
    return r;
}

// Bounded wait used while draining after an abort: ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait_sleep(a, parity, kSuspendHintNs)) {
        if (globaltimer() - t0 > kWaitLimitNs) return;
    }
}

// 2^x as the single MUFU.EX2 instruction, flushing subnormal results to zero.
// The softmax's P = 2^g lies in [0, 256]; a result below 2^-126 encodes to
// E4M3 zero either way and cannot move an FP32 row mass of at least 256, so
// this gives the same bytes and mass as exp2f with fewer instructions.
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
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
    int loaded = 0;
    for (int j = 0; j < p.T; ++j) {
        const int s = j % kStages, u = j / kStages;
        // stage s last held tile j - kStages, free once PV of that tile is done (o_full of its buffer)
        if (u > 0 && !mbar_wait(&B.o_full[(j - kStages) & 1], ((j - kStages) >> 1) & 1, abort)) break;
        uint8_t* st = smem + kOffStages + s * kStageBytes;
        mbar_arrive_expect_tx(&B.kv_full[s], 2 * kTile);
        tma_load_3d(st, &p.tm_k, &B.kv_full[s], 0, j * kBN, head);
        tma_load_3d(st + kTile, &p.tm_v, &B.kv_full[s], 0, j * 128, head);
        loaded = j + 1;
    }
    if (*abort) {   // no TMA write may land after the CTA exits
        drain_wait(B.q_full, 0);
        for (int s = 0; s < kStages && s < loaded; ++s)     // last use of stage s: tile s + 4 u
            drain_wait(&B.kv_full[s], ((loaded - 1 - s) / kStages) & 1);
    }
}

// The per-tile V scales and means (1 KB) run on their own deeper ring, so a
// K/V stage is free as soon as the PV of its tile has been committed.
__device__ void meta_producer(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort, int head) {
    const float* meta = p.v_meta + (int64_t)head * p.T * 256;
    int loaded = 0;
    for (int j = 0; j < p.T; ++j) {
        const int s = j % kMetaSlots, u = j / kMetaSlots;
        if (u > 0 && !mbar_wait(&B.meta_empty[s], (u - 1) & 1, abort)) break;
        mbar_arrive_expect_tx(&B.meta_full[s], kMetaBytes);
        bulk_load(smem + kOffMeta + s * kMetaBytes, meta + (int64_t)j * 256, kMetaBytes, &B.meta_full[s]);
        loaded = j + 1;
    }
    if (*abort)
        for (int s = 0; s < kMetaSlots && s < loaded; ++s)
            drain_wait(&B.meta_full[s], ((loaded - 1 - s) / kMetaSlots) & 1);
}

// The MMA thread shares its SM sub-partition with four busy softmax /
// correction warps, and every instruction it issues waits for a scheduler
// slot (a microbenchmark: 64 cycles per MMA alone, ~270 next to four FMA-bound
// warps).  So its instruction stream is kept short: shared-memory descriptors
// differ only in the low word (start address >> 4), which the loop advances
// by constants; the high word (stride, version, 128B swizzle) is one register.
__device__ __forceinline__ void mma_ss_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t hi, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "mov.b64 da, {%1, %3};\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], da, db, %4, p;\n\t}"
        ::"r"(d_tmem), "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_ts_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t hi, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], db, %4, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The tile loop is unrolled by the 4 K/V stages, so stage and TMEM buffer
// offsets are compile-time constants.
__device__ void mma_issuer(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort, uint32_t tmem) {
    const uint32_t idesc = idesc_e4m3_f32(kBM, kBN);
    const uint64_t q64 = smem_desc_k128(smem + kOffQ);
    const uint32_t hi = (uint32_t)(q64 >> 32);
    const uint32_t qlo = (uint32_t)q64;
    // descriptor low word of stage 0's K tile; the others are constant offsets (bytes >> 4)
    const uint32_t k0lo = (uint32_t)smem_desc_k128(smem + kOffStages);
    constexpr uint32_t kStageLo = kStageBytes >> 4, kTileLo = kTile >> 4;
    auto qk = [&](uint32_t d, uint32_t klo) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma_ss_lo(d, qlo + 2 * kk, klo + 2 * kk, hi, idesc, kk > 0);
    };
    bool ok = mbar_wait(B.q_full, 0, abort);
    for (int j = 0; ok && j < 2 && j < p.T; ++j) {
        if (!mbar_wait(&B.kv_full[j], 0, abort)) { ok = false; break; }
        tc_fence_after();
        qk(tmem + kColS + j * kBN, k0lo + j * kStageLo);
        mma_commit(&B.s_full[j]);
    }
    auto step = [&](auto U_, int j) -> bool {
        constexpr int U = decltype(U_)::value;       // j % 4
        constexpr int b = U & 1, s = U, s2 = (U + 2) & 3;
        if (!mbar_wait(&B.p_full[b], (j >> 1) & 1, abort)) return false;
        if (j >= 2 && !mbar_wait(&B.o_free[b], ((j - 2) >> 1) & 1, abort)) return false;
        const bool next = j + 2 < p.T;
        if (next && !mbar_wait(&B.kv_full[s2], ((j + 2) >> 2) & 1, abort)) return false;
        tc_fence_after();
        const uint32_t pa = tmem + kColS + b * kBN;
        const uint32_t vlo = k0lo + s * kStageLo + kTileLo;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
            mma_ts_lo(tmem + kColO + b * 128, pa + (kk >> 1) * 64 + (kk & 1) * 8, vlo + 2 * kk, hi, idesc, kk > 0);
        mma_commit(&B.o_full[b]);      // also frees K/V stage s (the producer waits on it)
        if (next) {
            qk(pa, k0lo + s2 * kStageLo);
            mma_commit(&B.s_full[b]);
        }
        return true;
    };
    for (int j = 0; ok && j < p.T; j += 4) {
        ok = step(std::integral_constant<int, 0>{}, j);
        if (ok && j + 1 < p.T) ok = step(std::integral_constant<int, 1>{}, j + 1);
        if (ok && j + 2 < p.T) ok = step(std::integral_constant<int, 2>{}, j + 2);
        if (ok && j + 3 < p.T) ok = step(std::integral_constant<int, 3>{}, j + 3);
    }
    mma_commit(B.drain);
    drain_wait(B.drain, 0);
}

// Two threads of one warp per query row: warp w (quarter w % 4, sub (w-4)/4)
// owns TMEM lanes 32*quarter + 16*sub + [0, 16); lane t < 16 reads columns
// [0, 64) of its row and lane t + 16 columns [64, 128), so the partial row
// maxima meet in one shuffle.

// 16 TMEM lanes x 32 columns per half: thread t < 16 reads lane base + t at
// columns [c, c + 32), thread t + 16 the same lane at [c + 64, c + 96)
// (tcgen05 .16x32bx2 with a half split of 64 columns).
template <int OFF, int N>
__device__ __forceinline__ void tmem_ld16x2_at(uint32_t taddr, uint32_t (&r)[N]) {
    static_assert(OFF + 32 <= N, "range");
    asm volatile(
        "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32], 64;"
        : "=r"(r[OFF + 0]), "=r"(r[OFF + 1]), "=r"(r[OFF + 2]), "=r"(r[OFF + 3]), "=r"(r[OFF + 4]),
          "=r"(r[OFF + 5]), "=r"(r[OFF + 6]), "=r"(r[OFF + 7]), "=r"(r[OFF + 8]), "=r"(r[OFF + 9]),
          "=r"(r[OFF + 10]), "=r"(r[OFF + 11]), "=r"(r[OFF + 12]), "=r"(r[OFF + 13]), "=r"(r[OFF + 14]),
          "=r"(r[OFF + 15]), "=r"(r[OFF + 16]), "=r"(r[OFF + 17]), "=r"(r[OFF + 18]), "=r"(r[OFF + 19]),
          "=r"(r[OFF + 20]), "=r"(r[OFF + 21]), "=r"(r[OFF + 22]), "=r"(r[OFF + 23]), "=r"(r[OFF + 24]),
          "=r"(r[OFF + 25]), "=r"(r[OFF + 26]), "=r"(r[OFF + 27]), "=r"(r[OFF + 28]), "=r"(r[OFF + 29]),
          "=r"(r[OFF + 30]), "=r"(r[OFF + 31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16x2_16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], 64, {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

template <bool EXPCAST, bool PROBE>
__device__ void softmax_role(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort, uint32_t tmem,
                             int qtile, int head, int quarter, int sub, int lane) {
    // warp (quarter, sub) owns rows quarter*32 + sub*16 + [0, 16); lanes t and
    // t + 16 share row t, columns [0, 64) and [64, 128)
    const int hs = lane >> 4;
    const int row = quarter * 32 + sub * 16 + (lane & 15);
    const int64_t grow = (int64_t)qtile * kBM + row;
    int qb = (int)(grow / p.q_block);
    if (qb >= p.nqb) qb = p.nqb - 1;
    const float qs_scale = p.q_scale[(int64_t)head * p.nqb + qb];
    const float* ksp = p.k_scale + (int64_t)head * p.nkb;
    float* st_alpha = reinterpret_cast<float*>(smem + kOffStats);
    float* st_mass = st_alpha + 4 * 128;                       // [4][2][128]
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32 + sub * 16) << 16);
    const int kstep = p.kq / kBN;
    int kidx = 0, kcnt = 0;
    float m = -INFINITY;
    for (int j = 0; j < p.T; ++j) {
        const int b = j & 1;
        const float ks = __ldg(ksp + kidx);
        if (++kcnt == kstep) {          // K scale block changes every kq / 128 tiles
            kcnt = 0;
            ++kidx;
        }
        if (!mbar_wait(&B.s_full[b], (j >> 1) & 1, abort)) break;
        tc_fence_after();
        uint32_t r[64];
        const uint32_t ts = trow + kColS + b * kBN;
        tmem_ld16x2_at<0>(ts, r);
        tmem_ld16x2_at<32>(ts + 32, r);
        tmem_wait_ld();
        if (j == p.T - 1) {             // only the last tile can be partial
            const int nvalid = (int)(p.sk - (int64_t)j * kBN) - 64 * hs;
            if (nvalid < 64) {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (i >= nvalid) r[i] = 0xff800000u;   // -inf: masked key
            }
        }
        float mx[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) mx[k] = fmaxf(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
#pragma unroll
        for (int t = 1; t < 8; ++t)
#pragma unroll
            for (int k = 0; k < 4; ++k)
                mx[k] = fmax3(mx[k], __uint_as_float(r[8 * t + 2 * k]), __uint_as_float(r[8 * t + 2 * k + 1]));
        const float pmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]);
        const float omax = __shfl_xor_sync(0xffffffffu, pmax, 16);   // the other half of the row
        const float rmax = fmaxf(pmax, omax);
        const float c = __fmul_rn(__fmul_rn(qs_scale, ks), p.scale);
        const float m_new = fmaxf(m, __fmul_rn(rmax, c));
        // alpha = e^(m - m_new) as 2^((m - m_new) log2 e) on MUFU.EX2: a few
        // FP32 ulps from expf, inside the output tolerance, and exactly 1
        // when the maximum did not move (the correction skips its rescale then)
        const float alpha = ex2_ftz(__fmul_rn(m - m_new, kLog2e));
        float A, Bc;
        // A is kept at or above the smallest normal float: a masked key (-inf)
        // times A must stay -inf (code 0, no mass), never -inf * 0 = NaN.  When
        // c underflows that far, every logit s * c is below 2^-100 and the
        // codes come out as for A = 0, as in the reference.
        if (EXPCAST) {
            // in units of 2^-24 throughout: scaling by a power of two is exact,
            // so this is the unscaled computation times 2^-24, bit for bit
            A = fmaxf(__fmul_rn(c, kC1 * kTwoM24), kMinNormal);
            Bc = __fsub_rn(kC2 * kTwoM24, __fmul_rn(m_new, kC1 * kTwoM24));
            const float umax = fmaf(rmax, A, Bc);
            if (umax > 120.25f * kTwoM24) Bc = __fsub_rn(Bc, __fsub_rn(umax, kC2 * kTwoM24));
        } else {
            A = fmaxf(__fmul_rn(c, kLog2e), kMinNormal);
            Bc = __fsub_rn(8.0f, __fmul_rn(m_new, kLog2e));
        }
        const float2 AA = make_float2(A, A), BB = make_float2(Bc, Bc);
        float ms[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        uint32_t pk[16];
#pragma unroll
        for (int w = 0; w < 16; ++w) {
            const float2 g01 = ffma2(make_float2(__uint_as_float(r[4 * w]), __uint_as_float(r[4 * w + 1])), AA, BB);
            const float2 g23 =
                ffma2(make_float2(__uint_as_float(r[4 * w + 2]), __uint_as_float(r[4 * w + 3])), AA, BB);
            if (EXPCAST) {
                const uint32_t h01 = cvt_relu_f16x2(g01.y, g01.x);   // integer codes as f16 subnormals
                const uint32_t h23 = cvt_relu_f16x2(g23.y, g23.x);
                pk[w] = __byte_perm(h01, h23, 0x6420);
                // code << 7 read as f16 is exactly decode(code) / 256
                add_f16x2_to_f32(ms[0], ms[1], h01 << 7);
                add_f16x2_to_f32(ms[2], ms[3], h23 << 7);
            } else {
                const float e0 = ex2_ftz(g01.x), e1 = ex2_ftz(g01.y), e2 = ex2_ftz(g23.x), e3 = ex2_ftz(g23.y);
                // packed adds: each lane is the same round-to-nearest FP32 add
                const float2 s01 = fadd2(make_float2(ms[0], ms[1]), make_float2(e0, e1));
                const float2 s23 = fadd2(make_float2(ms[2], ms[3]), make_float2(e2, e3));
                ms[0] = s01.x; ms[1] = s01.y; ms[2] = s23.x; ms[3] = s23.y;
                pk[w] = e4m3x2(e0, e1) | (e4m3x2(e2, e3) << 16);
            }
        }
        // ExpCast: ms holds sum(p) = mass; scale to units of 256.  Otherwise
        // ms already holds sum(p * 256).
        float M = __fadd_rn(__fadd_rn(ms[0], ms[1]), __fadd_rn(ms[2], ms[3]));
        if (EXPCAST) M = __fmul_rn(M, 256.0f);
        if (PROBE && head == p.pr_head && qtile == p.pr_qtile && j >= p.pr_begin && j < p.pr_begin + p.pr_count) {
            const int64_t t = j - p.pr_begin;
            float* lg = p.pr_logits + (t * 128 + row) * 128 + hs * 64;
            uint32_t* cd = reinterpret_cast<uint32_t*>(p.pr_codes + (t * 128 + row) * 128 + hs * 64);
#pragma unroll
            for (int i = 0; i < 64; ++i) lg[i] = __uint_as_float(r[i]);
#pragma unroll
            for (int w = 0; w < 16; ++w) cd[w] = pk[w];
            if (hs == 0) {
                float* rs = p.pr_rowstat + (t * 128 + row) * 4;
                rs[0] = m_new; rs[1] = A; rs[2] = Bc; rs[3] = alpha;
            }
        }
        // P_j over this thread's own (already read) S_j columns: 4 codes per
        // 32-bit column, the A-operand layout of the PV MMA
        tmem_st16x2_16(ts, pk);
        const int slot = j & 3;
        if (j >= 4 && !mbar_wait(&B.st_free[slot], ((j >> 2) - 1) & 1, abort)) break;
        if (hs == 0) st_alpha[slot * 128 + row] = alpha;
        st_mass[(slot * 2 + hs) * 128 + row] = M;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        mbar_arrive_if(&B.p_full[b], lane == 0);
        mbar_arrive_if(&B.st_full[slot], lane == 0);
        m = m_new;
    }
}

template <bool HAS_MEAN>
__device__ void correction_role(const Params& p, uint8_t* smem, const Bars& B, volatile int* abort,
                                uint32_t tmem, int qtile, int head, int quarter, int half, int lane) {
    const int row = quarter * 32 + lane;
    const float* st_alpha = reinterpret_cast<const float*>(smem + kOffStats);
    const float* st_mass = st_alpha + 4 * 128;          // [4][2][128]
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const int c0 = half * 64;
    float2 acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.0f, 0.0f);
    float den = 0.0f;
    bool done = true;
    for (int j = 0; j < p.T; ++j) {
        const int b = j & 1, slot = j & 3, s = j % kMetaSlots;
        if (!mbar_wait(&B.o_full[b], (j >> 1) & 1, abort) ||
            !mbar_wait(&B.st_full[slot], (j >> 2) & 1, abort) ||
            !mbar_wait(&B.meta_full[s], (j / kMetaSlots) & 1, abort)) {
            done = false;
            break;
        }
        tc_fence_after();
        const float alpha = st_alpha[slot * 128 + row];
        const float M = __fadd_rn(st_mass[(slot * 2) * 128 + row], st_mass[(slot * 2 + 1) * 128 + row]);
        __syncwarp();
        mbar_arrive_if(&B.st_free[slot], lane == 0);
        const float4* meta = reinterpret_cast<const float4*>(smem + kOffMeta + s * kMetaBytes);
        const bool rescale = __any_sync(0xffffffffu, alpha != 1.0f);
        const float2 aa = make_float2(alpha, alpha), MM = make_float2(M, M);
        const uint32_t to = trow + kColO + b * 128 + c0;
        if (rescale) {      // warp-uniform; alpha == 1 leaves acc unchanged
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = fmul2(acc[i], aa);
        }
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
            uint32_t o[32];
            tmem_ld32_at<0>(to + 32 * ch, o);
            tmem_wait_ld();
            if (ch == 1) {
                tc_fence_before();
                __syncwarp();
                mbar_arrive_if(&B.o_free[b], lane == 0);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 vs = meta[(c0 >> 2) + 8 * ch + q];
                float4 mu = make_float4(0.f, 0.f, 0.f, 0.f);
                if (HAS_MEAN) mu = meta[32 + (c0 >> 2) + 8 * ch + q];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = 16 * ch + 2 * q + h;
                    const int k = 4 * q + 2 * h;
                    float2 x = make_float2(__uint_as_float(o[k]), __uint_as_float(o[k + 1]));
                    const float2 v2 = h ? make_float2(vs.z, vs.w) : make_float2(vs.x, vs.y);
                    if (HAS_MEAN) x = ffma2(MM, h ? make_float2(mu.z, mu.w) : make_float2(mu.x, mu.y), x);
                    acc[i] = ffma2(x, v2, acc[i]);
                }
            }
        }
        den = __fadd_rn(__fmul_rn(alpha, den), M);
        __syncwarp();
        mbar_arrive_if(&B.meta_empty[s], lane == 0);
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
                const float2 a = acc[4 * q + e];
                __nv_bfloat162 h2 = __floats2bfloat162_rn(__fdiv_rn(a.x, den), __fdiv_rn(a.y, den));
                w[e] = *reinterpret_cast<uint32_t*>(&h2);
            }
            dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) {
        const int col = c0 + i;
        if (col >= p.dv) break;
        const float val = __fdiv_rn((i & 1) ? acc[i >> 1].y : acc[i >> 1].x, den);
        if (p.out_dtype == VCB_BF16) static_cast<__nv_bfloat16*>(p.out)[base + col] = __float2bfloat16_rn(val);
        else if (p.out_dtype == VCB_F16) static_cast<__half*>(p.out)[base + col] = __float2half_rn(val);
        else static_cast<float*>(p.out)[base + col] = val;
    }
}

template <bool EXPCAST, bool HAS_MEAN, bool PROBE>
__global__ void __launch_bounds__(kThreads, 1) attn_kernel(const __grid_constant__ Params p) {
    // The swizzled TMA/MMA layouts need a 1024-byte aligned base; the kernel
    // declares no static shared memory, so the dynamic window starts aligned.
    // Checked anyway: a misaligned window reports an error and does nothing.
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_u32(smem) & 1023u) {
        if (threadIdx.x == 0) flag_status(p.status, VCB_FLAG_INTERNAL);
        return;
    }
    const Bars B = bars_at(smem);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qtile = blockIdx.x, head = blockIdx.y;

    if (threadIdx.x == 0) {
        mbar_init(B.q_full, 1);
        for (int s = 0; s < kStages; ++s) mbar_init(&B.kv_full[s], 1);
        for (int s = 0; s < kMetaSlots; ++s) {
            mbar_init(&B.meta_full[s], 1);
            mbar_init(&B.meta_empty[s], 8);       // 8 correction warps
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&B.s_full[b], 1);
            mbar_init(&B.p_full[b], 8);
            mbar_init(&B.o_full[b], 1);
            mbar_init(&B.o_free[b], 8);           // 8 correction warps
        }
        for (int s = 0; s < 4; ++s) {
            mbar_init(&B.st_full[s], 8);
            mbar_init(&B.st_free[s], 8);
        }
        mbar_init(B.drain, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Register split of the 640 x 96 launch budget: producer/MMA group 64
    // (the unrolled MMA loop spills below that), softmax groups 96
    // (unchanged), correction groups 112; 8192 + 24576 + 28672 = 61440.
    if (warp < 4) {
        reg_dealloc<64>();
        if (warp == 0 && lane == 0) producer(p, smem, B, abort, qtile, head);
        if (warp == 1 && lane == 0) mma_issuer(p, smem, B, abort, tmem);
        if (warp == 2 && lane == 0) meta_producer(p, smem, B, abort, head);
    } else if (warp < 12) {
        softmax_role<EXPCAST, PROBE>(p, smem, B, abort, tmem, qtile, head, warp & 3, (warp - 4) >> 2, lane);
    } else {
        reg_alloc<112>();
        correction_role<HAS_MEAN>(p, smem, B, abort, tmem, qtile, head, warp & 3, (warp - 12) >> 2, lane);
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

template <bool E, bool M, bool P>
int launch(const Params& p, dim3 grid, cudaStream_t st) {
    VCB_CUDA(cudaFuncSetAttribute(attn_kernel<E, M, P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kSmemAlloc));
    attn_kernel<E, M, P><<<grid, kThreads, kSmemAlloc, st>>>(p);
    VCB_CUDA(cudaGetLastError());
    return VCB_OK;
}

// Self-test of the bounded waits, with no GPU fault involved.  One CTA sets up
// what an attention CTA holds when a wait expires: tensor memory, a bulk copy
// in flight and a tcgen05 commit to drain.  Lane 0 of each of the four warps
// then waits through mbar_wait on a barrier phase that only `complete`
// finishes.  Without it the first wait to pass kWaitLimitNs raises the abort
// flag and the other warps give up on seeing it.  The CTA then runs the
// attention kernel's teardown: drain the copy and the commit, free tensor
// memory, set VCB_FLAG_TIMEOUT.  report: [0] waits that gave up, [1] waits
// that completed, [2] 1 when the drained copy equals src, [3] elapsed ms.
__global__ void __launch_bounds__(128, 1)
    wait_selftest_kernel(int complete, const int32_t* __restrict__ src, int32_t* status, int32_t* report) {
    __shared__ __align__(128) int32_t buf[256];
    __shared__ __align__(8) uint64_t bars[3];   // 0: the awaited phase, 1: the copy, 2: the tcgen05 drain
    __shared__ int abort_flag;
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t t0 = globaltimer();
    if (threadIdx.x == 0) {
        for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_slot, 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int* abort = &abort_flag;
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bars[1], (uint32_t)sizeof(buf));
        bulk_load(buf, src, (uint32_t)sizeof(buf), &bars[1]);
        if (complete) mbar_arrive(&bars[0]);
    }
    if (lane == 0) atomicAdd(&report[mbar_wait(&bars[0], 0, abort) ? 1 : 0], 1);
    if (threadIdx.x == 0) {
        mma_commit(&bars[2]);            // no MMA issued: arrives once earlier tcgen05 work is done
        drain_wait(&bars[2], 0);
    }
    drain_wait(&bars[1], 0);             // no copy may land after the CTA exits
    int same = 1;
    for (int i = threadIdx.x; i < 256; i += 128) same &= buf[i] == src[i];
    tc_fence_before();
    same = __syncthreads_and(same);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
    if (threadIdx.x == 0) {
        report[2] = same;
        report[3] = (int32_t)((globaltimer() - t0) / 1000000ull);
        if (*abort) flag_status(status, VCB_FLAG_TIMEOUT);
    }
}

}  // namespace

int attn_run(const vcb_attn_args* a, const vcb_attn_probe* probe, cudaStream_t st) {
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
    p.out_dtype = a->out_dtype;
    p.scale = a->scale;
    const dim3 grid((unsigned)((a->sq + kBM - 1) / kBM), (unsigned)a->heads);
    if (probe) {
        p.pr_logits = probe->logits;
        p.pr_codes = probe->codes;
        p.pr_rowstat = probe->rowstat;
        p.pr_head = (int)probe->head;
        p.pr_qtile = (int)probe->q_tile;
        p.pr_begin = probe->tile_begin;
        p.pr_count = probe->tile_count;
        if (a->expcast)
            return a->has_mean ? launch<true, true, true>(p, grid, st) : launch<true, false, true>(p, grid, st);
        return a->has_mean ? launch<false, true, true>(p, grid, st) : launch<false, false, true>(p, grid, st);
    }
    if (a->expcast)
        return a->has_mean ? launch<true, true, false>(p, grid, st) : launch<true, false, false>(p, grid, st);
    return a->has_mean ? launch<false, true, false>(p, grid, st) : launch<false, false, false>(p, grid, st);
}

int wait_selftest_run(int complete, const void* src, int32_t* status, int32_t* report, cudaStream_t st) {
    VCB_CUDA(cudaMemsetAsync(report, 0, 4 * sizeof(int32_t), st));
    wait_selftest_kernel<<<1, 128, 0, st>>>(complete, static_cast<const int32_t*>(src), status, report);
    VCB_CUDA(cudaGetLastError());
    return VCB_OK;
}

}  // namespace vcb
