// Fused VC-Attention forward for the exp modes (fp8_control, v_smooth:
// P8 = e4m3(exp(S - m) * 256) with the FP32 row mass of the unrounded
// probabilities, core.py:326-332) on pairs of SMs.  The ExpCast modes run on
// the kernel of vcb_attn.cu; the two share the pair machinery of
// vcb_attn_pair.cuh.
//
// Work decomposition as in vcb_attn.cu: two CTAs form a cluster and share
// every KV tile, CTA rank r owns query tile 2p + r of a head (128 rows), and
// the pair's MMAs are tcgen05.mma.cta_group::2 with M = 256, issued by one
// thread of the even CTA.  Each CTA loads its half of every K tile (64 keys),
// V tile (64 channels) and mean-operand tile with ordinary (non-multicast)
// TMA loads that report to the even CTA's barrier.
//
// Roles per CTA (640 threads, register budgets rebalanced with setmaxnreg):
//   warp 0      TMA producer: Q tile of each item (2 buffers), then this
//               CTA's halves of K / V / mean-operand tiles into an 8-stage ring.
//   warps 1, 3  MMA issuers (even CTA, one thread each; warp 1 takes the
//               even tiles g and buffers S0 / O0, warp 3 the odd ones and
//               S1 / O1): S_g = Q8 K8_g^T and O_g = P_g R_g (+ M_g mu_g).
//   warp 2      the per-tile V scales into a 16-slot ring.
//   warps 4-11  softmax, two threads of one warp per query row (64 scores
//               each): row max, alpha, exp + E4M3(p * 256), the FP32 row
//               mass; P_g back over its own S_g columns, and with V-Smooth
//               the row mass as three bf16 pieces beside it.
//   warps 12-19 correction, two threads per row (64 channels each):
//               acc = alpha acc + O_g vscale_g, den = alpha den + M_g;
//               epilogue acc / den in the output dtype after each item.
//
// V-mean recovery on the tensor core.  The reference adds rowmass * mu_g to
// PV / 256 before scaling by vscale_g (core.py:335).  Here one extra MMA of
// kind::f16 (K = 16, bf16 operands) adds M_g mu_g into O_g: A is the row
// mass split into bf16 pieces M1 + M2 + M3, B the stored mean mu / vscale
// split into u1 + u2 + u3 (written by the V tile kernel), and the K slots
// hold the six products Mi uj with i + j <= 4, which carry the FP32 product
// to about 2^-24.  The correction then does one packed FMA per two channels
// instead of two, and reads no means.
//
// Latency hiding: S and O are double-buffered in TMEM (S0, S1, O0, O1 use all
// 512 columns).  P_g lives in S_g's columns, so the MMA issues PV_g and then
// QK_{g+2} into the same buffer (the tensor pipe keeps issue order).  PV_g
// waits for the correction of tile g - 2 and for K_{g+2}.  The commit that
// signals PV_g done (o_full, to both CTAs) also frees K/V stage g % 8.
//
// Every mbarrier wait is bounded (vcb_common.cuh); a CTA that gives up tells
// its peer, and the pair drains and frees its tensor memory together.
#include "vcb_attn_pair.cuh"
#include <type_traits>

namespace vcb {

namespace {

constexpr int kStages = 8;
constexpr int kMetaSlots = 16;                    // per-tile vscale ring
constexpr int kThreads = 640;                     // 20 warps: 4 producer/MMA, 8 softmax, 8 correction
constexpr uint32_t kMopHalf = 64 * 32;            // this CTA's half of a mean-operand tile (2 KB)
constexpr uint32_t kStageBytes = 2 * kHalf + kMopHalf;   // 18 KB, a multiple of 1024
constexpr uint32_t kOffQ = 0;                     // Q buffers 0, 1
constexpr uint32_t kOffStages = 2 * kQBytes;
constexpr uint32_t kMetaBytes = 512;              // vscale[128]
constexpr uint32_t kOffMeta = kOffStages + kStages * kStageBytes;
constexpr int kStatSlots = 8;                     // per-tile alpha / row-mass ring
constexpr uint32_t kOffStats = kOffMeta + kMetaSlots * kMetaBytes;  // alpha[8][128], mass[8][128]
constexpr uint32_t kOffBars = kOffStats + 2 * kStatSlots * 128 * 4;
constexpr int kNumBars = 2 + 2 + 2 * kStages + 2 * kMetaSlots + 4 * 2 + 2 * kStatSlots + 2;
constexpr uint32_t kOffMisc = kOffBars + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 16;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr int kRegSplit = 32 * (4 * 80 + 8 * 88 + 8 * 112);   // the roles' setmaxnreg shares, per CTA
constexpr uint32_t kColS = 0;                     // S0, S1 (P and the row-mass pieces inside)
constexpr uint32_t kColO = 256;                   // O0, O1
constexpr uint32_t kColMass = 16;                 // row-mass operand: S_b columns [16, 24)
static_assert(kStageBytes % 1024 == 0, "swizzled tiles need 1024-byte aligned stages");

struct Params {
    CUtensorMap tm_q, tm_k, tm_v, tm_mop;
    const float* q_scale;
    const float* k_scale;
    const float* v_meta;
    void* out;
    int32_t* status;
    int64_t sq, sk;
    int dv, q_block, kq, nqb, nkb, T;
    int pairs;             // pairs of query tiles per head
    int items;             // heads * pairs
    int out_dtype;
    float scale;
    // diagnostic dump of one CTA's softmax (vcb_attention_fp8_probe)
    float* pr_logits;      // [pr_count][128][128] raw accumulators q8 . k8 (masked keys -inf)
    uint8_t* pr_codes;     // [pr_count][128][128] P bytes as stored for the PV MMA
    float* pr_rowstat;     // [pr_count][128][4]: running max after the tile, A, B, alpha
    int pr_head, pr_qtile, pr_begin, pr_count;
};

struct Bars {
    uint64_t* q_full;      // [2]  even CTA: both Q tiles of an item landed
    uint64_t* q_free;      // [2]  both: the item's QK MMAs are done with Q buffer
    uint64_t* kv_full;     // [kStages]  even CTA: both halves of K / V (/ mean operand) landed
    uint64_t* kv_empty;    // [kStages]  both: the PV of the stage's tile is done
    uint64_t* meta_full;   // [kMetaSlots]
    uint64_t* meta_empty;  // [kMetaSlots]  the 8 correction warps have read the slot
    uint64_t* s_full;      // [2]  both: QK_g done
    uint64_t* p_full;      // [2]  even CTA: P_g (and the mass pieces) of all 256 rows in TMEM
    uint64_t* o_full;      // [2]  both: PV_g done; also frees K/V stage g % kStages
    uint64_t* o_free;      // [2]  even CTA: both corrections have read O_g
    uint64_t* st_full;     // [kStatSlots]  alpha / mass of tile g
    uint64_t* st_free;     // [kStatSlots]
    uint64_t* drain;       // [2]  one per MMA thread
};

__device__ __forceinline__ Bars bars_at(uint8_t* smem) {
    uint64_t* b = reinterpret_cast<uint64_t*>(smem + kOffBars);
    Bars r;
    r.q_full = b; b += 2;
    r.q_free = b; b += 2;
    r.kv_full = b; b += kStages;
    r.kv_empty = b; b += kStages;
    r.meta_full = b; b += kMetaSlots;
    r.meta_empty = b; b += kMetaSlots;
    r.s_full = b; b += 2;
    r.p_full = b; b += 2;
    r.o_full = b; b += 2;
    r.o_free = b; b += 2;
    r.st_full = b; b += kStatSlots;
    r.st_free = b; b += kStatSlots;
    r.drain = b;
    return r;
}

__device__ __forceinline__ uint32_t cvt_bf16x2(float hi, float lo) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

template <bool HAS_MEAN>
__device__ void producer(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t rank, int c,
                         int ncl) {
    prefetch_tmap(&p.tm_q);
    prefetch_tmap(&p.tm_k);
    prefetch_tmap(&p.tm_v);
    if (HAS_MEAN) prefetch_tmap(&p.tm_mop);
    const uint32_t lead_q = peer_addr(B.q_full, 0);       // q_full[b] at + 8 b
    const uint32_t lead_kv = peer_addr(B.kv_full, 0);     // kv_full[s] at + 8 s
    const uint32_t kv_bytes = 2 * (2 * kHalf + (HAS_MEAN ? kMopHalf : 0));
    uint32_t g = 0, li = 0;
    int q_loaded = 0;          // items whose Q this CTA has requested
    uint32_t loaded = 0;       // tiles requested
    bool ok = true;
    for (int it = c; ok && it < p.items; it += ncl, ++li) {
        const int head = it / p.pairs, pair = it - head * p.pairs;
        const int qb = li & 1;
        if (li >= 2 && !wait.parked(&B.q_free[qb], ((li - 2) >> 1) & 1)) break;
        if (rank == 0) mbar_arrive_expect_tx(&B.q_full[qb], 2 * kQBytes);
        tma_load_3d_pair(smem + kOffQ + qb * kQBytes, &p.tm_q, lead_q + 8 * qb, 0, (2 * pair + (int)rank) * kBM, head);
        q_loaded = li + 1;
        for (int j = 0; j < p.T; ++j, ++g) {
            const int s = g % kStages;
            // stage s last held tile g - kStages: free once its PV is done
            if (g >= kStages && !wait.parked(&B.kv_empty[s], ((g / kStages) - 1) & 1)) {
                ok = false;
                break;
            }
            uint8_t* st = smem + kOffStages + s * kStageBytes;
            if (rank == 0) mbar_arrive_expect_tx(&B.kv_full[s], kv_bytes);
            const int row = j * kBN + 64 * (int)rank;
            tma_load_3d_pair(st, &p.tm_k, lead_kv + 8 * s, 0, row, head);
            tma_load_3d_pair(st + kHalf, &p.tm_v, lead_kv + 8 * s, 0, row, head);
            if (HAS_MEAN) tma_load_3d_pair(st + 2 * kHalf, &p.tm_mop, lead_kv + 8 * s, 0, row, head);
            loaded = g + 1;
        }
    }
    if (*wait.abort) {
        // No TMA write may land after the pair exits.  The even CTA's barriers
        // count both CTAs' bytes; the odd CTA gives its copies a bounded
        // millisecond, far longer than any copy in flight needs.
        if (rank == 0) {
            for (int b = 0; b < 2 && b < q_loaded; ++b) drain_wait(&B.q_full[b], ((q_loaded - 1 - b) >> 1) & 1);
            for (uint32_t s = 0; s < (uint32_t)kStages && s < loaded; ++s)
                drain_wait(&B.kv_full[s], ((loaded - 1 - s) / kStages) & 1);
        } else {
            const uint64_t t0 = globaltimer();
            while (globaltimer() - t0 < 1000000ull) {
            }
        }
    }
}

// The per-tile V scales (512 B) run on their own deeper ring, so a K/V stage
// is free as soon as the PV of its tile has been committed.
__device__ void meta_producer(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, int c, int ncl) {
    uint32_t g = 0, loaded = 0;
    bool ok = true;
    for (int it = c; ok && it < p.items; it += ncl) {
        const int head = it / p.pairs;
        const float* meta = p.v_meta + (int64_t)head * p.T * 256;
        for (int j = 0; j < p.T; ++j, ++g) {
            const int s = g % kMetaSlots;
            if (g >= (uint32_t)kMetaSlots && !wait.parked(&B.meta_empty[s], ((g / kMetaSlots) - 1) & 1)) {
                ok = false;
                break;
            }
            mbar_arrive_expect_tx(&B.meta_full[s], kMetaBytes);
            bulk_load(smem + kOffMeta + s * kMetaBytes, meta + (int64_t)j * 256, kMetaBytes, &B.meta_full[s]);
            loaded = g + 1;
        }
    }
    if (*wait.abort)
        for (uint32_t s = 0; s < (uint32_t)kMetaSlots && s < loaded; ++s)
            drain_wait(&B.meta_full[s], ((loaded - 1 - s) / kMetaSlots) & 1);
}

// D += A B^T with bf16 A in tensor memory and bf16 B in shared memory (K = 16)
__device__ __forceinline__ void mma2_ts_bf16(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t hi,
                                             uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .b64 db;\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], db, %4, 1;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "r"(b_lo), "r"(hi), "r"(idesc)
        : "memory");
}

// Instruction descriptor, kind::f16 with bf16 A and B (format 1 at [7,10)
// and [10,13)), F32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Shared-memory descriptor for a K-major operand laid out by a TMA load with
// 32-byte swizzle: rows of 32 bytes, 8-row atoms 256 bytes apart (SBO),
// layout type 6 = SWIZZLE_32B at [61,64), version 1 at [46,48).
__device__ __forceinline__ uint64_t smem_desc_k32(const void* p) {
    const uint64_t addr = smem_u32(p);
    return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((256ull >> 4) << 32) | (1ull << 46) | (6ull << 61);
}

// Two MMA threads of the even CTA, on different SM sub-partitions, split the
// issue work: thread X (warp 1 for X = 0, warp 3 for X = 1) owns TMEM buffers
// S_X / O_X and issues PV_g then QK_{g+2} for the tiles g of its parity, g
// running over the tiles of all items of this pair.  No accumulator is shared
// between the threads, so the tensor pipe may interleave their MMAs freely;
// each thread's own issue order keeps QK_{g+2} after the PV_g that reads P_g
// from the same buffer.  Every MMA instruction waits for issue slots next to
// the busy softmax and correction warps, so two issuers halve the per-tile
// issue latency on the critical path.  The loop is unrolled by the thread's
// two K/V stages (X and X + 2), so stage and buffer offsets are constants.
template <bool HAS_MEAN, uint32_t X>
__device__ void mma_issuer(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t tmem, int c,
                           int ncl) {
    static_assert(kStages == 8, "two issuers with four stages each");
    const uint32_t idesc = idesc_e4m3_f32(2 * kBM, kBN);
    const uint32_t idesc_mean = idesc_bf16_f32(2 * kBM, kBN);
    const uint64_t q64 = smem_desc_k128(smem + kOffQ);
    const uint32_t hi = (uint32_t)(q64 >> 32);
    const uint32_t q0lo = (uint32_t)q64;
    const uint32_t k0lo = (uint32_t)smem_desc_k128(smem + kOffStages);
    const uint64_t m64 = smem_desc_k32(smem + kOffStages + 2 * kHalf);
    const uint32_t mhi = (uint32_t)(m64 >> 32), m0lo = (uint32_t)m64;
    constexpr uint32_t kStageLo = kStageBytes >> 4, kHalfLo = kHalf >> 4, kQLo = kQBytes >> 4;
    const uint32_t T = (uint32_t)p.T;
    const uint32_t G = (uint32_t)local_items(p.items, c, ncl) * T;
    const uint32_t d = tmem + kColS + X * kBN, od = tmem + kColO + X * 128;
    // cursor of this thread's next QK: local item and tile; every item the
    // cursor leaves gets this thread's q_free arrival (count 2: both threads)
    uint32_t qli = 0, qj = X, q_waited = 0xffffffffu;
    while (qj >= T) {                   // an item of one tile holds no QK of thread 1
        qj -= T;
        commit_both(&B.q_free[qli & 1]);
        ++qli;
    }
    auto qk = [&](uint32_t s2) -> bool {
        if (qli != q_waited) {
            if (!wait(&B.q_full[qli & 1], (qli >> 1) & 1)) return false;
            tc_fence_after();
            q_waited = qli;
        }
        const uint32_t qlo = q0lo + (qli & 1) * kQLo, klo = k0lo + s2 * kStageLo;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma2_ss(d, qlo + 2 * kk, klo + 2 * kk, hi, idesc, kk > 0);
        commit_both(&B.s_full[X]);
        qj += 2;
        while (qj >= T) {               // this thread's QKs of item qli are all issued
            qj -= T;
            commit_both(&B.q_free[qli & 1]);
            ++qli;
        }
        return true;
    };
    bool ok = true;
    if (X < G) {
        ok = wait(&B.kv_full[X], 0);
        if (ok) {
            tc_fence_after();
            ok = qk(X);
        }
    }
    auto step = [&](auto S_, uint32_t g) -> bool {
        constexpr uint32_t s = decltype(S_)::value, s2 = (s + 2) % kStages;   // g % kStages
        const bool next = g + 2 < G;
        if (!wait.all(&B.p_full[X], (g >> 1) & 1, g >= 2 ? &B.o_free[X] : nullptr, ((g - 2) >> 1) & 1,
                      next ? &B.kv_full[s2] : nullptr, ((g + 2) / kStages) & 1))
            return false;
        tc_fence_after();
        const uint32_t vlo = k0lo + s * kStageLo + kHalfLo;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma2_ts(od, d + (kk >> 1) * 64 + (kk & 1) * 8, vlo + 2 * kk, hi, idesc, kk > 0);
        if (HAS_MEAN) mma2_ts_bf16(od, d + kColMass, m0lo + s * kStageLo, mhi, idesc_mean);
        commit_both(&B.o_full[X]);
        commit_both(&B.kv_empty[s]);     // the producers may refill stage s
        if (next) return qk(s2);
        return true;
    };
    for (uint32_t g = X; ok && g < G; g += 8) {
        ok = step(std::integral_constant<uint32_t, X>{}, g);
        if (ok && g + 2 < G) ok = step(std::integral_constant<uint32_t, X + 2>{}, g + 2);
        if (ok && g + 4 < G) ok = step(std::integral_constant<uint32_t, X + 4>{}, g + 4);
        if (ok && g + 6 < G) ok = step(std::integral_constant<uint32_t, X + 6>{}, g + 6);
    }
    commit_local_pair(&B.drain[X]);
    drain_wait(&B.drain[X], 0);
}

__device__ __forceinline__ void tmem_st16x2_16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x32bx2.x16.b32 [%0], 64, {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
// thread t < 16: lane base + t, columns [c, c + 4); thread t + 16: the same
// lane, columns [c + 4, c + 8): one row's 8 consecutive columns from the pair
__device__ __forceinline__ void tmem_st16x2_4_split4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c,
                                                     uint32_t d) {
    asm volatile("tcgen05.st.sync.aligned.16x32bx2.x4.b32 [%0], 4, {%1, %2, %3, %4};"
                 ::"r"(taddr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

template <bool HAS_MEAN, bool PROBE>
__device__ void softmax_role(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t tmem,
                             uint32_t rank, int c, int ncl, int quarter, int sub, int lane) {
    // warp (quarter, sub) owns rows quarter*32 + sub*16 + [0, 16); lanes t and
    // t + 16 share row t, columns [0, 64) and [64, 128)
    const int hs = lane >> 4;
    const int row = quarter * 32 + sub * 16 + (lane & 15);
    float* st_alpha = reinterpret_cast<float*>(smem + kOffStats);
    float* st_mass = st_alpha + kStatSlots * 128;               // [kStatSlots][128]
    const uint32_t lead_p = peer_addr(B.p_full, 0);            // p_full[b] at + 8 b
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32 + sub * 16) << 16);
    const int kstep = p.kq / kBN;
    uint32_t g = 0;
    for (int it = c; it < p.items; it += ncl) {
        const int head = it / p.pairs, pair = it - head * p.pairs;
        const int qtile = 2 * pair + (int)rank;
        const int64_t grow = (int64_t)qtile * kBM + row;
        int qb = (int)(grow / p.q_block);
        if (qb >= p.nqb) qb = p.nqb - 1;
        const float qs_scale = p.q_scale[(int64_t)head * p.nqb + qb];
        const float* ksp = p.k_scale + (int64_t)head * p.nkb;
        const bool probe = PROBE && head == p.pr_head && qtile == p.pr_qtile;
        int kidx = 0, kcnt = 0;
        float m = -INFINITY;
        for (int j = 0; j < p.T; ++j, ++g) {
            const uint32_t b = g & 1;
            const float ks = __ldg(ksp + kidx);
            if (++kcnt == kstep) {          // K scale block changes every kq / 128 tiles
                kcnt = 0;
                ++kidx;
            }
            const uint32_t ts = trow + kColS + b * kBN;
            const int slot = g % kStatSlots;
            // the scores of tile g, and (checked alongside) the statistics
            // slot this tile writes at its end
            if (!wait.all(&B.s_full[b], (g >> 1) & 1,
                          g >= (uint32_t)kStatSlots ? &B.st_free[slot] : nullptr, ((g / kStatSlots) - 1) & 1))
                return;
            tc_fence_after();
            uint32_t r[64];
            tmem_ld16x2_at<0>(ts, r);
            tmem_ld16x2_at<32>(ts + 32, r);
            tmem_wait_ld();
            if (j == p.T - 1) {             // only the last tile of an item can be partial
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
            const float cs = __fmul_rn(__fmul_rn(qs_scale, ks), p.scale);
            const float m_new = fmaxf(m, __fmul_rn(rmax, cs));
            // alpha = e^(m - m_new) as 2^((m - m_new) log2 e) on MUFU.EX2: a few
            // FP32 ulps from expf, inside the output tolerance, and exactly 1
            // when the maximum did not move (the correction skips its rescale then)
            const float alpha = ex2_ftz(__fmul_rn(m - m_new, kLog2e));
            // A is kept at or above the smallest normal float: a masked key (-inf)
            // times A must stay -inf (p = 0), never -inf * 0 = NaN.  p * 256 =
            // 2^(s A + Bc) with the 256 folded into Bc as + 8.
            const float A = fmaxf(__fmul_rn(cs, kLog2e), kMinNormal);
            const float Bc = __fsub_rn(8.0f, __fmul_rn(m_new, kLog2e));
            const float2 AA = make_float2(A, A), BB = make_float2(Bc, Bc);
            float ms[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            uint32_t pk[16];
#pragma unroll
            for (int w = 0; w < 16; ++w) {
                const float2 g01 =
                    ffma2(make_float2(__uint_as_float(r[4 * w]), __uint_as_float(r[4 * w + 1])), AA, BB);
                const float2 g23 =
                    ffma2(make_float2(__uint_as_float(r[4 * w + 2]), __uint_as_float(r[4 * w + 3])), AA, BB);
                const float e0 = ex2_ftz(g01.x), e1 = ex2_ftz(g01.y), e2 = ex2_ftz(g23.x), e3 = ex2_ftz(g23.y);
                // packed adds: each lane is the same round-to-nearest FP32 add
                const float2 s01 = fadd2(make_float2(ms[0], ms[1]), make_float2(e0, e1));
                const float2 s23 = fadd2(make_float2(ms[2], ms[3]), make_float2(e2, e3));
                ms[0] = s01.x; ms[1] = s01.y; ms[2] = s23.x; ms[3] = s23.y;
                pk[w] = e4m3x2(e0, e1) | (e4m3x2(e2, e3) << 16);
            }
            // ms holds sum(p * 256); the row's two halves add up to M
            const float Mh = __fadd_rn(__fadd_rn(ms[0], ms[1]), __fadd_rn(ms[2], ms[3]));
            const float M = __fadd_rn(Mh, __shfl_xor_sync(0xffffffffu, Mh, 16));
            if (probe && j >= p.pr_begin && j < p.pr_begin + p.pr_count) {
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
            // P_g over this thread's own (already read) S_g columns: 4 codes per
            // 32-bit column, the A-operand layout of the PV MMA
            tmem_st16x2_16(ts, pk);
            if (HAS_MEAN) {
                // the row mass as bf16 pieces M1 + M2 + M3 (each remainder exact
                // in FP32), in the K slots [M1, M1, M1, M2, M2, M3, 0 ...] that
                // meet [u1, u2, u3, u1, u2, u1, 0 ...] of the mean operand
                const uint32_t p1 = cvt_bf16x2(M, M);
                const float r1 = __fsub_rn(M, __uint_as_float(p1 << 16));
                const uint32_t p2 = cvt_bf16x2(r1, r1);
                const float r2 = __fsub_rn(r1, __uint_as_float(p2 << 16));
                const uint32_t w1 = __byte_perm(p1, p2, 0x5410);   // (M1, M2)
                const uint32_t w2 = cvt_bf16x2(r2, r1);              // (M2, M3)
                tmem_st16x2_4_split4(ts + kColMass, hs ? 0u : p1, hs ? 0u : w1, hs ? 0u : w2, 0u);
            }
            if (hs == 0) {
                st_alpha[slot * 128 + row] = alpha;
                st_mass[slot * 128 + row] = M;
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            mbar_arrive_cluster_if(lead_p + 8 * b, lane == 0);
            mbar_arrive_if(&B.st_full[slot], lane == 0);
            m = m_new;
        }
    }
}

__device__ void correction_role(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t tmem,
                                uint32_t rank, int c, int ncl, int quarter, int half, int lane) {
    const int row = quarter * 32 + lane;
    const float* st_alpha = reinterpret_cast<const float*>(smem + kOffStats);
    const float* st_mass = st_alpha + kStatSlots * 128;
    const uint32_t lead_o = peer_addr(B.o_free, 0);            // o_free[b] at + 8 b
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const int c0 = half * 64;
    uint32_t g = 0;
    for (int it = c; it < p.items; it += ncl) {
        const int head = it / p.pairs, pair = it - head * p.pairs;
        const int64_t grow = (int64_t)(2 * pair + (int)rank) * kBM + row;
        float2 acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = make_float2(0.0f, 0.0f);
        float den = 0.0f;
        for (int j = 0; j < p.T; ++j, ++g) {
            const uint32_t b = g & 1, slot = g % kStatSlots, s = g % kMetaSlots;
            if (!wait.all(&B.o_full[b], (g >> 1) & 1, &B.st_full[slot], (g / kStatSlots) & 1, &B.meta_full[s],
                          (g / kMetaSlots) & 1))
                return;
            tc_fence_after();
            const float alpha = st_alpha[slot * 128 + row];
            const float M = st_mass[slot * 128 + row];
            __syncwarp();
            mbar_arrive_if(&B.st_free[slot], lane == 0);
            const float4* vsp = reinterpret_cast<const float4*>(smem + kOffMeta + s * kMetaBytes);
            const bool rescale = __any_sync(0xffffffffu, alpha != 1.0f);
            const float2 aa = make_float2(alpha, alpha);
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
                    mbar_arrive_cluster_if(lead_o + 8 * b, lane == 0);
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 vs = vsp[(c0 >> 2) + 8 * ch + q];
                    const int i = 16 * ch + 2 * q;
                    acc[i] = ffma2(make_float2(__uint_as_float(o[4 * q]), __uint_as_float(o[4 * q + 1])),
                                   make_float2(vs.x, vs.y), acc[i]);
                    acc[i + 1] = ffma2(make_float2(__uint_as_float(o[4 * q + 2]), __uint_as_float(o[4 * q + 3])),
                                       make_float2(vs.z, vs.w), acc[i + 1]);
                }
            }
            den = __fadd_rn(__fmul_rn(alpha, den), M);
            __syncwarp();
            mbar_arrive_if(&B.meta_empty[s], lane == 0);
        }
        if (grow >= p.sq) continue;
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
            continue;
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
}

template <bool HAS_MEAN, bool PROBE>
__global__ void __launch_bounds__(kThreads, 1) attn_kernel(const __grid_constant__ Params p) {
    pdl_wait();
    // The swizzled TMA/MMA layouts need a 1024-byte aligned base; the kernel
    // declares no static shared memory, so the dynamic window starts aligned.
    // Checked anyway: a misaligned window reports an error and does nothing
    // (both CTAs of a pair see the same offset, so both return here).
    extern __shared__ __align__(1024) uint8_t smem[];
    if (smem_u32(smem) & 1023u) {
        if (threadIdx.x == 0) flag_status(p.status, VCB_FLAG_INTERNAL);
        return;
    }
    const Bars B = bars_at(smem);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int c = (int)(blockIdx.x >> 1), ncl = (int)(gridDim.x >> 1);

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&B.q_full[i], 1);
            mbar_init(&B.q_free[i], 2);           // both MMA threads
            mbar_init(&B.drain[i], 1);
            mbar_init(&B.s_full[i], 1);
            mbar_init(&B.p_full[i], 16);          // 8 softmax warps in each CTA
            mbar_init(&B.o_full[i], 1);
            mbar_init(&B.o_free[i], 16);          // 8 correction warps in each CTA
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&B.kv_full[s], 1);
            mbar_init(&B.kv_empty[s], 1);
        }
        for (int s = 0; s < kMetaSlots; ++s) {
            mbar_init(&B.meta_full[s], 1);
            mbar_init(&B.meta_empty[s], 8);
        }
        for (int s = 0; s < kStatSlots; ++s) {
            mbar_init(&B.st_full[s], 8);
            mbar_init(&B.st_free[s], 8);
        }
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();        // both CTAs' barriers are initialised before any remote arrive or copy
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const Waiter wait{abort, peer_addr(const_cast<int*>(abort), rank ^ 1u)};

    // Register split of the 640 x 96 launch budget (ptxas allocates each
    // role's code within its share): producer/MMA group 80 (the unrolled MMA
    // loop with its item cursor spills below 72), softmax groups 88,
    // correction groups 112; 10240 + 22528 + 28672 = 61440.
    if (warp < 4) {
        reg_dealloc<80>();
        if (warp == 0 && lane == 0) producer<HAS_MEAN>(p, smem, B, wait, rank, c, ncl);
        if (warp == 1 && lane == 0 && rank == 0) mma_issuer<HAS_MEAN, 0>(p, smem, B, wait, tmem, c, ncl);
        if (warp == 3 && lane == 0 && rank == 0) mma_issuer<HAS_MEAN, 1>(p, smem, B, wait, tmem, c, ncl);
        if (warp == 2 && lane == 0) meta_producer(p, smem, B, wait, c, ncl);
    } else if (warp < 12) {
        reg_dealloc<88>();
        softmax_role<HAS_MEAN, PROBE>(p, smem, B, wait, tmem, rank, c, ncl, warp & 3, (warp - 4) >> 2, lane);
    } else {
        reg_alloc<112>();
        correction_role(p, smem, B, wait, tmem, rank, c, ncl, warp & 3, (warp - 12) >> 2, lane);
    }
    tc_fence_before();
    __syncwarp();
    // No CTA leaves while its peer may still arrive on its barriers, read its
    // shared memory through an MMA or hold its tensor memory.
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort) flag_status(p.status, VCB_FLAG_TIMEOUT);
}

template <bool M, bool P>
int launch(const Params& p, cudaStream_t st) {
    static int max_clusters[64][8] = {};
    return launch_pairs(attn_kernel<M, P>, p, p.items, kThreads, kSmemAlloc, kRegSplit, max_clusters,
                        (M ? 2 : 0) | (P ? 1 : 0), st);
}

}  // namespace

int attn_exp_run(const vcb_attn_args* a, const vcb_attn_probe* probe, cudaStream_t st) {
    if (a->has_mean && !a->v_mean_op)
        return fail(VCB_ERR_INVALID_ARGUMENT, "has_mean needs the mean operand (v_mean_op) of vcb_prepare_v");
    if (a->has_mean && (reinterpret_cast<uintptr_t>(a->v_mean_op) & 15u))
        return fail(VCB_ERR_INVALID_ARGUMENT, "v_mean_op must be 16-byte aligned");
    Params p;
    memset(&p, 0, sizeof(p));
    const int64_t sq_pad = vcb_padded_rows(a->sq, a->q_block);
    const int64_t sk_pad = vcb_padded_rows(a->sk, a->k_quant_block);
    const int64_t T = (a->sk + kBN - 1) / kBN;
    const int64_t qtiles = (a->sq + kBM - 1) / kBM;
    const int64_t pairs = (qtiles + 1) / 2;
    const int64_t items = pairs * a->heads;
    // the per-pair tile counter is 32-bit: items of one pair x tiles < 2^31
    // (the grid never has fewer than one pair per 2^31 / T items)
    if (items >= (1ll << 31) || ((items + 73) / 74) * T >= (1ll << 31))
        return fail(VCB_ERR_INVALID_ARGUMENT, "problem too large for the attention kernel's tile counters");
    int rc = make_map(&p.tm_q, a->q8, 128, (uint64_t)sq_pad, (uint64_t)a->heads, kBM);
    if (!rc) rc = make_map(&p.tm_k, a->k8, 128, (uint64_t)sk_pad, (uint64_t)a->heads, 64);
    if (!rc) rc = make_map(&p.tm_v, a->v8, 128, (uint64_t)T * 128, (uint64_t)a->heads, 64);
    if (!rc && a->has_mean) rc = make_map(&p.tm_mop, a->v_mean_op, 32, (uint64_t)T * 128, (uint64_t)a->heads, 64);
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
    p.T = (int)T;
    p.pairs = (int)pairs;
    p.items = (int)items;
    p.out_dtype = a->out_dtype;
    p.scale = a->scale;
    if (probe) {
        p.pr_logits = probe->logits;
        p.pr_codes = probe->codes;
        p.pr_rowstat = probe->rowstat;
        p.pr_head = (int)probe->head;
        p.pr_qtile = (int)probe->q_tile;
        p.pr_begin = probe->tile_begin;
        p.pr_count = probe->tile_count;
        return a->has_mean ? launch<true, true>(p, st) : launch<false, true>(p, st);
    }
    return a->has_mean ? launch<true, false>(p, st) : launch<false, false>(p, st);
}

}  // namespace vcb
