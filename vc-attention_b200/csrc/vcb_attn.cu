// Fused VC-Attention forward for sm_100a on pairs of SMs.
//
// Replaces the reference's host loop over heads x Q tiles x KV tiles
// (kernels.cu:313-330: a cuBLASLt E4M3 GEMM for S, softmax_update, a second
// GEMM for PV and accumulate, all through HBM scratch) with one persistent
// kernel that keeps every intermediate on chip.
//
// Work decomposition.  Two CTAs form a cluster and share every KV tile: CTA
// rank r of the pair owns query tile 2p + r of a head (128 rows), and the
// pair's MMAs are tcgen05.mma.cta_group::2 with M = 256: one instruction,
// issued by one thread of the even CTA, multiplies both CTAs' rows.  Each CTA
// loads only its half of every K tile (64 keys) and its share of every V tile
// (channels 0..71 or 72..127), with ordinary (non-multicast) TMA loads that
// report to the even CTA's barrier.  The grid holds as many pairs as fit on
// the GPU at once, and each pair walks the (head, pair-of-query-tiles) items
// c, c + clusters, ... in order, so the K/V of one or two heads are in L2 at
// a time.  Barrier phases run on across items; the prologue and epilogue of
// consecutive items overlap.
//
// Roles per CTA (384 threads, register budgets rebalanced with setmaxnreg):
//   warp 0      TMA producer: this CTA's Q tile of each item (2 buffers),
//               then its share of K / V tiles into an 8-stage ring.
//   warp 1      QK issuer (even CTA, one thread): S_g = Q8 K8_g^T into the
//               one S buffer once the softmax has read S_{g-1}.
//   warp 3      PV issuer (even CTA, one thread): O_b = P_g [V8_g | 1],
//               b = g % 2; both with cta_group::2.
//   warp 2      the per-tile V scales and stored means into a 16-slot ring.
//   warps 4-7   softmax, one thread per query row (128 scores): row max,
//               alpha, the ExpCast encode (one packed FMA per pair of
//               scores; the f16-subnormal conversion rounds to the integer
//               code and clamps it at zero); P_g into P_b.
//   warps 8-11  correction, one thread per row (128 channels):
//               acc = alpha acc + (O + M u) vscale with u = mu / vscale,
//               den = alpha den + M;
//               epilogue acc / den in the output dtype after each item.
//
// Row mass on the tensor core.  The PV MMA has N = 144: the odd CTA's B rows
// 56..71 of every stage hold E4M3 ones, so O columns 128..143 each receive
// sum(P) of the row, the ExpCast row mass of decoded probabilities
// (core.py:330-332), from the same products as PV.  The softmax then only
// encodes.  (The exp modes, whose row mass is the FP32 sum of unrounded
// probabilities, run on the kernel of vcb_attn_exp.cu.)
//
// Latency hiding: TMEM holds one S buffer, two O buffers with their mass
// columns and two compact P buffers (480 of 512 columns).  The softmax
// releases S (s_free) as soon as its row is in registers, so QK_{g+1} runs
// during tile g's encode.  PV_g waits for P_g, for the corrections' read of
// O_b from tile g - 2 and for its stage; the softmax overwrites P_b only after
// PV_{g-2} has read it.  The commit that signals PV_g done (o_full, to both
// CTAs) lets the corrections read O_b; another frees K/V stage g % 8.  In the
// combined mode the chain PV_g -> the corrections' read of O_b -> PV_{g+2} is
// on the critical path, so with V-Smooth the correction prefetches O's
// chunks and only one TMEM load latency comes before the release.
//
// Numerical contract (core.py:307-341): S = (q8 . k8) * qs * ks * scale;
// ExpCast code = rne(clamp(fma(S - m, 8 log2 e, 119.65), 0, 120)) viewed as
// E4M3 with a 1/256 scale, row mass = sum of decoded P; V-mean recovery adds
// rowmass * mu / vscale to PV before the scale and is rescaled with the
// running max.  The accumulators are kept in units of 256 (acc256 = 256 acc,
// den256 = 256 den); 256 is a power of two, so no rounding changes.  Every
// mbarrier wait is bounded (vcb_common.cuh); a CTA that gives up tells its
// peer, and the pair drains and frees its tensor memory together.
#include "vcb_attn_pair.cuh"
#include <type_traits>

namespace vcb {

namespace {

constexpr int kStages = 8;
constexpr int kMetaSlots = 16;                    // per-tile vscale ring
constexpr int kThreads = 384;                     // 12 warps: 4 producer/MMA, 4 softmax, 4 correction
// The PV MMA's B operand: 72 rows of 128 keys in each CTA (N = 144).  The
// even CTA loads V channels 0..71, the odd CTA channels 72..127 into rows
// 0..55 and keeps E4M3 ones in rows 56..71, so O columns 0..127 are the 128
// channels in order and columns 128..143 each hold the row mass sum(P).
constexpr int kVRows0 = 72, kVRows1 = 56;         // V channels loaded by the even / odd CTA
constexpr uint32_t kVBytes = 72 * 128;            // one CTA's B rows of a stage (9 KB)
constexpr uint32_t kStageBytes = kHalf + kVBytes; // 17 KB, a multiple of 1024
constexpr uint32_t kOffQ = 0;                     // Q buffers 0, 1
constexpr uint32_t kOffStages = 2 * kQBytes;
constexpr uint32_t kMetaBytes = 1024;             // vscale[128], stored mean mu / vscale [128]
constexpr uint32_t kOffMeta = kOffStages + kStages * kStageBytes;
constexpr int kStatSlots = kMetaSlots;            // per-tile alpha ring, as deep as the meta ring
constexpr uint32_t kOffStats = kOffMeta + kMetaSlots * kMetaBytes;  // alpha[8][128]
constexpr uint32_t kOffBars = kOffStats + kStatSlots * 128 * 4;
constexpr int kNumBars = 2 + 2 + 2 * kStages + 2 * kMetaSlots + 5 * 2 + kStatSlots + 2;
constexpr uint32_t kOffMisc = kOffBars + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 16;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;
constexpr uint32_t kTmemCols = 512;
// the roles' setmaxnreg shares, per CTA (the correction's is 224 with V-Smooth)
constexpr int reg_split(bool has_mean) { return 32 * (4 * 80 + 4 * 192 + 4 * (has_mean ? 224 : 192)); }
// Tensor memory: one S buffer, and two of P (the E4M3 codes, 4 per column)
// and O (128 channels, then 16 columns of row mass).  The D operands sit at
// multiples of 64 columns.
constexpr uint32_t kColS = 0;
constexpr uint32_t kColO0 = 128, kColO1 = 320;
constexpr uint32_t kColP0 = 272, kColP1 = 464;
constexpr uint32_t kColMass = 128;                // the row-mass column inside O_b
constexpr int kPvN = 144;                         // N of the PV MMA with the row-mass columns
static_assert(kColS + 128 <= kColO0 && kColO0 + kPvN <= kColP0 && kColP0 + 32 <= kColO1 &&
                  kColO1 + kPvN <= kColP1 && kColP1 + 32 <= kTmemCols,
              "S, O0, P0, O1 and P1 must not overlap in the allocated columns");
static_assert(kStageBytes % 1024 == 0, "swizzled tiles need 1024-byte aligned stages");
static_assert(kVRows0 + kVRows1 == 128 && kVRows1 % 8 == 0 && 2 * kVRows0 == kPvN, "V split");

struct Params {
    CUtensorMap tm_q, tm_k, tm_v0, tm_v1;      // V boxes of kVRows0 / kVRows1 channel rows
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
    uint64_t* meta_empty;  // [kMetaSlots]  the correction warps have read the tile's meta and alpha slots
    uint64_t* s_full;      // [1]  both: QK_g done
    uint64_t* s_free;      // [1]  even CTA: the softmax of all 256 rows has read S_g
    uint64_t* p_full;      // [2]  even CTA: P_g of all 256 rows in P_b, b = g % 2
    uint64_t* o_full;      // [2]  both: PV_g done, for the tiles g of parity b
    uint64_t* o_free;      // [2]  even CTA: both corrections have read O for a tile of parity b
    uint64_t* st_full;     // [kStatSlots]  alpha of tile g (freed by meta_empty: one release per tile)
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
    r.s_free = b; b += 2;
    r.p_full = b; b += 2;
    r.o_full = b; b += 2;
    r.o_free = b; b += 2;
    r.st_full = b; b += kStatSlots;
    r.drain = b;
    return r;
}

__device__ void producer(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t rank, int c,
                         int ncl) {
    const CUtensorMap* tm_v = rank ? &p.tm_v1 : &p.tm_v0;
    const int v_row0 = rank ? kVRows0 : 0;               // first V channel this CTA loads
    prefetch_tmap(&p.tm_q);
    prefetch_tmap(&p.tm_k);
    prefetch_tmap(tm_v);
    const uint32_t lead_q = peer_addr(B.q_full, 0);       // q_full[b] at + 8 b
    const uint32_t lead_kv = peer_addr(B.kv_full, 0);     // kv_full[s] at + 8 s
    const uint32_t kv_bytes = 2 * kHalf + 128 * 128;      // both K halves, all 128 V channel rows
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
            tma_load_3d_pair(st, &p.tm_k, lead_kv + 8 * s, 0, j * kBN + 64 * (int)rank, head);
            tma_load_3d_pair(st + kHalf, tm_v, lead_kv + 8 * s, 0, j * 128 + v_row0, head);
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

// The per-tile V scales (and with V-Smooth the stored means u = mu / vscale,
// core.py:114) run on their own deeper ring, so a K/V stage is free as soon
// as the PV of its tile has been committed.
template <bool HAS_MEAN>
__device__ void meta_producer(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, int c, int ncl) {
    constexpr uint32_t bytes = HAS_MEAN ? 1024 : 512;
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
            mbar_arrive_expect_tx(&B.meta_full[s], bytes);
            bulk_load(smem + kOffMeta + s * kMetaBytes, meta + (int64_t)j * 256, bytes, &B.meta_full[s]);
            loaded = g + 1;
        }
    }
    if (*wait.abort)
        for (uint32_t s = 0; s < (uint32_t)kMetaSlots && s < loaded; ++s)
            drain_wait(&B.meta_full[s], ((loaded - 1 - s) / kMetaSlots) & 1);
}

// Two MMA threads of the even CTA, on different SM sub-partitions, split the
// issue work: warp 1 issues every QK, warp 3 every PV, g running over the
// tiles of all items of this pair.  They share no tensor memory (QK writes S;
// PV reads P_b and writes O_b), so the tensor pipe may interleave their MMAs
// freely.  Every MMA instruction waits for issue slots next to the busy
// softmax and correction warps, so each thread's stream is kept short.

// S_g = Q8 K8_g^T into the one S buffer, as soon as K_g has landed and the
// softmax has read S_{g-1} into registers.  The q_free commit after an item's
// last QK frees its Q buffer once those MMAs complete.
__device__ void qk_issuer(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t tmem, int c,
                          int ncl) {
    const uint32_t idesc = idesc_e4m3_f32(2 * kBM, kBN);
    const uint64_t q64 = smem_desc_k128(smem + kOffQ);
    const uint32_t hi = (uint32_t)(q64 >> 32);
    const uint32_t q0lo = (uint32_t)q64;
    const uint32_t k0lo = (uint32_t)smem_desc_k128(smem + kOffStages);
    constexpr uint32_t kStageLo = kStageBytes >> 4, kQLo = kQBytes >> 4;
    const uint32_t T = (uint32_t)p.T;
    const int nitems = local_items(p.items, c, ncl);
    const uint32_t d = tmem + kColS;
    uint32_t g = 0;
    bool ok = true;
    for (int li = 0; ok && li < nitems; ++li) {
        if (!wait(&B.q_full[li & 1], (li >> 1) & 1)) break;
        const uint32_t qlo = q0lo + (li & 1) * kQLo;
        for (uint32_t j = 0; j < T; ++j, ++g) {
            const uint32_t s = g % kStages;
            if (!wait.all(&B.kv_full[s], (g / kStages) & 1, g >= 1 ? &B.s_free[0] : nullptr, (g - 1) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t klo = k0lo + s * kStageLo;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) mma2_ss(d, qlo + 2 * kk, klo + 2 * kk, hi, idesc, kk > 0);
            commit_both(&B.s_full[0]);
        }
        if (ok) commit_both(&B.q_free[li & 1]);
    }
    commit_local_pair(&B.drain[0]);
    drain_wait(&B.drain[0], 0);
}

// O_b = P_g [V8_g | 1] with b = g % 2 (N = 144).  PV_g
// waits for P_g, for the corrections' read of O_b (tile g - 2) and for its
// stage.  The commit that signals PV_g done (o_full, to both CTAs) also
// frees K/V stage g % kStages (QK_g, which read the stage's K, completed
// before the softmax of tile g began).  The loop is unrolled by the 8
// stages, so stage and buffer offsets are constants.
__device__ void pv_issuer(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t tmem, int c,
                          int ncl) {
    static_assert(kStages == 8, "the unrolled loop");
    const uint32_t idesc = idesc_e4m3_f32(2 * kBM, kPvN);
    const uint64_t k64 = smem_desc_k128(smem + kOffStages);
    const uint32_t hi = (uint32_t)(k64 >> 32);
    const uint32_t v0lo = (uint32_t)k64 + (kHalf >> 4);
    constexpr uint32_t kStageLo = kStageBytes >> 4;
    const uint32_t G = (uint32_t)local_items(p.items, c, ncl) * (uint32_t)p.T;
    auto step = [&](auto S_, uint32_t g) -> bool {
        constexpr uint32_t s = decltype(S_)::value, b = s & 1;   // g % kStages, g % 2
        if (!wait.all(&B.p_full[b], (g >> 1) & 1, g >= 2 ? &B.o_free[b] : nullptr, ((g - 2) >> 1) & 1,
                      &B.kv_full[s], (g / kStages) & 1))
            return false;
        tc_fence_after();
        const uint32_t pa = tmem + (b ? kColP1 : kColP0), od = tmem + (b ? kColO1 : kColO0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma2_ts(od, pa + 8 * kk, v0lo + s * kStageLo + 2 * kk, hi, idesc, kk > 0);
        commit_both(&B.o_full[b]);
        commit_both(&B.kv_empty[s]);     // the producers may refill stage s
        return true;
    };
    bool ok = true;
    for (uint32_t g = 0; ok && g < G; g += 8) {
        ok = step(std::integral_constant<uint32_t, 0>{}, g);
        if (ok && g + 1 < G) ok = step(std::integral_constant<uint32_t, 1>{}, g + 1);
        if (ok && g + 2 < G) ok = step(std::integral_constant<uint32_t, 2>{}, g + 2);
        if (ok && g + 3 < G) ok = step(std::integral_constant<uint32_t, 3>{}, g + 3);
        if (ok && g + 4 < G) ok = step(std::integral_constant<uint32_t, 4>{}, g + 4);
        if (ok && g + 5 < G) ok = step(std::integral_constant<uint32_t, 5>{}, g + 5);
        if (ok && g + 6 < G) ok = step(std::integral_constant<uint32_t, 6>{}, g + 6);
        if (ok && g + 7 < G) ok = step(std::integral_constant<uint32_t, 7>{}, g + 7);
    }
    commit_local_pair(&B.drain[1]);
    drain_wait(&B.drain[1], 0);
}

// Two threads of one warp per query row: warp w (quarter w % 4, sub (w-4)/4)
// owns TMEM lanes 32*quarter + 16*sub + [0, 16); lane t < 16 reads columns
// [0, 64) of its row and lane t + 16 columns [64, 128), so the partial row
// maxima meet in one shuffle.

// 32 TMEM lanes x 32 consecutive columns from r[0 .. 31]: thread i writes
// lane i (one row's 128 P codes, 4 per column).
__device__ __forceinline__ void tmem_st32_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// One thread per query row: warp `quarter` owns rows quarter * 32 + lane and
// reads all 128 scores of its row, so the row maximum needs no exchange and
// the per-tile scalar work, waits and arrivals run in four warps per CTA.
template <bool PROBE>
__device__ void softmax_role(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t tmem,
                             uint32_t rank, int c, int ncl, int quarter, int lane) {
    const int row = quarter * 32 + lane;
    float* st_alpha = reinterpret_cast<float*>(smem + kOffStats);
    const uint32_t lead_p = peer_addr(B.p_full, 0);            // p_full[b] at + 8 b
    const uint32_t lead_s = peer_addr(B.s_free, 0);
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
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
            const int slot = g % kStatSlots;
            // the scores of tile g, and (checked alongside) the statistics
            // slot this tile writes at its end and the completion of PV_{g-2},
            // the last reader of the P buffer this tile writes
            if (!wait.all(&B.s_full[0], g & 1,
                          g >= (uint32_t)kStatSlots ? &B.meta_empty[slot] : nullptr, ((g / kStatSlots) - 1) & 1,
                          g >= 2 ? &B.o_full[b] : nullptr, ((g - 2) >> 1) & 1))
                return;
            tc_fence_after();
            uint32_t r[128];
            tmem_ld32_at<0>(trow + kColS, r);
            tmem_ld32_at<32>(trow + kColS + 32, r);
            tmem_ld32_at<64>(trow + kColS + 64, r);
            tmem_ld32_at<96>(trow + kColS + 96, r);
            tmem_wait_ld();
            // S is in registers: QK_{g+1} may overwrite it
            tc_fence_before();
            __syncwarp();
            mbar_arrive_cluster_if(lead_s, lane == 0);
            if (j == p.T - 1) {             // only the last tile of an item can be partial
                const int nvalid = (int)(p.sk - (int64_t)j * kBN);
                if (nvalid < 128) {
#pragma unroll
                    for (int i = 0; i < 128; ++i)
                        if (i >= nvalid) r[i] = 0xff800000u;   // -inf: masked key
                }
            }
            float mx[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = fmaxf(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
#pragma unroll
            for (int t = 1; t < 8; ++t)
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    mx[k] = fmax3(mx[k], __uint_as_float(r[16 * t + 2 * k]), __uint_as_float(r[16 * t + 2 * k + 1]));
            const float rmax = fmaxf(fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), mx[6]), mx[7]);
            const float cs = __fmul_rn(__fmul_rn(qs_scale, ks), p.scale);
            const float m_new = fmaxf(m, __fmul_rn(rmax, cs));
            // alpha = e^(m - m_new) as 2^((m - m_new) log2 e) on MUFU.EX2: a few
            // FP32 ulps from expf, inside the output tolerance, and exactly 1
            // when the maximum did not move (the correction skips its rescale then)
            const float alpha = ex2_ftz(__fmul_rn(m - m_new, kLog2e));
            // A is kept at or above the smallest normal float: a masked key (-inf)
            // times A must stay -inf (code 0, no mass), never -inf * 0 = NaN.  When
            // c underflows that far, every logit s * c is below 2^-100 and the
            // codes come out as for A = 0, as in the reference.  In units of
            // 2^-24 throughout: scaling by a power of two is exact, so this is
            // the unscaled computation times 2^-24, bit for bit.
            const float A = fmaxf(__fmul_rn(cs, kC1 * kTwoM24), kMinNormal);
            float Bc = __fsub_rn(kC2 * kTwoM24, __fmul_rn(m_new, kC1 * kTwoM24));
            const float umax = fmaf(rmax, A, Bc);
            if (umax > 120.25f * kTwoM24) Bc = __fsub_rn(Bc, __fsub_rn(umax, kC2 * kTwoM24));
            const float2 AA = make_float2(A, A), BB = make_float2(Bc, Bc);
            uint32_t pk[32];
#pragma unroll
            for (int w = 0; w < 32; ++w) {
                const float2 g01 =
                    ffma2(make_float2(__uint_as_float(r[4 * w]), __uint_as_float(r[4 * w + 1])), AA, BB);
                const float2 g23 =
                    ffma2(make_float2(__uint_as_float(r[4 * w + 2]), __uint_as_float(r[4 * w + 3])), AA, BB);
                const uint32_t h01 = cvt_relu_f16x2(g01.y, g01.x);   // integer codes as f16 subnormals
                const uint32_t h23 = cvt_relu_f16x2(g23.y, g23.x);
                pk[w] = __byte_perm(h01, h23, 0x6420);
            }
            // The row mass, the sum of the decoded P, is formed by the PV MMA
            // in its ones columns.
            if (probe && j >= p.pr_begin && j < p.pr_begin + p.pr_count) {
                const int64_t t = j - p.pr_begin;
                float* lg = p.pr_logits + (t * 128 + row) * 128;
                uint32_t* cd = reinterpret_cast<uint32_t*>(p.pr_codes + (t * 128 + row) * 128);
#pragma unroll
                for (int i = 0; i < 128; ++i) lg[i] = __uint_as_float(r[i]);
#pragma unroll
                for (int w = 0; w < 32; ++w) cd[w] = pk[w];
                float* rs = p.pr_rowstat + (t * 128 + row) * 4;
                rs[0] = m_new; rs[1] = A; rs[2] = Bc; rs[3] = alpha;
            }
            // P_g into P_b: 4 codes per 32-bit column, the A-operand layout of
            // the PV MMA (K slice kk of 32 keys in columns [8 kk, 8 kk + 8))
            tmem_st32_x32(trow + (b ? kColP1 : kColP0), pk);
            st_alpha[slot * 128 + row] = alpha;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            mbar_arrive_cluster_if(lead_p + 8 * b, lane == 0);
            mbar_arrive_if(&B.st_full[slot], lane == 0);
            m = m_new;
        }
    }
}

// One thread per row (warp `quarter`: rows quarter * 32 + lane, all 128
// channels).  Per tile, in units of 256 as the softmax: acc = alpha acc +
// (PV + M mu / vscale) vscale (core.py:335-336: rowmass times the stored
// scaled mean, then the scale), den = alpha den + M, with M the mass column
// of O_b.  O_b is read in four 32-column chunks and released (o_free) once
// the last is in registers.
template <bool HAS_MEAN>
__device__ void correction_role(const Params& p, uint8_t* smem, const Bars& B, const Waiter& wait, uint32_t tmem,
                                uint32_t rank, int c, int ncl, int quarter, int lane) {
    const int row = quarter * 32 + lane;
    const float* st_alpha = reinterpret_cast<const float*>(smem + kOffStats);
    const uint32_t lead_o = peer_addr(B.o_free, 0);            // o_free[b] at + 8 b
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    uint32_t g = 0;
    for (int it = c; it < p.items; it += ncl) {
        const int head = it / p.pairs, pair = it - head * p.pairs;
        const int64_t grow = (int64_t)(2 * pair + (int)rank) * kBM + row;
        float2 acc[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = make_float2(0.0f, 0.0f);
        float den = 0.0f;
        for (int j = 0; j < p.T; ++j, ++g) {
            const uint32_t b = g & 1, slot = g % kStatSlots, s = g % kMetaSlots;
            // without V-Smooth the correction has slack enough to park in its
            // waits, which leaves their issue slots to the softmax warps
            if (!wait.all_or_parked<!HAS_MEAN>(&B.o_full[b], (g >> 1) & 1, &B.st_full[slot], (g / kStatSlots) & 1,
                                               &B.meta_full[s], (g / kMetaSlots) & 1))
                return;
            tc_fence_after();
            const float alpha = st_alpha[slot * 128 + row];
            const float4* vsp = reinterpret_cast<const float4*>(smem + kOffMeta + s * kMetaBytes);
            const float4* usp = vsp + 32;                          // the stored means follow the scales
            const bool rescale = __any_sync(0xffffffffu, alpha != 1.0f);
            const float2 aa = make_float2(alpha, alpha);
            const uint32_t ob = trow + (b ? kColO1 : kColO0);
            if (rescale) {      // warp-uniform; alpha == 1 leaves acc unchanged
#pragma unroll
                for (int i = 0; i < 64; ++i) acc[i] = fmul2(acc[i], aa);
            }
            float M;
            auto chunk = [&](const uint32_t (&o)[32], int ch) {
                const float2 mm = make_float2(M, M);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 vs = vsp[8 * ch + q];
                    const int i = 16 * ch + 2 * q;
                    float2 o01 = make_float2(__uint_as_float(o[4 * q]), __uint_as_float(o[4 * q + 1]));
                    float2 o23 = make_float2(__uint_as_float(o[4 * q + 2]), __uint_as_float(o[4 * q + 3]));
                    if (HAS_MEAN) {
                        const float4 u = usp[8 * ch + q];
                        o01 = ffma2(mm, make_float2(u.x, u.y), o01);
                        o23 = ffma2(mm, make_float2(u.z, u.w), o23);
                    }
                    acc[i] = ffma2(o01, make_float2(vs.x, vs.y), acc[i]);
                    acc[i + 1] = ffma2(o23, make_float2(vs.z, vs.w), acc[i + 1]);
                }
            };
            if (HAS_MEAN) {
                // V-Smooth: the next 32-column chunk of O_b loads while the
                // current one is computed, so that only the first load's
                // latency comes before the release of O_b, which PV_{g+2}
                // waits for (two chunks in registers: the 224-register share)
                uint32_t oc[2][32];
                tmem_ld32_at<0>(ob, oc[0]);
                M = __uint_as_float(tmem_ld32_x1(ob + kColMass));
                tmem_wait_ld();
                tmem_ld32_at<0>(ob + 32, oc[1]);
                chunk(oc[0], 0);
                tmem_wait_ld();
                tmem_ld32_at<0>(ob + 64, oc[0]);
                chunk(oc[1], 1);
                tmem_wait_ld();
                tmem_ld32_at<0>(ob + 96, oc[1]);
                chunk(oc[0], 2);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                mbar_arrive_cluster_if(lead_o + 8 * b, lane == 0);
                chunk(oc[1], 3);
            } else {
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    uint32_t o[32];
                    tmem_ld32_at<0>(ob + 32 * ch, o);
                    uint32_t mraw = 0;
                    if (ch == 0) mraw = tmem_ld32_x1(ob + kColMass);
                    tmem_wait_ld();
                    if (ch == 0) M = __uint_as_float(mraw);
                    if (ch == 3) {
                        tc_fence_before();
                        __syncwarp();
                        mbar_arrive_cluster_if(lead_o + 8 * b, lane == 0);
                    }
                    chunk(o, ch);
                }
            }
            den = __fadd_rn(__fmul_rn(alpha, den), M);
            __syncwarp();
            mbar_arrive_if(&B.meta_empty[s], lane == 0);
        }
        // With V-Smooth (the correction warp paces the combined mode) acc / den
        // is acc times the correctly rounded 1 / den: within 1.5 FP32 ulp of the
        // quotient, far inside the output tolerance, and a tenth of the
        // instructions of 128 correctly rounded divisions.
        const float rcp_den = HAS_MEAN ? __frcp_rn(den) : 0.0f;
        const float2 rr = make_float2(rcp_den, rcp_den);
        if (grow >= p.sq) continue;
        const int64_t base = ((int64_t)head * p.sq + grow) * p.dv;
        if (p.out_dtype == VCB_BF16 && p.dv == 128) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + base);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 a = acc[4 * q + e];
                    const float2 v = HAS_MEAN ? fmul2(a, rr) : make_float2(__fdiv_rn(a.x, den), __fdiv_rn(a.y, den));
                    __nv_bfloat162 h2 = __floats2bfloat162_rn(v.x, v.y);
                    w[e] = *reinterpret_cast<uint32_t*>(&h2);
                }
                dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
            }
            continue;
        }
        // other dtypes or dv < 128: channel by channel (static indices only, so
        // acc stays in registers)
#pragma unroll
        for (int i = 0; i < 64; ++i) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int col = 2 * i + e;
                if (col < p.dv) {
                    const float a = e ? acc[i].y : acc[i].x;
                    const float val = HAS_MEAN ? __fmul_rn(a, rr.x) : __fdiv_rn(a, den);
                    if (p.out_dtype == VCB_BF16)
                        static_cast<__nv_bfloat16*>(p.out)[base + col] = __float2bfloat16_rn(val);
                    else if (p.out_dtype == VCB_F16)
                        static_cast<__half*>(p.out)[base + col] = __float2half_rn(val);
                    else
                        static_cast<float*>(p.out)[base + col] = val;
                }
            }
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
            mbar_init(&B.q_free[i], 1);           // the QK thread
            mbar_init(&B.drain[i], 1);
            mbar_init(&B.s_full[i], 1);
            mbar_init(&B.s_free[i], 8);           // 4 softmax warps in each CTA
            mbar_init(&B.p_full[i], 8);           // 4 softmax warps in each CTA
            mbar_init(&B.o_full[i], 1);
            mbar_init(&B.o_free[i], 8);           // 4 correction warps in each CTA
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&B.kv_full[s], 1);
            mbar_init(&B.kv_empty[s], 1);
        }
        for (int s = 0; s < kMetaSlots; ++s) {
            mbar_init(&B.meta_full[s], 1);
            mbar_init(&B.meta_empty[s], 4);
        }
        for (int s = 0; s < kStatSlots; ++s) {
            mbar_init(&B.st_full[s], 4);
        }
        *abort = 0;
        fence_barrier_init();
    }
    if (rank == 1) {
        // the odd CTA's constant B rows 56..71 of every stage: E4M3 1.0 (0x38)
        // in every byte, so the 128-byte swizzle needs no care; written before
        // the cluster barrier, and made visible to the tensor cores' (async)
        // proxy by each writing thread
        constexpr uint32_t kOnesBytes = (uint32_t)(kVRows0 - kVRows1) * 128;   // 2 KB per stage
        for (uint32_t i = threadIdx.x; i < kStages * (kOnesBytes / 16); i += kThreads) {
            const uint32_t st = i / (kOnesBytes / 16), off = i % (kOnesBytes / 16);
            reinterpret_cast<uint4*>(smem + kOffStages + st * kStageBytes + kHalf + kVRows1 * 128)[off] =
                make_uint4(0x38383838u, 0x38383838u, 0x38383838u, 0x38383838u);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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

    // Register split of the 384 x 168 launch budget (ptxas allocates each
    // role's code within its share): producer/MMA group 80 (the unrolled MMA
    // loop with its item cursor spills below 72), softmax 192 (a row's 128
    // scores and 32 code words), correction 192 (a row's 128 accumulators and
    // one 32-column chunk of O; 224 with V-Smooth, two chunks); 10240 + 24576
    // + 24576 = 59392, or + 28672 = 63488, of 64512.
    if (warp < 4) {
        reg_dealloc<80>();
        if (warp == 0 && lane == 0) producer(p, smem, B, wait, rank, c, ncl);
        if (warp == 1 && lane == 0 && rank == 0) qk_issuer(p, smem, B, wait, tmem, c, ncl);
        if (warp == 3 && lane == 0 && rank == 0) pv_issuer(p, smem, B, wait, tmem, c, ncl);
        if (warp == 2 && lane == 0) meta_producer<HAS_MEAN>(p, smem, B, wait, c, ncl);
    } else if (warp < 8) {
        reg_alloc<192>();
        softmax_role<PROBE>(p, smem, B, wait, tmem, rank, c, ncl, warp & 3, lane);
    } else {
        if (HAS_MEAN) reg_alloc<224>();
        else reg_alloc<192>();
        correction_role<HAS_MEAN>(p, smem, B, wait, tmem, rank, c, ncl, warp & 3, lane);
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
    return launch_pairs(attn_kernel<M, P>, p, p.items, kThreads, kSmemAlloc, reg_split(M), max_clusters,
                        (M ? 2 : 0) | (P ? 1 : 0), st);
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

// The ExpCast modes run here; the exp modes (fp8_control, v_smooth) on the
// kernel of vcb_attn_exp.cu, whose softmax forms the FP32 row mass itself.
int attn_run(const vcb_attn_args* a, const vcb_attn_probe* probe, cudaStream_t st) {
    if (!a->expcast) return attn_exp_run(a, probe, st);
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
    if (!rc) rc = make_map(&p.tm_v0, a->v8, 128, (uint64_t)T * 128, (uint64_t)a->heads, kVRows0);
    if (!rc) rc = make_map(&p.tm_v1, a->v8, 128, (uint64_t)T * 128, (uint64_t)a->heads, kVRows1);
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

int wait_selftest_run(int complete, const void* src, int32_t* status, int32_t* report, cudaStream_t st) {
    VCB_CUDA(cudaMemsetAsync(report, 0, 4 * sizeof(int32_t), st));
    wait_selftest_kernel<<<1, 128, 0, st>>>(complete, static_cast<const int32_t*>(src), status, report);
    VCB_CUDA(cudaGetLastError());
    return VCB_OK;
}

}  // namespace vcb
