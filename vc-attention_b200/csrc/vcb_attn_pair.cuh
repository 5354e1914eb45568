// Pieces shared by the two paired attention kernels (vcb_attn.cu for the
// ExpCast modes, vcb_attn_exp.cu for the exp modes): cluster and tensor-memory
// PTX for a CTA pair, the bounded waits, the MMA wrappers, the softmax
// constants of the reference's numerical contract (core.py:307-341) and the
// TMA descriptor encoder.  Every definition has internal linkage, so each
// kernel file gets its own copy.
#pragma once
#include "vcb_internal.h"

namespace vcb {
namespace {

constexpr int kBM = 128;                          // query rows per CTA (256 per pair)
constexpr int kBN = 128;                          // keys per KV tile
constexpr uint32_t kQBytes = 128 * 128;           // one E4M3 Q tile (16 KB)
constexpr uint32_t kHalf = 64 * 128;              // this CTA's half of a K tile (8 KB)
constexpr float kC1 = 11.541560173034668f;        // 8 log2(e) in fp32
constexpr float kC2 = 119.6500015258789f;         // 119.65 in fp32
constexpr float kTwoM24 = 5.9604644775390625e-08f;    // 2^-24
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMinNormal = 1.17549435e-38f;     // 2^-126
constexpr uint32_t kParkHintNs = 20000;           // longest park of a parked wait between checks

// ------------------------------------------------------------- cluster PTX
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
    return d;
}
// Arrive on an mbarrier anywhere in the cluster, with the default
// (CTA-scope) release.  The data these arrivals publish is tensor memory,
// ordered for the MMA by tcgen05.wait::st / tcgen05.fence::before_thread_sync
// before the arrive and tcgen05.fence::after_thread_sync after the wait; a
// cluster-scope release here cost ~1000 cycles per tile.
__device__ __forceinline__ void mbar_arrive_cluster_if(uint32_t addr, bool pred) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "@p mbarrier.arrive.shared::cluster.b64 _, [%0];\n\t}"
        ::"r"(addr), "r"((uint32_t)pred)
        : "memory");
}
__device__ __forceinline__ void store_cluster_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on
// the even CTA's barrier (`bar` a shared::cluster address); no multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrives on the barrier at this offset in both CTAs once every tcgen05
// operation this thread issued before is complete.
__device__ __forceinline__ void commit_both(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(smem_u32(bar)), "h"((uint16_t)3)
        : "memory");
}
__device__ __forceinline__ void commit_local_pair(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait used while draining after an abort: ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait_sleep(a, parity, kSuspendHintNs)) {
        if (globaltimer() - t0 > kWaitLimitNs) return;
    }
}

// Non-blocking check of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// A wait that gives up (mbar_wait) and, when it does, raises the peer CTA's
// abort flag too, so the pair stops together.
struct Waiter {
    volatile int* abort;
    uint32_t peer_abort;     // shared::cluster address of the other CTA's flag
    __device__ __forceinline__ bool operator()(uint64_t* bar, uint32_t parity) const {
        if (mbar_wait(bar, parity, abort)) return true;
        store_cluster_u32(peer_abort, 1u);
        return false;
    }
    // Waits for up to three phases.  A barrier check costs a shared-memory
    // round trip even when the phase is long complete, so the three checks
    // are issued back to back (non-blocking test_wait) and their latencies
    // overlap; only a phase found incomplete falls back to the polling wait.
    // A null barrier is skipped.
    __device__ __forceinline__ bool all(uint64_t* b0, uint32_t p0, uint64_t* b1, uint32_t p1, uint64_t* b2 = nullptr,
                                        uint32_t p2 = 0) const {
        const bool r0 = mbar_test(smem_u32(b0), p0);
        const bool r1 = !b1 || mbar_test(smem_u32(b1), p1);
        const bool r2 = !b2 || mbar_test(smem_u32(b2), p2);
        if (r0 && r1 && r2) return true;
        return (r0 || (*this)(b0, p0)) && (r1 || (*this)(b1, p1)) && (r2 || (*this)(b2, p2));
    }
    // The same wait parked in the barrier between polls (try_wait with a
    // suspend-time hint): for roles off the critical path, whose polling would
    // otherwise take issue slots from the softmax and correction warps that
    // share their SM sub-partition.
    __device__ __forceinline__ bool parked(uint64_t* bar, uint32_t parity) const {
        const uint32_t a = smem_u32(bar);
        if (mbar_try_wait(a, parity)) return true;
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait_sleep(a, parity, kParkHintNs)) {
            if (*abort) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                *abort = 1;
                store_cluster_u32(peer_abort, 1u);
                return false;
            }
        }
        return true;
    }
    // all() for a role off the critical path: parks in each incomplete phase
    __device__ __forceinline__ bool parked_all(uint64_t* b0, uint32_t p0, uint64_t* b1, uint32_t p1,
                                               uint64_t* b2 = nullptr, uint32_t p2 = 0) const {
        return parked(b0, p0) && (!b1 || parked(b1, p1)) && (!b2 || parked(b2, p2));
    }
    template <bool PARK>
    __device__ __forceinline__ bool all_or_parked(uint64_t* b0, uint32_t p0, uint64_t* b1, uint32_t p1,
                                                  uint64_t* b2 = nullptr, uint32_t p2 = 0) const {
        return PARK ? parked_all(b0, p0, b1, p1, b2, p2) : all(b0, p0, b1, p1, b2, p2);
    }
};

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

// The items of cluster `c` are c, c + ncl, ...
__device__ __forceinline__ int local_items(int items, int c, int ncl) {
    return c < items ? (items - c + ncl - 1) / ncl : 0;
}


// The MMA thread shares its SM sub-partition with four busy softmax /
// correction warps, and every instruction it issues waits for a scheduler
// slot, so its instruction stream is kept short: shared-memory descriptors
// differ only in the low word (start address >> 4), which the loop advances
// by constants; the high word (stride, version, swizzle) is one register.
__device__ __forceinline__ void mma2_ss(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t hi, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "mov.b64 da, {%1, %3};\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], da, db, %4, p;\n\t}"
        ::"r"(d_tmem), "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma2_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t hi, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], [%1], db, %4, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
}

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

// One TMEM column of the warp's 32 lanes: thread i gets lane i.
__device__ __forceinline__ uint32_t tmem_ld32_x1(uint32_t taddr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
    return r;
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

// 3-D byte tensor [planes][rows][width] with `width`-byte rows, boxes of
// width x box_rows, swizzled to the row width (128 B or 32 B).
int make_map(CUtensorMap* map, const void* base, uint64_t width, uint64_t rows, uint64_t planes, uint32_t box_rows) {
    EncodeTiledFn enc;
    int rc = get_encoder(&enc);
    if (rc) return rc;
    const cuuint64_t dims[3] = {width, rows, planes};
    const cuuint64_t strides[2] = {width, width * rows};
    const cuuint32_t box[3] = {(cuuint32_t)width, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw = width == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B;
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(VCB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return VCB_OK;
}


// Launches a paired kernel (clusters of 2 CTAs) with as many pairs as are
// resident at once, looked up once per device and variant.  `reg_split` is
// the sum of the roles' setmaxnreg shares (registers per CTA): a kernel
// whose launch registers cannot hold it would wait in setmaxnreg.inc
// forever, so that build is refused before it runs.
template <typename Kernel, typename P>
int launch_pairs(Kernel kernel, const P& p, int items, int threads, uint32_t smem_bytes, int reg_split,
                 int (&cache)[64][8], int variant, cudaStream_t st) {
    VCB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // the kernel begins with pdl_wait()
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;          // the occupancy query takes the cluster shape alone
    int dev = 0;
    VCB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(VCB_ERR_INVALID_ARGUMENT, "device ordinal %d out of range", dev);
    int& ncl_max = cache[dev][variant];
    if (ncl_max == 0) {
        cudaFuncAttributes fa;
        VCB_CUDA(cudaFuncGetAttributes(&fa, kernel));
        if (fa.numRegs * threads < reg_split)
            return fail(VCB_ERR_CUDA, "attention kernel launched with %d registers x %d threads, below its %d-register "
                        "split", fa.numRegs, threads, reg_split);
        cfg.gridDim = dim3(2 * 148);
        int n = 0;
        VCB_CUDA(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
        if (n < 1) return fail(VCB_ERR_CUDA, "the attention kernel's CTA pairs do not fit on this GPU");
        ncl_max = n;
    }
    const int ncl = items < ncl_max ? items : ncl_max;
    cfg.gridDim = dim3(2 * ncl);
    cfg.numAttrs = 2;
    VCB_CUDA(cudaLaunchKernelEx(&cfg, kernel, p));
    return VCB_OK;
}

}  // namespace
}  // namespace vcb
