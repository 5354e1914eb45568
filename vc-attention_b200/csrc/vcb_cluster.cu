// Per-head V clustering for sm_100a: Lloyd k-means with equispaced (or
// warm-started) centres and a stable permutation of the final labels
// (reference: core.py:138-163; the Hopper extension drove ATen ops from a
// host loop, bindings.cpp:182-217).
//
// Fixed orders, mirrored by the CPU checker:
//   distances  ||x||^2, ||c||^2 and x.c are fmaf chains over channels
//              0..D-1; distance = (xx + cc) - 2*xc; the first minimum wins.
//   sums       chunks of kChunk tokens, each split into sub-chunks of kSub
//              tokens; inside a sub-chunk each cluster adds its tokens in
//              token order; a chunk adds its sub-chunk sums in order (from
//              0); chunks are added in order.
//   permutation  a counting sort: cluster-major, token order inside a
//              cluster, i.e. argsort(labels, stable=True).
#include "vcb_internal.h"

namespace vcb {

constexpr int kChunk = 256;
constexpr int kSub = 32;
constexpr int kMaxClusters = 32;
// clusters whose sub-chunk sums the 128-channel assign pass reduces per round:
// 8 warps x 2 x 128 floats fit in the centres' 8 KB (8 clusters), so that the
// pass takes ~75 KB of shared memory and three CTAs fit on an SM
constexpr int kSumGroup = 2;

struct ClusterArgs {
    const void* v;
    int64_t S;
    int D;
    int count;
    int nchunk;
    float* centers;   // [heads, count, D]
    uint8_t* labels;  // [heads, S]
    float* psum;      // [heads, nchunk, count, 128]
    int32_t* pcnt;    // [heads, nchunk, count]
    int32_t* off;     // [heads, nchunk, count]
    int32_t* pi;      // [heads, S]
};

struct InitIdx { long long idx[kMaxClusters]; };

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__global__ void cluster_init_kernel(ClusterArgs a, const float* __restrict__ centers_in, InitIdx init) {
    pdl_wait();
    pdl_open();
    const int64_t h = blockIdx.x;
    for (int i = threadIdx.x; i < a.count * a.D; i += blockDim.x) {
        const int c = i / a.D, d = i % a.D;
        float val;
        if (centers_in) val = centers_in[(h * a.count + c) * a.D + d];
        else val = Elem<T>::load(static_cast<const T*>(a.v) + (h * a.S + init.idx[c]) * a.D + d);
        a.centers[(h * a.count + c) * a.D + d] = val;
    }
}

template <typename T>
__global__ void __launch_bounds__(256) cluster_assign_kernel(ClusterArgs a) {
    pdl_wait();
    pdl_open();
    __shared__ __align__(16) float cen[kMaxClusters * 128];
    __shared__ float cnorm[kMaxClusters];
    __shared__ uint8_t lab[kChunk];
    const int64_t h = blockIdx.y;
    const int chunk = blockIdx.x;
    const int tid = threadIdx.x;
    const int D = a.D, count = a.count;
    for (int i = tid; i < kMaxClusters * 128; i += 256) {
        const int c = i / 128, d = i % 128;
        cen[i] = (c < count && d < D) ? a.centers[(h * count + c) * D + d] : 0.0f;
    }
    __syncthreads();
    if (tid < count) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc = fmaf(cen[tid * 128 + d], cen[tid * 128 + d], acc);
        cnorm[tid] = acc;
    }
    __syncthreads();
    const int64_t base = (int64_t)chunk * kChunk;
    const int nvalid = (int)min((int64_t)kChunk, a.S - base);
    const T* vh = static_cast<const T*>(a.v) + h * a.S * D;
    if (tid < nvalid) {
        float x[128];
        const T* row = vh + (base + tid) * D;
        if (D == 128) {
#pragma unroll
            for (int i = 0; i < 16; ++i) load8(row + 8 * i, x + 8 * i);
        } else {
#pragma unroll
            for (int d = 0; d < 128; ++d) x[d] = d < D ? Elem<T>::load(row + d) : 0.0f;
        }
        float xx = 0.0f;
#pragma unroll
        for (int d = 0; d < 128; ++d)
            if (d < D) xx = fmaf(x[d], x[d], xx);
        int best = 0;
        float bestd = 0.0f;
        for (int c0 = 0; c0 < count; c0 += 8) {
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
            for (int d = 0; d < 128; d += 4) {
                if (d < D) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float4 cv = *reinterpret_cast<const float4*>(&cen[(c0 + i) * 128 + d]);
                        acc[i] = fmaf(x[d], cv.x, acc[i]);
                        if (d + 1 < D) acc[i] = fmaf(x[d + 1], cv.y, acc[i]);
                        if (d + 2 < D) acc[i] = fmaf(x[d + 2], cv.z, acc[i]);
                        if (d + 3 < D) acc[i] = fmaf(x[d + 3], cv.w, acc[i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = c0 + i;
                if (c < count) {
                    const float dist = __fsub_rn(__fadd_rn(xx, cnorm[c]), __fmul_rn(2.0f, acc[i]));
                    if (c == 0 || dist < bestd) { bestd = dist; best = c; }
                }
            }
        }
        lab[tid] = (uint8_t)best;
        a.labels[h * a.S + base + tid] = (uint8_t)best;
    }
    __syncthreads();
    // Stable order of the chunk's tokens by cluster (a counting sort): the
    // rank of token j among earlier tokens of its cluster comes from warp
    // match/ballot masks plus the per-warp counts of the warps before it.
    __shared__ int wcnt[8][kMaxClusters];
    __shared__ int seg[kMaxClusters + 1];
    __shared__ uint16_t order[kChunk];
    const int warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < 8 * kMaxClusters; i += 256) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    const int lj = tid < nvalid ? lab[tid] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, lj);
    const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
    if (lj >= 0 && rank_in_warp == 0) wcnt[warp][lj] = __popc(same);
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int c = 0; c < count; ++c) {
            seg[c] = run;
            for (int w = 0; w < 8; ++w) run += wcnt[w][c];
        }
        seg[count] = run;
    }
    __syncthreads();
    if (lj >= 0) {
        int before = 0;
        for (int w = 0; w < warp; ++w) before += wcnt[w][lj];
        order[seg[lj] + before + rank_in_warp] = (uint16_t)tid;
    }
    __syncthreads();
    // Per-cluster partial sums in the fixed order the CPU checker uses: a
    // cluster's tokens in token order inside each kSub sub-chunk, sub-chunk
    // sums added in order.  Threads 0..127 own clusters below count/2,
    // threads 128..255 the rest; channel d = tid % 128.
    const int d = tid & 127;
    const int c_lo = tid < 128 ? 0 : count / 2, c_hi = tid < 128 ? count / 2 : count;
    float* ps = a.psum + ((int64_t)h * a.nchunk + chunk) * count * 128;
    if (d < D) {
        for (int c = c_lo; c < c_hi; ++c) {
            float part = 0.0f, sub = 0.0f;
            int cur = -1;
            const int p1 = seg[c + 1];
            for (int pos = seg[c]; pos < p1; ++pos) {
                const int tok = order[pos];
                if (tok / kSub != cur) {   // a new sub-chunk: close the previous one
                    part += sub;
                    sub = 0.0f;
                    cur = tok / kSub;
                }
                sub += Elem<T>::load(vh + (base + tok) * D + d);
            }
            ps[c * 128 + d] = part + sub;
        }
    }
    if (tid < count) a.pcnt[((int64_t)h * a.nchunk + chunk) * count + tid] = seg[tid + 1] - seg[tid];
}

// D == 128: the chunk's rows are staged in shared memory once (coalesced
// 16-byte cp.async copies, no register staging; 16-byte chunks XOR-swizzled
// by row so that a warp reading one chunk of 32 rows hits every bank group),
// then
//   distances  thread t = tokens t % 128 and t % 128 + 128 in the two lanes
//              of packed FMAs against a doubled centre table, half of the
//              clusters per thread (t / 128); channels streamed in order from
//              shared memory, so every (token, cluster) chain is the fmaf
//              chain above; the two halves' first minima are merged;
//   sums       warp w = sub-chunk w (tokens 32w..32w+31), lane = 4 channels;
//              per cluster, a ballot of the sub-chunk's labels gives that
//              cluster's tokens, added lowest first (token order); sub-chunk
//              sums added in order by thread (cluster, d).
template <typename T>
__global__ void __launch_bounds__(256, 3) cluster_assign128_kernel(ClusterArgs a) {
    pdl_wait();
    pdl_open();
    constexpr int RB = 128 * (int)sizeof(T);        // bytes per staged row
    constexpr int NCH = RB / 16;                    // 16-byte chunks per row
    constexpr int E = 16 / (int)sizeof(T);          // elements per chunk
    extern __shared__ __align__(16) uint8_t dsm[];
    uint8_t* xs = dsm;                                               // [256][RB], swizzled
    // centres twice over for packed FMAs over two tokens: [c / 4][d][c % 4][2]
    float* cen2 = reinterpret_cast<float*>(dsm + kChunk * RB);
    // the sub-chunk sums [8 warps][kSumGroup clusters][128] reuse the centres'
    // space: they are first written two barriers after the last distance
    float* subs = cen2;
    __shared__ float cnorm[kMaxClusters];
    __shared__ float hbest[2][kChunk];
    __shared__ uint8_t hidx[2][kChunk];
    __shared__ uint8_t lab[kChunk];
    __shared__ int cnt[kMaxClusters];
    const int64_t h = blockIdx.y;
    const int chunk = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int count = a.count;
    const int64_t base = (int64_t)chunk * kChunk;
    const int nvalid = (int)min((int64_t)kChunk, a.S - base);
    const int ngroups = (count + 3) >> 2;
    for (int i = tid; i < ngroups * 4 * 128; i += 256) {
        const int c = i / 128, d = i % 128;
        const float val = c < count ? a.centers[(h * count) * 128 + i] : 0.0f;
        *reinterpret_cast<float2*>(cen2 + ((c >> 2) * 128 + d) * 8 + (c & 3) * 2) = make_float2(val, val);
    }
    if (tid < kMaxClusters) cnt[tid] = 0;
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(a.v) + (h * a.S + base) * 128);
    {   // the chunk straight into shared memory (cp.async, no register staging)
        constexpr int kPer = kChunk * NCH / 256;
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int g = tid + 256 * u, r = g / NCH, k = g % NCH;
            if (r < nvalid) {
                const uint32_t dst = smem_u32(xs + r * RB + ((k ^ (r & (NCH - 1))) << 4));
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                             ::"r"(dst), "l"(__cvta_generic_to_global(src + g)) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (tid < count) {
        float acc = 0.0f;
        const float* ct = cen2 + (tid >> 2) * 1024 + (tid & 3) * 2;
        for (int d = 0; d < 128; ++d) acc = fmaf(ct[d * 8], ct[d * 8], acc);
        cnorm[tid] = acc;
    }
    __syncthreads();

    {
        // thread t: tokens p and p + 128 (p = t % 128) in the two lanes of each
        // packed FMA, clusters 4 * (2g + half) .. + 3 of every group of eight
        // (half = t / 128); each (token, cluster) chain still runs over
        // d = 0..127 in order, as in the scalar form
        const int p = tid & 127, half = tid >> 7;
        const uint8_t* xa = xs + p * RB;
        const uint8_t* xb = xs + (p + 128) * RB;
        const int sw = p & (NCH - 1);            // (p + 128) & (NCH - 1) is the same
        float2 xx = make_float2(0.0f, 0.0f);
        float bd[2] = {0.0f, 0.0f};
        int bi[2] = {-1, -1};
        for (int c0 = 4 * half; c0 < count; c0 += 8) {
            const float* cg = cen2 + (c0 >> 2) * 1024;
            float2 acc[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll 2
            for (int k = 0; k < NCH; ++k) {
                const uint4 ra = *reinterpret_cast<const uint4*>(xa + ((k ^ sw) << 4));
                const uint4 rb = *reinterpret_cast<const uint4*>(xb + ((k ^ sw) << 4));
                float x0[E], x1[E];
                if constexpr (sizeof(T) == 4) {
                    x0[0] = __uint_as_float(ra.x); x0[1] = __uint_as_float(ra.y);
                    x0[2] = __uint_as_float(ra.z); x0[3] = __uint_as_float(ra.w);
                    x1[0] = __uint_as_float(rb.x); x1[1] = __uint_as_float(rb.y);
                    x1[2] = __uint_as_float(rb.z); x1[3] = __uint_as_float(rb.w);
                } else {
                    const T* ha = reinterpret_cast<const T*>(&ra);
                    const T* hb = reinterpret_cast<const T*>(&rb);
#pragma unroll
                    for (int e = 0; e < 8; ++e) { x0[e] = to_float(ha[e]); x1[e] = to_float(hb[e]); }
                }
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const int d = k * E + e;
                    const float2 x2 = make_float2(x0[e], x1[e]);
                    if (c0 < 8) xx = ffma2(x2, x2, xx);
                    const float4 ca = *reinterpret_cast<const float4*>(cg + d * 8);
                    const float4 cb = *reinterpret_cast<const float4*>(cg + d * 8 + 4);
                    acc[0] = ffma2(x2, make_float2(ca.x, ca.y), acc[0]);
                    acc[1] = ffma2(x2, make_float2(ca.z, ca.w), acc[1]);
                    acc[2] = ffma2(x2, make_float2(cb.x, cb.y), acc[2]);
                    acc[3] = ffma2(x2, make_float2(cb.z, cb.w), acc[3]);
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = c0 + i;
                if (c < count) {
                    const float cn = cnorm[c];
                    const float d0 = __fsub_rn(__fadd_rn(xx.x, cn), __fmul_rn(2.0f, acc[i].x));
                    const float d1 = __fsub_rn(__fadd_rn(xx.y, cn), __fmul_rn(2.0f, acc[i].y));
                    if (bi[0] < 0 || d0 < bd[0]) { bd[0] = d0; bi[0] = c; }
                    if (bi[1] < 0 || d1 < bd[1]) { bd[1] = d1; bi[1] = c; }
                }
            }
        }
        hbest[half][p] = bd[0]; hidx[half][p] = (uint8_t)(bi[0] < 0 ? 255 : bi[0]);
        hbest[half][p + 128] = bd[1]; hidx[half][p + 128] = (uint8_t)(bi[1] < 0 ? 255 : bi[1]);
    }
    __syncthreads();
    if (tid < nvalid) {
        // the first minimum over all clusters: the smaller distance, and the
        // smaller index on a tie (a half with no cluster has index 255)
        int best = hidx[0][tid];
        const int other = hidx[1][tid];
        if (other != 255 && (best == 255 || hbest[1][tid] < hbest[0][tid] ||
                             (hbest[1][tid] == hbest[0][tid] && other < best)))
            best = other;
        lab[tid] = (uint8_t)best;
        a.labels[h * a.S + base + tid] = (uint8_t)best;
        atomicAdd(&cnt[best], 1);
    }
    __syncthreads();

    float* ps = a.psum + ((int64_t)h * a.nchunk + chunk) * count * 128;
    const int t0 = warp * kSub, t1 = min(t0 + kSub, nvalid);
    for (int cg = 0; cg < count; cg += kSumGroup) {
        float s[kSumGroup][4];
#pragma unroll
        for (int i = 0; i < kSumGroup; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[i][e] = 0.0f;
        // each cluster of the group takes its tokens of the sub-chunk in token
        // order (lowest set bit first), the order of the per-token loop
        const int mine = t0 + lane < t1 ? lab[t0 + lane] - cg : -1;
#pragma unroll
        for (int i = 0; i < kSumGroup; ++i) {
            unsigned m = __ballot_sync(0xffffffffu, mine == i);
            while (m) {
                const int t = t0 + __ffs(m) - 1;
                m &= m - 1;
                float x[4];
                const uint8_t* xr = xs + t * RB;
                if constexpr (sizeof(T) == 4) {
                    const float4 v = *reinterpret_cast<const float4*>(xr + ((lane ^ (t & (NCH - 1))) << 4));
                    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
                } else {
                    const uint2 raw = *reinterpret_cast<const uint2*>(xr + (((lane >> 1) ^ (t & (NCH - 1))) << 4) +
                                                                      (lane & 1) * 8);
                    const T* hv = reinterpret_cast<const T*>(&raw);
#pragma unroll
                    for (int e = 0; e < 4; ++e) x[e] = to_float(hv[e]);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) s[i][e] += x[e];
            }
        }
#pragma unroll
        for (int i = 0; i < kSumGroup; ++i)
            *reinterpret_cast<float4*>(&subs[(warp * kSumGroup + i) * 128 + 4 * lane]) =
                make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
        __syncthreads();
        for (int idx = tid; idx < kSumGroup * 128; idx += 256) {
            const int i = idx >> 7, d = idx & 127;
            if (cg + i >= count) continue;
            float part = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) part += subs[(w * kSumGroup + i) * 128 + d];
            ps[(cg + i) * 128 + d] = part;
        }
        __syncthreads();
    }
    if (tid < count) a.pcnt[((int64_t)h * a.nchunk + chunk) * count + tid] = cnt[tid];
}

// One CTA per (head, cluster), thread d per channel; chunks added in order
// (the loads are independent, only the adds are chained).
__global__ void __launch_bounds__(128) cluster_update_kernel(ClusterArgs a) {
    pdl_wait();
    pdl_open();
    const int64_t h = blockIdx.x;
    const int c = blockIdx.y, d = threadIdx.x;
    if (d >= a.D) return;
    const float* src = a.psum + ((int64_t)h * a.nchunk * a.count + c) * 128 + d;
    const int32_t* cnt = a.pcnt + (int64_t)h * a.nchunk * a.count + c;
    const int64_t stride = (int64_t)a.count * 128;
    float total = 0.0f;
    long long n = 0;
#pragma unroll 8
    for (int ch = 0; ch < a.nchunk; ++ch) {
        total += __ldg(src + ch * stride);
        n += __ldg(cnt + (int64_t)ch * a.count);
    }
    if (n > 0) a.centers[(h * a.count + c) * a.D + d] = total / (float)n;
}

// Exclusive prefix of the per-(cluster, chunk) counts in cluster-major,
// chunk-minor order: one CTA per head, each thread a contiguous run of that
// order, the run totals scanned across warps (integer sums: any order).
__global__ void __launch_bounds__(256) cluster_offsets_kernel(ClusterArgs a) {
    pdl_wait();
    pdl_open();
    __shared__ int wsum[8];
    const int64_t h = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int len = a.count * a.nchunk;
    const int per = (len + 255) / 256;
    const int q0 = min(tid * per, len), q1 = min(q0 + per, len);
    auto at = [&](int q) { return ((int64_t)h * a.nchunk + q % a.nchunk) * a.count + q / a.nchunk; };
    int mine = 0;
    for (int q = q0; q < q1; ++q) mine += a.pcnt[at(q)];
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int run = incl - mine;
    for (int w = 0; w < warp; ++w) run += wsum[w];
    for (int q = q0; q < q1; ++q) {
        const int64_t i = at(q);
        const int c = a.pcnt[i];
        a.off[i] = run;
        run += c;
    }
}

// Stable counting-sort scatter: the rank of token j among the chunk's
// earlier tokens of its cluster = rank inside its warp (match mask) plus the
// counts of the warps before it.
__global__ void __launch_bounds__(256) cluster_scatter_kernel(ClusterArgs a) {
    pdl_wait();
    pdl_open();
    __shared__ int wcnt[8][kMaxClusters];
    const int64_t h = blockIdx.y;
    const int chunk = blockIdx.x;
    const int64_t base = (int64_t)chunk * kChunk;
    const int nvalid = (int)min((int64_t)kChunk, a.S - base);
    const int j = threadIdx.x, warp = j >> 5, lane = j & 31;
    for (int i = j; i < 8 * kMaxClusters; i += 256) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    const int c = j < nvalid ? a.labels[h * a.S + base + j] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, c);
    const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
    if (c >= 0 && rank_in_warp == 0) wcnt[warp][c] = __popc(same);
    __syncthreads();
    if (c < 0) return;
    int rank = rank_in_warp;
    for (int w = 0; w < warp; ++w) rank += wcnt[w][c];
    const int dst = a.off[((int64_t)h * a.nchunk + chunk) * a.count + c] + rank;
    a.pi[h * a.S + dst] = (int32_t)(base + j);
}

namespace {

void linspace_indices(int64_t S, int count, long long* out) {
    // torch.linspace(0, S-1, count) in float32, then .long() (core.py:148):
    // first half start + i*step, second half end - (count-1-i)*step.
    if (count == 1) { out[0] = 0; return; }
    volatile float start = 0.0f, end = (float)(S - 1);
    const float step = (end - start) / (float)(count - 1);
    const int half = count / 2;
    for (int i = 0; i < count; ++i) {
        volatile float prod = i < half ? step * (float)i : step * (float)(count - 1 - i);
        const float val = i < half ? start + prod : end - prod;
        out[i] = (long long)val;
    }
}

template <typename T>
int run(const vcb_group_args* p, cudaStream_t st) {
    const int count = (int)(p->clusters < p->s ? p->clusters : p->s);
    const int nchunk = (int)((p->s + kChunk - 1) / kChunk);
    char* ws = static_cast<char*>(p->workspace);
    ClusterArgs a{};
    a.v = p->v; a.S = p->s; a.D = p->d; a.count = count; a.nchunk = nchunk;
    a.centers = p->centers_out; a.pi = p->pi;
    size_t o = 0;
    auto take = [&](size_t bytes) { char* r = ws + o; o += (bytes + 255) & ~size_t(255); return r; };
    a.labels = reinterpret_cast<uint8_t*>(take((size_t)p->heads * p->s));
    a.psum = reinterpret_cast<float*>(take((size_t)p->heads * nchunk * count * 128 * sizeof(float)));
    a.pcnt = reinterpret_cast<int32_t*>(take((size_t)p->heads * nchunk * count * sizeof(int32_t)));
    a.off = reinterpret_cast<int32_t*>(take((size_t)p->heads * nchunk * count * sizeof(int32_t)));
    InitIdx init{};
    linspace_indices(p->s, count, init.idx);
    VCB_CUDA(launch_pdl(cluster_init_kernel<T>, dim3((unsigned)p->heads), dim3(256), 0, st, a, p->centers_in,
                        init));
    const size_t cen2_bytes = (size_t)((count + 3) / 4) * 128 * 8 * sizeof(float);
    const size_t subs_bytes = (size_t)8 * kSumGroup * 128 * sizeof(float);
    const size_t fast_smem = (size_t)kChunk * 128 * sizeof(T) + (cen2_bytes > subs_bytes ? cen2_bytes : subs_bytes);
    if (p->d == 128) {
        VCB_CUDA(cudaFuncSetAttribute(cluster_assign128_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)fast_smem));
        VCB_CUDA(cudaFuncSetAttribute(cluster_assign128_kernel<T>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      (int)cudaSharedmemCarveoutMaxShared));
    }
    for (int it = 0; it < p->iterations; ++it) {
        if (p->d == 128)
            VCB_CUDA(launch_pdl(cluster_assign128_kernel<T>, dim3(nchunk, (unsigned)p->heads), dim3(256), fast_smem,
                                st, a));
        else
            VCB_CUDA(launch_pdl(cluster_assign_kernel<T>, dim3(nchunk, (unsigned)p->heads), dim3(256), 0, st, a));
        VCB_CUDA(launch_pdl(cluster_update_kernel, dim3((unsigned)p->heads, (unsigned)count), dim3(128), 0, st, a));
    }
    VCB_CUDA(launch_pdl(cluster_offsets_kernel, dim3((unsigned)p->heads), dim3(256), 0, st, a));
    VCB_CUDA(launch_pdl(cluster_scatter_kernel, dim3(nchunk, (unsigned)p->heads), dim3(256), 0, st, a));
    return VCB_OK;
}

}  // namespace

size_t group_workspace_bytes(int64_t heads, int64_t s, int d, int clusters) {
    (void)d;
    const int64_t count = clusters < s ? clusters : s;
    const int64_t nchunk = (s + kChunk - 1) / kChunk;
    auto r = [](size_t b) { return (b + 255) & ~size_t(255); };
    return r((size_t)(heads * s)) + r((size_t)(heads * nchunk * count * 128 * 4)) +
           2 * r((size_t)(heads * nchunk * count * 4));
}

int group_run(const vcb_group_args* p, cudaStream_t st) {
    switch (p->dtype) {
        case VCB_F32: return run<float>(p, st);
        case VCB_F16: return run<__half>(p, st);
        case VCB_BF16: return run<__nv_bfloat16>(p, st);
        default: return fail(VCB_ERR_INVALID_ARGUMENT, "unknown dtype %d", p->dtype);
    }
}

}  // namespace vcb
