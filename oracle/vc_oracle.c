/*
 * CPU restatement of the VC-Attention preprocessing contract.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the bit-exact checker for the CUDA
 * kernels in vc-attention_b200/csrc.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it.  The product never links it.
 *
 * Every function restates a piece of the reference algorithm
 * (czfsdg/vc-attention, src/vc_attention/core.py); the citation is given on
 * each function.  Where the reference leaves a floating-point reduction order
 * unspecified (torch .mean / .sum / scatter_add / BLAS), this file fixes one
 * order and the CUDA kernels use exactly the same one:
 *
 *   K channel mean   : per head, in original token order (before any
 *                      permutation), rows are split into chunks of VCO_KSUM_CHUNK
 *                      rows; inside a chunk, row r goes to lane (r % LANES);
 *                      each lane sums its rows in increasing order, the chunk
 *                      sum adds lanes 0..LANES-1 in order, the head total adds
 *                      chunks in order, mean = total / S.
 *   V block mean     : per (tile, channel) token j of the tile goes to
 *                      partial sum j % 4 (each in tile order), then
 *                      (p0 + p1) + (p2 + p3).
 *   Lloyd distances  : ||x||^2, ||c||^2 and x.c are fmaf chains over channels
 *                      0..D-1; distance = (xx + cc) - 2*xc, first minimum wins.
 *   Lloyd sums       : tokens are split into chunks of VCO_LLOYD_CHUNK and
 *                      each chunk into sub-chunks of VCO_LLOYD_SUB; inside a
 *                      sub-chunk each cluster sums its tokens in token order;
 *                      a chunk adds its sub-chunk sums in order (from 0), the
 *                      total adds chunk sums in order; centre = sum / count.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off, no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define VCO_KSUM_CHUNK 256
#define VCO_KSUM_LANES 16
#define VCO_LLOYD_CHUNK 256
#define VCO_LLOYD_SUB 32

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

int vco_constants(int which) {
    switch (which) {
        case 0: return VCO_KSUM_CHUNK;
        case 1: return VCO_KSUM_LANES;
        case 2: return VCO_LLOYD_CHUNK;
        case 3: return VCO_LLOYD_SUB;
        default: return -1;
    }
}

/* torch float8_e4m3fn conversion of an already clamped value (core.py:113,
 * core.py:121, core.py:332): round to nearest even; |x| >= 448 saturates
 * (only x = +-448 reaches it after the reference's clamp). */
uint8_t vco_e4m3_encode(float x) {
    uint8_t sign = (f2u(x) >> 24) & 0x80;
    float a = fabsf(x);
    if (isnan(x)) return 0x7F;
    if (a >= 448.0f) return sign | 0x7E;
    if (a < 0.015625f) {                      /* below 2^-6: step 2^-9 */
        float q = rintf(a * 512.0f);          /* exact scaling, RNE */
        return sign | (uint8_t)q;             /* q == 8 is the smallest normal */
    }
    int e2;
    frexpf(a, &e2);                           /* a = m * 2^e2, m in [0.5, 1) */
    int e = e2 - 1;                           /* a in [2^e, 2^(e+1)) */
    float step = ldexpf(1.0f, e - 3);
    float q = rintf(a / step);                /* exact division by 2^k */
    int mant = (int)q - 8;
    if (mant == 8) { e += 1; mant = 0; }
    int biased = e + 7;
    uint32_t code = ((uint32_t)biased << 3) | (uint32_t)mant;
    if (code > 0x7E) code = 0x7E;
    return sign | (uint8_t)code;
}

/* E4M3 decode (csrc/kernels.cu:54-59 for positive codes, plus sign). */
float vco_e4m3_decode(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
    float v;
    if (e == 15 && m == 7) v = NAN;
    else if (e == 0) v = ldexpf((float)m, -9);
    else v = ldexpf(1.0f + m * 0.125f, e - 7);
    return s ? -v : v;
}

void vco_e4m3_encode_n(const float* x, uint8_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = vco_e4m3_encode(x[i]);
}

void vco_e4m3_decode_n(const uint8_t* b, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = vco_e4m3_decode(b[i]);
}

static const float C1 = 11.541560173034668f;    /* 8 * log2(e) rounded to fp32 */
static const float C2 = 119.6500015258789f;     /* 119.65 rounded to fp32 */

static inline uint8_t clamp_code(float u) {
    if (!(u > 0.0f)) return 0;                    /* also maps NaN and -inf to 0 */
    float r = rintf(u);
    if (r > 120.0f) r = 120.0f;
    return (uint8_t)r;
}

/* ExpCast as the contract defines it: one FP32 FMA, RNE, clamp [0,120]
 * (core.py:60-68 docstring; csrc/kernels.cu:61-65). */
void vco_expcast_fma(const float* x, uint8_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = clamp_code(fmaf(x[i], C1, C2));
}

/* The fused kernel's form of the ExpCast encode, for counting how often it
 * differs from the reference's: u = fmaf(s, a, b) in units of 2^-24 (s the
 * raw FP32 logit q8 . k8, a and b the per-row slope and offset the kernel
 * derived from the scales and the running max), code = RNE(u * 2^24) with
 * negatives at 0 (the kernel's cvt.rn.relu to the f16 subnormal grid).  No
 * upper clamp: the kernel shifts b so that the row's largest code is <= 120. */
void vco_fused_codes(const float* s, const float* a, const float* b, int64_t n, uint8_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        const float u = fmaf(s[i], a[i], b[i]) * 16777216.0f;
        if (!(u > 0.0f)) { out[i] = 0; continue; }
        const float r = rintf(u);
        out[i] = (uint8_t)(r > 255.0f ? 255.0f : r);
    }
}

/* ExpCast exactly as core.py:67-68 evaluates it: widened product and sum in
 * FP64, one cast to FP32, torch.round (RNE), clamp. */
void vco_expcast_fp64(const float* x, uint8_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        double d = (double)x[i] * 11.541560173034668 + 119.6500015258789;
        out[i] = clamp_code((float)d);
    }
}

/* Normalised Sylvester transform of one row (core.py:71-85): pad to the next
 * power of two, butterflies with stride 1, 2, 4, ... each producing
 * (left + right, left - right), then multiply by fp32(width^-0.5). */
void vco_hadamard_rows(const float* x, int64_t rows, int d, float* out) {
    int width = 1;
    while (width < d) width <<= 1;
    const float norm = (float)pow((double)width, -0.5);
    float tmp[4096];
    for (int64_t r = 0; r < rows; ++r) {
        const float* src = x + r * d;
        float* dst = out + r * width;
        for (int c = 0; c < width; ++c) tmp[c] = c < d ? src[c] : 0.0f;
        for (int step = 1; step < width; step <<= 1) {
            for (int base = 0; base < width; base += 2 * step) {
                for (int t = 0; t < step; ++t) {
                    float left = tmp[base + t], right = tmp[base + step + t];
                    tmp[base + t] = left + right;
                    tmp[base + step + t] = left - right;
                }
            }
        }
        for (int c = 0; c < width; ++c) dst[c] = tmp[c] * norm;
    }
}

/* K channel mean over tokens (core.py:95-96) in the fixed chunk/lane order
 * documented at the top of this file.  k: [heads, S, D], mean: [heads, D]. */
void vco_k_mean(const float* k, int64_t heads, int64_t S, int D, float* mean) {
    for (int64_t h = 0; h < heads; ++h) {
        const float* kh = k + h * S * D;
        for (int c = 0; c < D; ++c) {
            float total = 0.0f;
            for (int64_t base = 0; base < S; base += VCO_KSUM_CHUNK) {
                int64_t end = base + VCO_KSUM_CHUNK < S ? base + VCO_KSUM_CHUNK : S;
                float chunk = 0.0f;
                for (int lane = 0; lane < VCO_KSUM_LANES; ++lane) {
                    float part = 0.0f;
                    for (int64_t r = base + lane; r < end; r += VCO_KSUM_LANES) part += kh[r * D + c];
                    chunk += part;
                }
                total += chunk;
            }
            mean[h * D + c] = total / (float)S;
        }
    }
}

/* Block quantisation (core.py:118-135): one scale per (block rows x 128
 * channels); scale = amax / 448 (0 -> 1); payload = e4m3(clamp(x / scale)).
 * x: [heads, S, W] with W <= 128.  payload: [heads, S_pad, 128] (zero padded
 * rows and channels), scales: [heads, ceil(S / block)]. */
void vco_quant_blocks(const float* x, int64_t heads, int64_t S, int W, int block,
                      int64_t S_pad, uint8_t* payload, float* scales) {
    int64_t nblk = (S + block - 1) / block;
    memset(payload, 0, (size_t)(heads * S_pad * 128));
    for (int64_t h = 0; h < heads; ++h) {
        for (int64_t b = 0; b < nblk; ++b) {
            int64_t r0 = b * block, r1 = r0 + block < S ? r0 + block : S;
            float amax = 0.0f;
            for (int64_t r = r0; r < r1; ++r)
                for (int c = 0; c < W; ++c) {
                    float a = fabsf(x[(h * S + r) * W + c]);
                    if (a > amax) amax = a;
                }
            float scale = amax / 448.0f;
            if (scale == 0.0f) scale = 1.0f;
            scales[h * nblk + b] = scale;
            for (int64_t r = r0; r < r1; ++r)
                for (int c = 0; c < W; ++c) {
                    float q = x[(h * S + r) * W + c] / scale;
                    if (q > 448.0f) q = 448.0f;
                    if (q < -448.0f) q = -448.0f;
                    payload[(h * S_pad + r) * 128 + c] = vco_e4m3_encode(q);
                }
        }
    }
}

/* torch.linspace(0, S-1, count) in float32 followed by .long()
 * (core.py:148): first half start + i*step, second half end - (n-1-i)*step. */
void vco_linspace_indices(int64_t S, int count, int64_t* out) {
    if (count == 1) { out[0] = 0; return; }
    const float start = 0.0f, end = (float)(S - 1);
    const float step = (end - start) / (float)(count - 1);
    const int half = count / 2;
    for (int i = 0; i < count; ++i) {
        float v = i < half ? start + step * (float)i : end - step * (float)(count - 1 - i);
        out[i] = (int64_t)v;
    }
}

static float dot_fma(const float* a, const float* b, int D) {
    float acc = 0.0f;
    for (int d = 0; d < D; ++d) acc = fmaf(a[d], b[d], acc);
    return acc;
}

/* Lloyd clustering with a stable permutation (core.py:138-163).
 * v: [heads, S, D]; centers_in: [heads, count, D] or NULL (equispaced init);
 * centers_out: [heads, count, D]; pi: [heads, S]; labels: [heads, S] (last
 * iteration's assignment).  count = min(clusters, S).  Returns count. */
int vco_group_values(const float* v, int64_t heads, int64_t S, int D, int clusters, int iters,
                     const float* centers_in, float* centers_out, int32_t* pi, uint8_t* labels) {
    int count = clusters < S ? clusters : (int)S;
    int64_t idx[256];
    float* cen = (float*)malloc(sizeof(float) * count * D);
    float* sums = (float*)malloc(sizeof(float) * count * D);
    float* part = (float*)malloc(sizeof(float) * count * D);
    float* sub = (float*)malloc(sizeof(float) * count * D);
    int64_t* counts = (int64_t*)malloc(sizeof(int64_t) * count);
    float* cnorm = (float*)malloc(sizeof(float) * count);
    vco_linspace_indices(S, count, idx);
    for (int64_t h = 0; h < heads; ++h) {
        const float* vh = v + h * S * D;
        uint8_t* lab = labels + h * S;
        if (centers_in) memcpy(cen, centers_in + h * count * D, sizeof(float) * count * D);
        else for (int c = 0; c < count; ++c) memcpy(cen + c * D, vh + idx[c] * D, sizeof(float) * D);
        for (int it = 0; it < iters; ++it) {
            for (int c = 0; c < count; ++c) cnorm[c] = dot_fma(cen + c * D, cen + c * D, D);
            memset(sums, 0, sizeof(float) * count * D);
            memset(counts, 0, sizeof(int64_t) * count);
            for (int64_t base = 0; base < S; base += VCO_LLOYD_CHUNK) {
                int64_t end = base + VCO_LLOYD_CHUNK < S ? base + VCO_LLOYD_CHUNK : S;
                for (int64_t t = base; t < end; ++t) {
                    const float* x = vh + t * D;
                    float xx = dot_fma(x, x, D);
                    int best = 0;
                    float bestd = 0.0f;
                    for (int c = 0; c < count; ++c) {
                        float xc = dot_fma(x, cen + c * D, D);
                        float dist = (xx + cnorm[c]) - 2.0f * xc;
                        if (c == 0 || dist < bestd) { bestd = dist; best = c; }
                    }
                    lab[t] = (uint8_t)best;
                }
                memset(part, 0, sizeof(float) * count * D);
                for (int64_t sb = base; sb < end; sb += VCO_LLOYD_SUB) {
                    int64_t se = sb + VCO_LLOYD_SUB < end ? sb + VCO_LLOYD_SUB : end;
                    memset(sub, 0, sizeof(float) * count * D);
                    for (int64_t t = sb; t < se; ++t) {
                        int c = lab[t];
                        counts[c] += 1;
                        for (int d = 0; d < D; ++d) sub[c * D + d] += vh[t * D + d];
                    }
                    for (int i = 0; i < count * D; ++i) part[i] += sub[i];
                }
                for (int i = 0; i < count * D; ++i) sums[i] += part[i];
            }
            for (int c = 0; c < count; ++c)
                if (counts[c] > 0)
                    for (int d = 0; d < D; ++d) cen[c * D + d] = sums[c * D + d] / (float)counts[c];
        }
        memcpy(centers_out + h * count * D, cen, sizeof(float) * count * D);
        /* stable argsort of labels == counting sort in token order */
        int64_t start[257];
        memset(start, 0, sizeof(start));
        for (int64_t t = 0; t < S; ++t) start[lab[t] + 1] += 1;
        for (int c = 0; c < count; ++c) start[c + 1] += start[c];
        for (int64_t t = 0; t < S; ++t) pi[h * S + start[lab[t]]++] = (int32_t)t;
    }
    free(cen); free(sums); free(part); free(sub); free(counts); free(cnorm);
    return count;
}

static float round_mean_dtype(float x, int mean_dtype) {
    if (mean_dtype == 1) {                         /* float16, RNE */
        _Float16 h = (_Float16)x;
        return (float)h;
    }
    if (mean_dtype == 2) {                         /* bfloat16, RNE */
        uint32_t u = f2u(x);
        if ((u & 0x7F800000u) == 0x7F800000u) return x;
        u += 0x7FFFu + ((u >> 16) & 1u);
        u &= 0xFFFF0000u;
        return u2f(u);
    }
    return x;
}

static float mean_dtype_max(int mean_dtype) {
    if (mean_dtype == 1) return 65504.0f;
    if (mean_dtype == 2) return 3.3895313892515355e38f;
    return 3.4028234663852886e38f;
}

/* V tile preparation (core.py:102-115, applied per kv_block tile as at
 * core.py:300-304), after the optional permutation (core.py:288-290).
 * v: [heads, S, Dv]; pi: [heads, S] or NULL.  Outputs per tile t and channel
 * c < 128 (channels >= Dv are zero payload, scale 1, mean 0):
 *   payload[h][t][c][j]  e4m3 residual of token j of the tile (column-major
 *                        tile, zero for padded tokens),
 *   vscale[h][t][c]      per-channel scale,
 *   mu[h][t][c]          mu / vscale rounded to mean_dtype, as fp32. */
void vco_value_tiles(const float* v, int64_t heads, int64_t S, int Dv, const int32_t* pi,
                     int active, int mean_dtype, int kv_block,
                     uint8_t* payload, float* vscale, float* mu) {
    int64_t T = (S + kv_block - 1) / kv_block;
    const float limit = mean_dtype_max(mean_dtype);
    memset(payload, 0, (size_t)(heads * T * 128 * kv_block));
    for (int64_t h = 0; h < heads; ++h) {
        for (int64_t t = 0; t < T; ++t) {
            int64_t s0 = t * kv_block;
            int cnt = (int)(S - s0 < kv_block ? S - s0 : kv_block);
            for (int c = 0; c < 128; ++c) {
                int64_t meta = (h * T + t) * 128 + c;
                uint8_t* out = payload + meta * kv_block;
                if (c >= Dv) { vscale[meta] = 1.0f; mu[meta] = 0.0f; continue; }
                float part[4] = {0.0f, 0.0f, 0.0f, 0.0f}, mean = 0.0f;
                if (active) {
                    for (int j = 0; j < cnt; ++j) {
                        int64_t tok = pi ? pi[h * S + s0 + j] : s0 + j;
                        part[j & 3] += v[(h * S + tok) * Dv + c];
                    }
                    mean = ((part[0] + part[1]) + (part[2] + part[3])) / (float)cnt;
                }
                float amax = 0.0f;
                for (int j = 0; j < cnt; ++j) {
                    int64_t tok = pi ? pi[h * S + s0 + j] : s0 + j;
                    float r = v[(h * S + tok) * Dv + c] - mean;
                    if (fabsf(r) > amax) amax = fabsf(r);
                }
                float scale = amax / 448.0f;
                if (scale == 0.0f) scale = 1.0f;
                float guard = fabsf(mean) / limit;
                if (guard > scale) scale = guard;
                for (int j = 0; j < cnt; ++j) {
                    int64_t tok = pi ? pi[h * S + s0 + j] : s0 + j;
                    float q = (v[(h * S + tok) * Dv + c] - mean) / scale;
                    if (q > 448.0f) q = 448.0f;
                    if (q < -448.0f) q = -448.0f;
                    out[j] = vco_e4m3_encode(q);
                }
                vscale[meta] = scale;
                mu[meta] = round_mean_dtype(mean / scale, mean_dtype);
            }
        }
    }
}
