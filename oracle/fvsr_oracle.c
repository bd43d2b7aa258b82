/*
 * fvsr_oracle.c — CPU restatement of FlashVSR's LCSA hot path (block selection + block-sparse attention).
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the sm_100a kernels. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it; the product library never links, loads or
 * calls it, and nothing here is a fallback for the CUDA path.
 *
 * Every function restates one piece of the reference (paths relative to the xocialize/mlx-flashvsr-swift tree):
 *   orc_window_partition / orc_window_reverse  Sources/FlashVSRMLX/DiT.swift:113-126
 *   orc_prepare                                Sources/FlashVSRMLX/DiT.swift:34-47 (WanRMSNorm), 100-107 (ropeApply),
 *                                              113-118 (windowPartition) — the q/k/v side of blockForward, 497-506
 *   orc_local_block_mask                       Sources/FlashVSRMLX/DiT.swift:130-145
 *   orc_geometry_topk                          Sources/FlashVSRMLX/DiT.swift:478-485
 *   orc_pool                                   Sources/FlashVSRMLX/DiT.swift:161-162 (fp32 mean over 128 tokens)
 *   orc_select                                 Sources/FlashVSRMLX/DiT.swift:158-174 (draftBlockMaskAndProbs)
 *   orc_mask_to_lists                          Sources/FlashVSRMLX/SparseAttention.swift:175-177 (kcnt / kidx)
 *   orc_attention(_fast)                       Sources/FlashVSRMLX/DiT.swift:279-313 and oracle/block_sparse_attn.py:20-38
 *                                              (softmax attention restricted to the selected blocks, empty → 0)
 *
 * Fixed fp32 operation order. MLX does not document its reduction orders, so bit-level agreement with MLX is not
 * claimed; the selection mask is instead defined by the order below, which the GPU kernels reproduce exactly:
 *   pool    : four sequential fp32 sums over tokens [0,32) [32,64) [64,96) [96,128), combined (s0+s1)+(s2+s3),
 *             times 1/128 (exact for a power of two).
 *   score   : acc = fmaf(pq[e], pk[e], acc) for e = 0..127 from acc = 0, then acc / sqrtf(128) (IEEE division).
 *   softmax : m = max over the row; e_j = fvsr_exp(s_j - m); 32 partial sums, partial l adds e_j for j ≡ l (mod 32)
 *             in increasing j; then a butterfly v[l] += v[l ^ o] for o = 16, 8, 4, 2, 1; p_j = e_j / sum.
 *   exp     : fvsr_exp below — Cody–Waite range reduction (W. J. Cody, W. Waite, "Software Manual for the
 *             Elementary Functions", 1980) with a degree-7 Taylor polynomial evaluated by Horner's rule in fmaf.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_BLOCK 128
#define ORC_D 128

/* ------------------------------------------------------------------------------------------------------------ */
/* exp — the softmax exponential shared (by specification) with the GPU selection kernel.                          */
/* ------------------------------------------------------------------------------------------------------------ */

static inline float orc_pow2i(int n) {          /* 2^n for n in [-126, 127], built from the exponent bits */
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)(n + 127) << 23;
    return v.f;
}

/* e^x in fp32. Range reduction: n = rint(x·log2 e), r = x − n·ln2 with ln 2 split into a 24-bit-exact high part
 * (0x3f317200) and a low correction, both applied by fmaf. e^r by the Taylor series Σ r^k/k!, k ≤ 7 (|r| ≤ 0.347,
 * truncation < 6e-9 relative). Scaling by 2^n is one IEEE multiply for −126 ≤ n ≤ 127 and two (the first exact)
 * outside that range, so subnormal results round exactly once and e^x just below the overflow bound stays finite. */
float fvsr_exp(float x) {
    if (x != x) return x;
    if (x < -104.0f) return 0.0f;                 /* below half the smallest subnormal */
    if (x > 88.72f) return INFINITY;
    const float log2e = 1.44269502925872802734375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.428606765330187045e-06f;
    float n = rintf(x * log2e);
    float r = fmaf(-n, ln2_hi, x);
    r = fmaf(-n, ln2_lo, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) return (p * orc_pow2i(ni - 1)) * 2.0f;
    if (ni >= -126) return p * orc_pow2i(ni);
    return (p * orc_pow2i(ni + 64)) * orc_pow2i(-64);
}

/* ------------------------------------------------------------------------------------------------------------ */
/* Layout: window partition (2, 8, 8) on the patch grid, DiT.swift:113-126.                                       */
/* ------------------------------------------------------------------------------------------------------------ */

/* x (B, F, H, W, C) → (B·F/2·H/8·W/8, 128, C); windows ordered (nf, nh, nw), tokens (wf, wh, ww). */
int orc_window_partition(const float* x, int b, int f, int h, int w, int c, float* out) {
    if (f % 2 || h % 8 || w % 8) return 1;
    const int nf = f / 2, nh = h / 8, nw = w / 8;
    for (int bb = 0; bb < b; ++bb)
        for (int ff = 0; ff < f; ++ff)
            for (int hh = 0; hh < h; ++hh)
                for (int ww = 0; ww < w; ++ww) {
                    const int64_t win = (((int64_t)bb * nf + ff / 2) * nh + hh / 8) * nw + ww / 8;
                    const int tok = ((ff % 2) * 8 + hh % 8) * 8 + ww % 8;
                    const float* src = x + ((((int64_t)bb * f + ff) * h + hh) * w + ww) * c;
                    memcpy(out + (win * 128 + tok) * c, src, sizeof(float) * (size_t)c);
                }
    return 0;
}

/* Inverse of orc_window_partition, back to (B, F·H·W, C) token order. */
int orc_window_reverse(const float* x, int b, int f, int h, int w, int c, float* out) {
    if (f % 2 || h % 8 || w % 8) return 1;
    const int nf = f / 2, nh = h / 8, nw = w / 8;
    for (int bb = 0; bb < b; ++bb)
        for (int ff = 0; ff < f; ++ff)
            for (int hh = 0; hh < h; ++hh)
                for (int ww = 0; ww < w; ++ww) {
                    const int64_t win = (((int64_t)bb * nf + ff / 2) * nh + hh / 8) * nw + ww / 8;
                    const int tok = ((ff % 2) * 8 + hh % 8) * 8 + ww % 8;
                    float* dst = out + ((((int64_t)bb * f + ff) * h + hh) * w + ww) * c;
                    memcpy(dst, x + (win * 128 + tok) * c, sizeof(float) * (size_t)c);
                }
    return 0;
}

/* ------------------------------------------------------------------------------------------------------------ */
/* Local block mask, DiT.swift:130-145, and the integer top-k of DiT.swift:482.                                   */
/* ------------------------------------------------------------------------------------------------------------ */

/* out (s, s) with s = bh·bw: key block (kr, kc) visible to query block (qr, qc) iff
 * kr ∈ [qr − r/2, qr − r/2 + r − 1] and kc ∈ [qc − r/2, qc − r/2 + r − 1], unclamped. */
void orc_local_block_mask(int bh, int bw, int r, uint8_t* out) {
    const int half = r / 2, s = bh * bw;
    for (int qr = 0; qr < bh; ++qr)
        for (int qc = 0; qc < bw; ++qc)
            for (int kr = 0; kr < bh; ++kr)
                for (int kc = 0; kc < bw; ++kc) {
                    const int in_row = kr >= qr - half && kr <= qr - half + r - 1;
                    const int in_col = kc >= qc - half && kc <= qc - half + r - 1;
                    out[(qr * bw + qc) * s + kr * bw + kc] = (uint8_t)(in_row && in_col);
                }
}

/* topk = Int(Double(s·s)·ratio) − 1 (Swift's Int() truncates toward zero). */
int orc_geometry_topk(int s, double ratio) { return (int)((double)s * (double)s * ratio) - 1; }

/* ------------------------------------------------------------------------------------------------------------ */
/* Pooling, DiT.swift:161-162.                                                                                    */
/* ------------------------------------------------------------------------------------------------------------ */

static inline float orc_bf16_to_f32(uint16_t v) {
    union { uint32_t u; float f; } t;
    t.u = (uint32_t)v << 16;
    return t.f;
}

/* x (nblocks·128, C) in fp32 (dtype 0) or bf16 (dtype 1) → out (nblocks, C) fp32 block means. */
void orc_pool(const void* x, int dtype, int64_t nblocks, int64_t c, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblocks; ++b) {
        for (int64_t ch = 0; ch < c; ++ch) {
            float part[4];
            for (int g = 0; g < 4; ++g) {
                float acc = 0.0f;
                for (int t = 32 * g; t < 32 * g + 32; ++t) {
                    const int64_t idx = (b * ORC_BLOCK + t) * c + ch;
                    const float v = dtype == 0 ? ((const float*)x)[idx] : orc_bf16_to_f32(((const uint16_t*)x)[idx]);
                    acc = acc + v;
                }
                part[g] = acc;
            }
            out[b * c + ch] = ((part[0] + part[1]) + (part[2] + part[3])) * 0.0078125f;
        }
    }
}

/* ------------------------------------------------------------------------------------------------------------ */
/* The q/k side of blockForward: WanRMSNorm (DiT.swift:34-47), ropeApply (DiT.swift:100-107), windowPartition      */
/* (DiT.swift:113-118).                                                                                           */
/* ------------------------------------------------------------------------------------------------------------ */

static inline uint16_t orc_f32_to_bf16(float f) {   /* round to nearest even (NaN stays NaN) */
    union { float f; uint32_t u; } v;
    v.f = f;
    if ((v.u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((v.u >> 16) | 0x40u);
    return (uint16_t)((v.u + 0x7FFFu + ((v.u >> 16) & 1u)) >> 16);
}

static inline float orc_round_t(float x, int dtype) { return dtype ? orc_bf16_to_f32(orc_f32_to_bf16(x)) : x; }

/* x (F·H·W, C = heads·128) in token order (row (f·H + y)·W + x), dtype 0 fp32 / 1 bf16 → out, same shape and dtype,
 * in window order (window (f/2, y/8, x/8), token (f%2, y%8, x%8)). weight: (C) in dtype, or NULL for no norm; cosv /
 * sinv: (F·H·W, 64) fp32 rows per token, or NULL for no rotation. T = the storage type.
 *   norm  : ss = Σ x² as 32 partials — partial l = (s0 + s1) + (s2 + s3), s_e summing x·x over channels
 *           128·i + 4l + e for i = 0..heads−1 in order — combined by the butterfly v[l] = v[l] + v[l ^ o] for
 *           o = 16, 8, 4, 2, 1 (all l at once);
 *           inv = 1/√(ss / C + eps) correctly rounded (evaluated in double); n = T(x·inv); y = T(n·w)
 *           (DiT.swift:44-45: normalise in fp32, cast to T, times the weight).
 *   rotate: for each head, pair (2j, 2j+1) = (re, im): re' = T(re·cos_j − im·sin_j), im' = T(re·sin_j + im·cos_j)
 *           with every product and sum an fp32 operation (DiT.swift:103-106). */
int orc_prepare(const void* x, int dtype, int f, int h, int w, int heads, const void* weight, float eps,
                const float* cosv, const float* sinv, void* out) {
    if (f % 2 || h % 8 || w % 8 || heads < 1) return 1;
    const int c = heads * ORC_D, nh = h / 8, nw = w / 8;
    const int64_t ntok = (int64_t)f * h * w;
#pragma omp parallel for schedule(static)
    for (int64_t tok = 0; tok < ntok; ++tok) {
        float* row = (float*)malloc(sizeof(float) * (size_t)c);
        const int ff = (int)(tok / ((int64_t)h * w)), yy = (int)(tok / w % h), xx = (int)(tok % w);
        for (int ch = 0; ch < c; ++ch)
            row[ch] = dtype == 0 ? ((const float*)x)[tok * c + ch] : orc_bf16_to_f32(((const uint16_t*)x)[tok * c + ch]);
        if (weight) {
            float v[32], t[32];
            for (int l = 0; l < 32; ++l) {
                float se[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int i = 0; i < heads; ++i)
                    for (int e = 0; e < 4; ++e) {
                        const float xv = row[ORC_D * i + 4 * l + e];
                        se[e] = se[e] + xv * xv;
                    }
                v[l] = (se[0] + se[1]) + (se[2] + se[3]);
            }
            for (int o = 16; o > 0; o >>= 1) {
                for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ o];
                memcpy(v, t, sizeof(v));
            }
            const float ms = v[0] / (float)c;
            const float a = ms + eps;
            const float inv = (float)(1.0 / sqrt((double)a));
            for (int ch = 0; ch < c; ++ch) {
                const float wv = dtype == 0 ? ((const float*)weight)[ch] : orc_bf16_to_f32(((const uint16_t*)weight)[ch]);
                const float n = orc_round_t(row[ch] * inv, dtype);
                row[ch] = orc_round_t(n * wv, dtype);
            }
        }
        if (cosv) {
            for (int i = 0; i < heads; ++i)
                for (int j = 0; j < ORC_D / 2; ++j) {
                    const float re = row[ORC_D * i + 2 * j], im = row[ORC_D * i + 2 * j + 1];
                    const float cs = cosv[tok * 64 + j], sn = sinv[tok * 64 + j];
                    row[ORC_D * i + 2 * j] = orc_round_t(re * cs - im * sn, dtype);
                    row[ORC_D * i + 2 * j + 1] = orc_round_t(re * sn + im * cs, dtype);
                }
        }
        const int64_t win = ((int64_t)(ff / 2) * nh + yy / 8) * nw + xx / 8;
        const int t = ((ff % 2) * 8 + yy % 8) * 8 + xx % 8;
        const int64_t o = (win * ORC_BLOCK + t) * c;
        for (int ch = 0; ch < c; ++ch) {
            if (dtype == 0)
                ((float*)out)[o + ch] = row[ch];
            else
                ((uint16_t*)out)[o + ch] = orc_f32_to_bf16(row[ch]);
        }
        free(row);
    }
    return 0;
}

/* ------------------------------------------------------------------------------------------------------------ */
/* Selection, DiT.swift:158-174.                                                                                  */
/* ------------------------------------------------------------------------------------------------------------ */

static int orc_cmp_float(const void* a, const void* b) {
    const float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

/* Block probabilities of one (head, query block) row: scores, local mask, softmax in the fixed order above. */
static void orc_softmax_row(int heads, int h, int i, int nk, int s, const uint8_t* local, float sqrt_d,
                            const float* pq, const float* pk, float* prow) {
    const int64_t ld = (int64_t)heads * ORC_D;
    const float* qv = pq + (int64_t)i * ld + (int64_t)h * ORC_D;
    float m = -INFINITY;
    for (int j = 0; j < nk; ++j) {
        float sc;
        if (local[(i % s) * s + (j % s)]) {
            const float* kv = pk + (int64_t)j * ld + (int64_t)h * ORC_D;
            float acc = 0.0f;
            for (int e = 0; e < ORC_D; ++e) acc = fmaf(qv[e], kv[e], acc);
            sc = acc / sqrt_d;
        } else {
            sc = -INFINITY;
        }
        prow[j] = sc;
        if (sc > m) m = sc;
    }
    float lane[32];
    for (int l = 0; l < 32; ++l) lane[l] = 0.0f;
    for (int j = 0; j < nk; ++j) {
        const float e = fvsr_exp(prow[j] - m);
        prow[j] = e;
        lane[j & 31] = lane[j & 31] + e;
    }
    for (int o = 16; o >= 1; o >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = lane[l] + lane[l ^ o];
        memcpy(lane, nxt, sizeof(lane));
    }
    const float sum = lane[0];
    for (int j = 0; j < nk; ++j) prow[j] = prow[j] / sum;
}

/* pq (nq, H·128), pk (nk, H·128) pooled fp32; local (s, s) 0/1 tiled over every (query slice, key slice) pair.
 * Outputs: probs (H, nq, nk) fp32; mask (H, nq, nk) 0/1 (optional); kidx (H, nq, nk) with the kept key blocks of
 * each row first, ascending (optional); kcnt (H, nq) (optional). The threshold is joint over each (head, query slice)
 * row of (nq/q_slices)·nk probabilities: keep p > the (k+1)-th largest, k = min(n − 1, topk).
 * Returns 0, or 1 on a bad shape. */
int orc_select(int heads, int nq, int nk, int s, int q_slices, const uint8_t* local, int topk,
               const float* pq, const float* pk, float* probs, uint8_t* mask, int32_t* kidx, int32_t* kcnt) {
    if (heads <= 0 || s <= 0 || q_slices <= 0 || nq % s || nk % s || nq % q_slices || topk < 0) return 1;
    const float sqrt_d = sqrtf((float)ORC_D);
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t r = 0; r < (int64_t)heads * nq; ++r) {
        const int h = (int)(r / nq), i = (int)(r % nq);
        orc_softmax_row(heads, h, i, nk, s, local, sqrt_d, pq, pk, probs + r * nk);
    }
    const int nqs = nq / q_slices;
    const int64_t n = (int64_t)nqs * nk;
    const int64_t k = topk < n - 1 ? topk : n - 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t row = 0; row < (int64_t)heads * q_slices; ++row) {
        const int h = (int)(row / q_slices), t = (int)(row % q_slices);
        const float* base = probs + ((int64_t)h * nq + (int64_t)t * nqs) * nk;   /* contiguous (nqs, nk) */
        float* tmp = (float*)malloc(sizeof(float) * (size_t)n);
        memcpy(tmp, base, sizeof(float) * (size_t)n);
        qsort(tmp, (size_t)n, sizeof(float), orc_cmp_float);
        const float thr = tmp[n - 1 - k];
        free(tmp);
        for (int ii = 0; ii < nqs; ++ii) {
            const int64_t qrow = (int64_t)h * nq + (int64_t)t * nqs + ii;
            const float* p = probs + qrow * nk;
            int cnt = 0;
            for (int j = 0; j < nk; ++j) {
                const int keep = p[j] > thr;
                if (mask) mask[qrow * nk + j] = (uint8_t)keep;
                if (keep && kidx) kidx[qrow * nk + cnt] = j;
                cnt += keep;
            }
            if (kidx)
                for (int j = cnt; j < nk; ++j) kidx[qrow * nk + j] = -1;
            if (kcnt) kcnt[qrow] = cnt;
        }
    }
    return 0;
}

/* SparseAttention.swift:175-177: sel = mask > 0.5; kcnt = Σ sel; kidx = selected key blocks first (ascending here;
 * the reference's order only changes the summation order), the rest −1. */
void orc_mask_to_lists(const float* mask, int heads, int nq, int nk, int32_t* kidx, int32_t* kcnt) {
    for (int64_t r = 0; r < (int64_t)heads * nq; ++r) {
        int cnt = 0;
        for (int j = 0; j < nk; ++j)
            if (mask[r * nk + j] > 0.5f) kidx[r * nk + cnt++] = j;
        for (int j = cnt; j < nk; ++j) kidx[r * nk + j] = -1;
        kcnt[r] = cnt;
    }
}

/* ------------------------------------------------------------------------------------------------------------ */
/* Attention over the kept (query block, key block) pairs, DiT.swift:279-313 / block_sparse_attn.py:20-38.        */
/* ------------------------------------------------------------------------------------------------------------ */

static inline float orc_load(const void* x, int dtype, int64_t idx) {
    return dtype == 0 ? ((const float*)x)[idx] : orc_bf16_to_f32(((const uint16_t*)x)[idx]);
}

#define ORC_ATTN_NAME orc_attention
#define ORC_ACC double
#define ORC_EXP exp
#include "attn_body.inc"
#undef ORC_ATTN_NAME
#undef ORC_ACC
#undef ORC_EXP

#define ORC_ATTN_NAME orc_attention_fast
#define ORC_ACC float
#define ORC_EXP expf
#include "attn_body.inc"
#undef ORC_ATTN_NAME
#undef ORC_ACC
#undef ORC_EXP

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
