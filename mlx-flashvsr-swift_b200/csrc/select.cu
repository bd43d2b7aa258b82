// select.cu — LCSA block selection (draftBlockMaskAndProbs, DiT.swift:158-174) on pooled fp32 Q/K.
//
// Kernels (in launch order):
//   select_scores_kernel    block scores pq·pk / sqrt(d) (fixed-order fmaf dot over 128 dims) with the spatial locality
//                           mask (DiT.swift:130-145, computed from (bh, bw, R) instead of a table; −inf outside),
//                           one 32 × 64 (query block × key block) tile per CTA → scores (H, Nq, Nk).
//   select_softmax_kernel   one warp per (head, query block) row: softmax over key blocks, in place → probs, and
//                           pass 1 of the radix select's histogram.
//   select_hist_kernel ×2   passes 2 and 3 of an MSB-first radix select (11 + 11 + 10 bits of the fp32 patterns —
//                           probabilities are ≥ 0, so unsigned order = float order; no sort) that finds, per
//                           (head, query slice) row of n = (Nq/q_slices)·Nk entries, the exact
//                           (min(n−1, topk)+1)-th largest probability, spread over many CTAs per row.
//   select_finish_kernel    compaction of p > threshold into ascending kidx lists, kcnt and the optional 0/1 mask.
//
// Bit-exactness. Every floating-point operation is an explicit round-to-nearest intrinsic (never contracted) in the
// order that the CPU restatement fixes: dot = fmaf chain over e = 0..127; score = dot / sqrtf(128); softmax
// e_j = fvsr_exp(s_j − max) with per-lane partial sums over j ≡ lane (mod 32) in increasing j, a xor-butterfly
// reduction, and p_j = e_j / sum. fvsr_exp is Cody–Waite range reduction (W. J. Cody, W. Waite, 1980) with a
// degree-7 Taylor polynomial — the same function, constant for constant, as the CPU restatement.
#include <math.h>

#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kTI = 64;   // query blocks per score tile
constexpr int kTJ = 64;   // key blocks per score tile
constexpr int kPS = 132;  // padded fp32 row stride of the staged pooled rows
constexpr int kSoftRows = 4;  // (head, query block) rows per softmax CTA, one per warp

__device__ __forceinline__ float pow2i(int n) { return __uint_as_float((uint32_t)(n + 127) << 23); }

// e^x: the softmax exponential of the selection (see the file comment for the method). Branch-free: the special
// cases are selected at the end, so a warp never diverges on it.
__device__ __forceinline__ float fvsr_exp(float x) {
    const float log2e = 1.44269502925872802734375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.428606765330187045e-06f;
    const float xc = fminf(fmaxf(x, -104.0f), 88.72f);  // keeps n in range; the out-of-range results are selected below
    const float n = rintf(__fmul_rn(xc, log2e));
    float r = __fmaf_rn(-n, ln2_hi, xc);
    r = __fmaf_rn(-n, ln2_lo, r);
    float p = 1.0f / 5040.0f;
    p = __fmaf_rn(p, r, 1.0f / 720.0f);
    p = __fmaf_rn(p, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n;
    // 2^n as one multiply for −126 ≤ n ≤ 127, else (p·2^(n+64))·2^−64 or (p·2^(n−1))·2 — the second factor is 1 in
    // the common case, which leaves the product unchanged
    const bool lo = ni < -126, hi = ni > 127;
    const int e1 = lo ? ni + 64 : (hi ? ni - 1 : ni);
    const float s2 = lo ? pow2i(-64) : (hi ? 2.0f : 1.0f);
    float y = __fmul_rn(__fmul_rn(p, pow2i(e1)), s2);
    y = x < -104.0f ? 0.0f : y;
    y = x > 88.72f ? INFINITY : y;
    return x != x ? x : y;
}

// Exact k-th largest by a 3-pass MSB-first radix select on the fp32 bit patterns (probabilities are ≥ 0, so the
// unsigned order of the bits is the float order): pass 1 bins bits [31:21] (2048 bins), pass 2 bits [20:10] (2048),
// pass 3 bits [9:0] (1024). Each pass only counts the entries whose higher bits equal the bins chosen so far.
constexpr int kBins1 = 2048, kBins2 = 2048, kBins3 = 1024;
// Per-row workspace words: the three histograms, then completion counters and the radix state after each pass.
// The last CTA of a pass (threadfence-and-count, no waiting) turns that pass's histogram into the next state.
constexpr int kOffCounter = kBins1 + kBins2 + kBins3;  // 3 counters (pass 1 counts per head, in the head's first row)
constexpr int kOffState = kOffCounter + 4;             // state after pass p at kOffState + 3·(p−1): prefix, mask, rank
constexpr int kHistPerRow = kOffState + 12;
constexpr int kHistPer = 16;                  // entries per thread per histogram CTA
constexpr int kHistChunk = 256 * kHistPer;    // entries of one selection row per histogram CTA
constexpr int kFinishRows = 8;                // query blocks compacted per finishing CTA

// Warp-aggregated shared-memory histogram increment (bins repeat heavily: probabilities share exponents).
__device__ __forceinline__ void hist_add(uint32_t* h, uint32_t key, bool valid) {
    const uint32_t k = valid ? key : 0xFFFFFFFFu;
    const uint32_t peers = __match_any_sync(0xffffffffu, k);
    const int lane = threadIdx.x & 31;
    if (valid && lane == __ffs(peers) - 1) atomicAdd(h + key, (uint32_t)__popc(peers));
}

// Finds, among `nbins` histogram bins scanned from the highest, the bin holding the entry of descending rank `rank`
// (0 = largest). All threads of the block call it (128 to 1024 threads, nbins / blockDim ≤ 16); the result is
// returned to every thread.
__device__ void block_find_bin(const uint32_t* __restrict__ hist, int nbins, uint32_t rank, uint32_t* out_bin,
                               uint32_t* out_rank) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t s_bin, s_rank;
    const int nt = blockDim.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = nbins / nt;
    const int top = nbins - 1 - per * tid;  // this thread covers bins top, top−1, …, top−per+1
    uint32_t c[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) c[i] = i < per ? __ldcg(hist + top - i) : 0u;
    uint32_t local = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) local += c[i];
    uint32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    if (tid == 0) {
        s_bin = 0;
        s_rank = 0;
    }
    __syncthreads();
    uint32_t before = 0;
    for (int w = 0; w < warp; ++w) before += warp_sums[w];
    const uint32_t excl = before + incl - local;
    if (rank >= excl && rank < excl + local) {
        uint32_t cum = excl;
        for (int i = 0; i < per; ++i) {
            if (rank < cum + c[i]) {
                s_bin = (uint32_t)(top - i);
                s_rank = rank - cum;
                break;
            }
            cum += c[i];
        }
    }
    __syncthreads();
    *out_bin = s_bin;
    *out_rank = s_rank;
    __syncthreads();
}

// Called by the last CTA of pass `pass` for row `hrow`: folds that pass's histogram into the radix state.
__device__ void advance_state(uint32_t* __restrict__ hrow, int pass, uint32_t rank0) {
    uint32_t prefix = 0, pmask = 0, rank = rank0;
    if (pass > 1) {
        const uint32_t* st = hrow + kOffState + 3 * (pass - 2);
        prefix = __ldcg(st);
        pmask = __ldcg(st + 1);
        rank = __ldcg(st + 2);
    }
    const int off = pass == 1 ? 0 : (pass == 2 ? kBins1 : kBins1 + kBins2);
    const int nb = pass == 3 ? kBins3 : kBins1;
    uint32_t b;
    block_find_bin(hrow + off, nb, rank, &b, &rank);
    if (pass == 1) {
        prefix = b << 21;
        pmask = 0xFFE00000u;
    } else if (pass == 2) {
        prefix |= b << 10;
        pmask |= 0x001FFC00u;
    } else {
        prefix |= b;
        pmask = 0xFFFFFFFFu;
    }
    if (threadIdx.x == 0) {
        uint32_t* st = hrow + kOffState + 3 * (pass - 1);
        st[0] = prefix;
        st[1] = pmask;
        st[2] = rank;
    }
}

// True in every thread of the CTA that completes `counter` (threadfence reduction: each CTA publishes its histogram
// atomics, fences, then counts itself; the CTA that sees total − 1 runs after all others' atomics are visible).
__device__ bool last_cta(uint32_t* counter, uint32_t total) {
    __shared__ uint32_t s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(counter, 1u) == total - 1 ? 1u : 0u;
    __syncthreads();
    const bool last = s_last != 0;
    if (last) __threadfence();
    return last;
}

__device__ __forceinline__ uint32_t row_rank0(int64_t n, int topk) {
    return (uint32_t)((int64_t)topk < n - 1 ? (int64_t)topk : n - 1);
}

// Score tile: kTI query blocks × kTJ key blocks of one head. Thread (ty, tx) computes the 4 × 4 micro-tile of rows
// 4·ty + a and keys tx + 16·u, each score a sequential fmaf chain over e = 0..127.
__global__ void __launch_bounds__(256) select_scores_kernel(const float* __restrict__ pq, const float* __restrict__ pk,
                                                            KvPages pages, int heads, int nq, int nk, int bh, int bw,
                                                            int local_range, float sqrt_d, float* __restrict__ scores) {
    griddep_wait_then_release();
    extern __shared__ float4 score_smem[];
    float* sq = reinterpret_cast<float*>(score_smem);  // [kTI][kPS]
    float* sk = sq + kTI * kPS;                         // [kTJ][kPS]
    const int h = blockIdx.z;
    const int i0 = blockIdx.y * kTI, j0 = blockIdx.x * kTJ;
    const int64_t ld = (int64_t)heads * kD;
    const int tid = threadIdx.x;
    {  // stage the tile's pooled rows: all 16 loads of a thread in flight before the first store
        constexpr int kPer = (kTI * 32) / 256;
        static_assert(kTI == kTJ && (kTI * 32) % 256 == 0, "staging layout");
        float4 vq[kPer], vk[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int idx = tid + 256 * k, r = idx >> 5, e4 = idx & 31;
            const int i = i0 + r, j = j0 + r;
            vq[k] = i < nq ? __ldg(reinterpret_cast<const float4*>(pq + i * ld + h * kD) + e4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
            vk[k] = j < nk ? __ldg(reinterpret_cast<const float4*>(pk + (int64_t)kv_phys_block(pages, j) * ld + h * kD) +
                                   e4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int idx = tid + 256 * k, r = idx >> 5, e4 = idx & 31;
            *reinterpret_cast<float4*>(sq + r * kPS + e4 * 4) = vq[k];
            *reinterpret_cast<float4*>(sk + r * kPS + e4 * 4) = vk[k];
        }
    }
    __syncthreads();
    // a warp covers tile rows [8·warp, 8·warp + 8): past the last query block it has nothing to write
    if (i0 + 8 * (tid >> 5) >= nq) return;
    const int ty = tid >> 4, tx = tid & 15;
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[a][u] = 0.0f;
#pragma unroll 2
    for (int e4 = 0; e4 < 32; ++e4) {
        float4 x[4], y[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) x[a] = reinterpret_cast<const float4*>(sq + (4 * ty + a) * kPS)[e4];
#pragma unroll
        for (int u = 0; u < 4; ++u) y[u] = reinterpret_cast<const float4*>(sk + (tx + 16 * u) * kPS)[e4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                acc[a][u] = __fmaf_rn(x[a].x, y[u].x, acc[a][u]);
                acc[a][u] = __fmaf_rn(x[a].y, y[u].y, acc[a][u]);
                acc[a][u] = __fmaf_rn(x[a].z, y[u].z, acc[a][u]);
                acc[a][u] = __fmaf_rn(x[a].w, y[u].w, acc[a][u]);
            }
    }
    // locality window of each of the 4 rows and grid position of each of the 4 keys, computed once
    const int s = bh * bw, half = local_range / 2;
    int lo_r[4], lo_c[4], kr[4], kc[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int qi = (i0 + 4 * ty + a) % s;
        lo_r[a] = qi / bw - half;
        lo_c[a] = qi % bw - half;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int kj = (j0 + tx + 16 * u) % s;
        kr[u] = kj / bw;
        kc[u] = kj % bw;
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int i = i0 + 4 * ty + a;
        if (i >= nq) continue;
        float* out = scores + ((int64_t)h * nq + i) * nk;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = j0 + tx + 16 * u;
            if (j >= nk) continue;
            const bool allowed = kr[u] >= lo_r[a] && kr[u] <= lo_r[a] + local_range - 1 && kc[u] >= lo_c[a] &&
                                 kc[u] <= lo_c[a] + local_range - 1;
            out[j] = allowed ? __fdiv_rn(acc[a][u], sqrt_d) : -INFINITY;
        }
    }
}

// Softmax over the key blocks of one (head, query block) row per warp, in place (scores → probs), plus the pass-1
// histogram of each (head, query slice) row. A CTA's rows lie in at most two slices whenever Nq/q_slices ≥ 8; rows
// of any further slice go straight to global atomics.
// NCH > 0: the row (at most NCH·256 key blocks) stays in registers between the three passes; NCH = 0 re-reads it.
template <int NCH>
__global__ void __launch_bounds__(kSoftRows * 32) select_softmax_kernel(float* __restrict__ probs, int nq, int nk,
                                                                       int q_slices, int topk,
                                                                       uint32_t* __restrict__ hist) {
    griddep_wait_then_release();
    __shared__ uint32_t shist[2][kBins1];
    const int h = blockIdx.y;
    const int i0 = blockIdx.x * kSoftRows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nqs = nq / q_slices;
    const int slice0 = i0 / nqs;
    for (int i = tid; i < 2 * kBins1; i += kSoftRows * 32) (&shist[0][0])[i] = 0;
    __syncthreads();
    const int i = i0 + warp;
    if (i < nq) {  // warp-uniform
        float* row = probs + ((int64_t)h * nq + i) * nk;
        constexpr int kR = NCH > 0 ? NCH * 8 : 1;
        float rv[kR];
        if (NCH > 0) {  // all loads in flight at once
#pragma unroll
            for (int c = 0; c < kR; ++c) {
                const int j = 256 * (c >> 3) + 32 * (c & 7) + lane;
                rv[c] = j < nk ? row[j] : -INFINITY;
            }
        }
        float m = -INFINITY;
        if (NCH > 0) {
#pragma unroll
            for (int c = 0; c < kR; ++c) m = fmaxf(m, rv[c]);
        } else {
            for (int jb = 0; jb < nk; jb += 256) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    v[u] = j < nk ? row[j] : -INFINITY;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) m = fmaxf(m, v[u]);
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float part = 0.0f;
        if (NCH > 0) {  // same order as below: j ≡ lane (mod 32), increasing j
#pragma unroll
            for (int c = 0; c < kR; ++c) {
                const int j = 256 * (c >> 3) + 32 * (c & 7) + lane;
                const float e = fvsr_exp(__fsub_rn(rv[c], m));
                rv[c] = j < nk ? e : 0.0f;
                if (j < nk) part = __fadd_rn(part, e);
            }
        } else {
            for (int jb = 0; jb < nk; jb += 256) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    v[u] = j < nk ? row[j] : -INFINITY;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    const float e = fvsr_exp(__fsub_rn(v[u], m));
                    if (j < nk) {
                        row[j] = e;
                        part = __fadd_rn(part, e);
                    }
                }
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
        const int sl = i / nqs, local = sl - slice0;
        uint32_t* gh = hist + (int64_t)(h * q_slices + sl) * kHistPerRow;
        auto emit = [&](int j, float v) {
            const float p = v == 0.0f ? 0.0f : __fdiv_rn(v, part);  // 0 / sum = +0 exactly
            if (j < nk) row[j] = p;
            const uint32_t bin = __float_as_uint(p) >> 21;
            if (local < 2)
                hist_add(&shist[local][0], bin, j < nk);
            else if (j < nk)
                atomicAdd(gh + bin, 1u);
        };
        if (NCH > 0) {
#pragma unroll
            for (int c = 0; c < kR; ++c) emit(256 * (c >> 3) + 32 * (c & 7) + lane, rv[c]);
        } else {
            for (int jb = 0; jb < nk; jb += 256) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    v[u] = j < nk ? row[j] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) emit(jb + 32 * u + lane, v[u]);
            }
        }
    }
    __syncthreads();
    for (int x = tid; x < 2 * kBins1; x += kSoftRows * 32) {
        const uint32_t c = (&shist[0][0])[x];
        const int sl = slice0 + x / kBins1;
        if (c && sl < q_slices) atomicAdd(hist + (int64_t)(h * q_slices + sl) * kHistPerRow + (x % kBins1), c);
    }
    uint32_t* head0 = hist + (int64_t)(h * q_slices) * kHistPerRow;
    if (last_cta(head0 + kOffCounter, gridDim.x))
        for (int t = 0; t < q_slices; ++t)
            advance_state(hist + (int64_t)(h * q_slices + t) * kHistPerRow, 1, row_rank0((int64_t)nqs * nk, topk));
}

// Passes 2 and 3 of the radix select: one CTA per kHistChunk entries of one (head, query slice) row.
__global__ void __launch_bounds__(256) select_hist_kernel(const float* __restrict__ probs, int nq, int nk, int q_slices,
                                                          int topk, uint32_t* __restrict__ hist, int pass) {
    griddep_wait_then_release();
    __shared__ uint32_t sh[kBins2];
    const int row = blockIdx.y;
    const int h = row / q_slices, t = row % q_slices;
    const int nqs = nq / q_slices;
    const int64_t n = (int64_t)nqs * nk;
    uint32_t* hrow = hist + (int64_t)row * kHistPerRow;
    const int tid = threadIdx.x;
    const float* base = probs + ((int64_t)h * nq + (int64_t)t * nqs) * nk;
    const int64_t e0 = (int64_t)blockIdx.x * kHistChunk;
    uint32_t u[kHistPer];
#pragma unroll
    for (int k = 0; k < kHistPer; ++k) {
        const int64_t idx = e0 + tid + 256 * k;
        u[k] = idx < n ? __float_as_uint(base[idx]) : 0xFFFFFFFFu;
    }
    for (int i = tid; i < kBins2; i += 256) sh[i] = 0;
    const uint32_t* st = hrow + kOffState + 3 * (pass - 2);
    const uint32_t prefix = __ldcg(st), pmask = __ldcg(st + 1);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kHistPer; ++k) {
        const int64_t idx = e0 + tid + 256 * k;
        const bool valid = idx < n && (u[k] & pmask) == prefix;
        const uint32_t bin = pass == 2 ? (u[k] >> 10) & (kBins2 - 1) : u[k] & (kBins3 - 1);
        hist_add(sh, bin, valid);
    }
    __syncthreads();
    uint32_t* gh = hrow + (pass == 2 ? kBins1 : kBins1 + kBins2);
    const int nb = pass == 2 ? kBins2 : kBins3;
    for (int i = tid; i < nb; i += 256)
        if (sh[i]) atomicAdd(gh + i, sh[i]);
    if (last_cta(hrow + kOffCounter + pass - 1, gridDim.x)) advance_state(hrow, pass, row_rank0(n, topk));
}

// Threshold = the exact (min(n−1, topk)+1)-th largest of the row; compaction of p > threshold into ascending kidx
// lists (the rest −1), kcnt, and the optional 0/1 mask. One CTA per kFinishRows query blocks of one row.
__global__ void __launch_bounds__(256) select_finish_kernel(const float* __restrict__ probs, int nq, int nk,
                                                            int q_slices, int topk, const uint32_t* __restrict__ hist,
                                                            int32_t* __restrict__ kidx, int32_t* __restrict__ kcnt,
                                                            uint8_t* __restrict__ mask) {
    griddep_wait_then_release();
    const int row = blockIdx.y;
    const int h = row / q_slices, t = row % q_slices;
    const int nqs = nq / q_slices;
    const float thr = __uint_as_float(__ldcg(hist + (int64_t)row * kHistPerRow + kOffState + 6));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ii = blockIdx.x * kFinishRows + warp;
    if (ii >= nqs) return;
    const int64_t qrow = (int64_t)h * nq + (int64_t)t * nqs + ii;
    const float* p = probs + qrow * nk;
    int32_t* lst = kidx + qrow * nk;
    int cnt = 0;
    for (int jb = 0; jb < nk; jb += 256) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = jb + 32 * u + lane;
            v[u] = j < nk ? p[j] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = jb + 32 * u + lane;
            const bool keep = j < nk && v[u] > thr;
            const uint32_t bal = __ballot_sync(0xffffffffu, keep);
            if (keep) lst[cnt + __popc(bal & ((1u << lane) - 1u))] = j;
            if (mask && j < nk) mask[qrow * nk + j] = keep ? 1 : 0;
            cnt += __popc(bal);
        }
    }
    for (int j = cnt + lane; j < nk; j += 32) lst[j] = -1;
    if (lane == 0) kcnt[qrow] = cnt;
}

__global__ void __launch_bounds__(256) mask_to_lists_kernel(const float* __restrict__ mask, int rows, int nk,
                                                            int32_t* __restrict__ kidx, int32_t* __restrict__ kcnt) {
    griddep_wait_then_release();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* m = mask + (int64_t)warp * nk;
    int32_t* lst = kidx + (int64_t)warp * nk;
    int cnt = 0;
    for (int j0 = 0; j0 < nk; j0 += 32) {
        const int j = j0 + lane;
        const bool keep = j < nk && m[j] > 0.5f;
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (keep) lst[cnt + __popc(bal & ((1u << lane) - 1u))] = j;
        cnt += __popc(bal);
    }
    for (int j = cnt + lane; j < nk; j += 32) lst[j] = -1;
    if (lane == 0) kcnt[warp] = cnt;
}

}  // namespace

size_t select_scores_smem_bytes(int) { return sizeof(float) * (size_t)(kTI + kTJ) * kPS; }

size_t select_hist_bytes(int heads, int q_slices) { return sizeof(uint32_t) * (size_t)heads * q_slices * kHistPerRow; }

cudaError_t launch_select_scores(const float* pq, const float* pk, const KvPages& pk_pages, int heads, int nq, int nk,
                                 int bh, int bw, int local_range, int q_slices, int topk, float* probs, uint32_t* hist,
                                 cudaStream_t st, bool clear_hist) {
    cudaError_t e = cudaSuccess;
    if (clear_hist && (e = cudaMemsetAsync(hist, 0, select_hist_bytes(heads, q_slices), st)) != cudaSuccess) return e;
    const int smem = (int)select_scores_smem_bytes(nk);
    e = cudaFuncSetAttribute(select_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const float sqrt_d = sqrtf((float)kD);
    dim3 grid((nk + kTJ - 1) / kTJ, (nq + kTI - 1) / kTI, heads);
    e = launch_pdl(select_scores_kernel, grid, dim3(256), (size_t)smem, st, pq, pk, pk_pages, heads, nq, nk, bh, bw,
                   local_range, sqrt_d, probs);
    if (e != cudaSuccess) return e;
    dim3 sgrid((nq + kSoftRows - 1) / kSoftRows, heads);
    auto soft = [&](auto kernel) {
        return launch_pdl(kernel, sgrid, dim3(kSoftRows * 32), 0, st, probs, nq, nk, q_slices, topk, hist);
    };
    if (nk <= 256) return soft(select_softmax_kernel<1>);
    if (nk <= 512) return soft(select_softmax_kernel<2>);
    if (nk <= 768) return soft(select_softmax_kernel<3>);
    if (nk <= 1024) return soft(select_softmax_kernel<4>);
    return soft(select_softmax_kernel<0>);
}

cudaError_t launch_select_threshold(const float* probs, int heads, int nq, int nk, int q_slices, int topk,
                                    uint32_t* hist, int32_t* kidx, int32_t* kcnt, uint8_t* mask, cudaStream_t st) {
    const int rows = heads * q_slices;
    const int64_t n = (int64_t)(nq / q_slices) * nk;
    dim3 hgrid((unsigned)((n + kHistChunk - 1) / kHistChunk), rows);
    for (int pass = 2; pass <= 3; ++pass) {
        const cudaError_t e =
            launch_pdl(select_hist_kernel, hgrid, dim3(256), 0, st, probs, nq, nk, q_slices, topk, hist, pass);
        if (e != cudaSuccess) return e;
    }
    dim3 fgrid((nq / q_slices + kFinishRows - 1) / kFinishRows, rows);
    return launch_pdl(select_finish_kernel, fgrid, dim3(256), 0, st, probs, nq, nk, q_slices, topk, hist, kidx, kcnt,
                      mask);
}

cudaError_t launch_mask_to_lists(const float* mask, int heads, int nq, int nk, int32_t* kidx, int32_t* kcnt,
                                 cudaStream_t st) {
    const int rows = heads * nq;
    return launch_pdl(mask_to_lists_kernel, dim3((rows * 32 + 255) / 256), dim3(256), 0, st, mask, rows, nk, kidx,
                      kcnt);
}

}  // namespace fvsr

namespace fvsr {

namespace {

// One CTA per head segment of the range. The order is: the non-empty items of each head segment in turn (segments in
// head order), longest key list first within a segment (ties by id); then every empty item of the range, ascending.
// Empty items only write zeros, so they go last: placed between heads they would delay the next head's long items.
// Rank of a non-empty item inside its segment = items of the segment with a longer key list, or an equal one and a
// smaller id; empty items rank after all non-empty ones, by id.
__global__ void __launch_bounds__(256) item_order_kernel(const int32_t* __restrict__ kcnt, int nq, int item_begin,
                                                         int item_count, int32_t* __restrict__ order) {
    griddep_wait_then_release();
    __shared__ int32_t sc[4096];
    __shared__ int cnt[4];  // non-empty before this segment, empty before it, non-empty in the range, in the segment
    const int h = item_begin / nq + blockIdx.x;
    const int s0 = max(item_begin, h * nq), s1 = min(item_begin + item_count, (h + 1) * nq);
    const int n = s1 - s0;
    if (n <= 0) return;
    if (threadIdx.x < 4) cnt[threadIdx.x] = 0;
    __syncthreads();
    {
        int a = 0, b = 0, c = 0, d = 0;
        for (int i = threadIdx.x; i < item_count; i += blockDim.x) {
            const int it = item_begin + i;
            const bool nz = kcnt[it] > 0;
            c += nz;
            if (it < s0) {
                a += nz;
                b += !nz;
            } else if (it < s1) {
                d += nz;
            }
        }
        atomicAdd(&cnt[0], a);
        atomicAdd(&cnt[1], b);
        atomicAdd(&cnt[2], c);
        atomicAdd(&cnt[3], d);
    }
    __syncthreads();
    const int ne_before = cnt[0], e_before = cnt[1], ne_total = cnt[2], ne_seg = cnt[3];
    auto place = [&](int i, int rank, bool nz) {  // rank: position inside the segment, non-empty items first
        const int pos = nz ? ne_before + rank : ne_total + e_before + (rank - ne_seg);
        order[pos] = s0 + i;
    };
    if (n > 4096) {  // no room to rank: each class in ascending id order
        if (threadIdx.x == 0) {
            int a = 0, b = 0;
            for (int i = 0; i < n; ++i) {
                const bool nz = kcnt[s0 + i] > 0;
                place(i, nz ? a++ : ne_seg + b++, nz);
            }
        }
        return;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) sc[i] = max(kcnt[s0 + i], 0);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ci = sc[i];
        int rank = 0;
        for (int t = 0; t < n; ++t) {
            const int ct = sc[t];
            rank += (ct > ci) || (ct == ci && t < i);
        }
        place(i, rank, ci > 0);
    }
}

}  // namespace

cudaError_t launch_item_order(const int32_t* kcnt, int nq, int item_begin, int item_count, int32_t* order,
                              cudaStream_t st) {
    if (item_count <= 0) return cudaSuccess;
    const int h0 = item_begin / nq, h1 = (item_begin + item_count - 1) / nq;
    return launch_pdl(item_order_kernel, dim3(h1 - h0 + 1), dim3(256), 0, st, kcnt, nq, item_begin, item_count, order);
}

}  // namespace fvsr
