// select.cu — LCSA block selection (draftBlockMaskAndProbs, DiT.swift:158-174) on pooled fp32 Q/K.
//
// Kernels (in launch order):
//   select_scores_kernel    per (head, 8 query blocks): block scores pq·pk / sqrt(d) (fixed-order fmaf dot), the
//                           spatial locality mask (DiT.swift:130-145, computed from (bh, bw, R) instead of a table),
//                           the softmax over key blocks → probs (H, Nq, Nk), and pass 1 of the radix select.
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

constexpr int kQR = 8;    // query blocks per CTA (one per warp)
constexpr int kKT = 64;   // key blocks per staged tile
constexpr int kKS = 132;  // padded fp32 row stride of the staged key tile (conflict-free float4 reads)

__device__ __forceinline__ float pow2i(int n) { return __uint_as_float((uint32_t)(n + 127) << 23); }

// e^x: the softmax exponential of the selection (see the file comment for the method).
__device__ __forceinline__ float fvsr_exp(float x) {
    if (x != x) return x;
    if (x < -104.0f) return 0.0f;
    if (x > 88.72f) return INFINITY;
    const float log2e = 1.44269502925872802734375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.428606765330187045e-06f;
    const float n = rintf(__fmul_rn(x, log2e));
    float r = __fmaf_rn(-n, ln2_hi, x);
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
    if (ni >= -126) {
        if (ni > 127) return INFINITY;
        return __fmul_rn(p, pow2i(ni));
    }
    return __fmul_rn(__fmul_rn(p, pow2i(ni + 64)), pow2i(-64));
}

// Exact k-th largest by a 3-pass MSB-first radix select on the fp32 bit patterns (probabilities are ≥ 0, so the
// unsigned order of the bits is the float order): pass 1 bins bits [31:21] (2048 bins), pass 2 bits [20:10] (2048),
// pass 3 bits [9:0] (1024). Each pass only counts the entries whose higher bits equal the bins chosen so far.
constexpr int kBins1 = 2048, kBins2 = 2048, kBins3 = 1024;
constexpr int kHistPerRow = kBins1 + kBins2 + kBins3;
constexpr int kHistChunk = 8192;  // entries of one selection row per histogram CTA
constexpr int kFinishRows = 8;    // query blocks compacted per finishing CTA

// Warp-aggregated shared-memory histogram increment (bins repeat heavily: probabilities share exponents).
__device__ __forceinline__ void hist_add(uint32_t* h, uint32_t key, bool valid) {
    const uint32_t k = valid ? key : 0xFFFFFFFFu;
    const uint32_t peers = __match_any_sync(0xffffffffu, k);
    const int lane = threadIdx.x & 31;
    if (valid && lane == __ffs(peers) - 1) atomicAdd(h + key, (uint32_t)__popc(peers));
}

// Finds, among `nbins` histogram bins scanned from the highest, the bin holding the entry of descending rank `rank`
// (0 = largest). All 256 threads of the block call it; the result is returned to every thread.
__device__ void block_find_bin(const uint32_t* __restrict__ hist, int nbins, uint32_t rank, uint32_t* out_bin,
                               uint32_t* out_rank) {
    __shared__ uint32_t warp_sums[8];
    __shared__ uint32_t s_bin, s_rank;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = nbins / 256;
    const int top = nbins - 1 - per * tid;  // this thread covers bins top, top−1, …, top−per+1
    uint32_t local = 0;
    for (int i = 0; i < per; ++i) local += hist[top - i];
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
            const uint32_t c = hist[top - i];
            if (rank < cum + c) {
                s_bin = (uint32_t)(top - i);
                s_rank = rank - cum;
                break;
            }
            cum += c;
        }
    }
    __syncthreads();
    *out_bin = s_bin;
    *out_rank = s_rank;
    __syncthreads();
}

// Row state after `passes` completed passes: the fixed high bits (prefix under pmask) and the remaining rank.
__device__ void row_state(const uint32_t* __restrict__ hrow, int passes, uint32_t rank0, uint32_t* prefix,
                          uint32_t* pmask, uint32_t* rank) {
    uint32_t b, r = rank0, pre = 0, msk = 0;
    if (passes >= 1) {
        block_find_bin(hrow, kBins1, r, &b, &r);
        pre = b << 21;
        msk = 0xFFE00000u;
    }
    if (passes >= 2) {
        block_find_bin(hrow + kBins1, kBins2, r, &b, &r);
        pre |= b << 10;
        msk |= 0x001FFC00u;
    }
    if (passes >= 3) {
        block_find_bin(hrow + kBins1 + kBins2, kBins3, r, &b, &r);
        pre |= b;
        msk = 0xFFFFFFFFu;
    }
    *prefix = pre;
    *pmask = msk;
    *rank = r;
}

__global__ void __launch_bounds__(256) select_scores_kernel(const float* __restrict__ pq, const float* __restrict__ pk,
                                                            KvPages pages, int heads, int nq, int nk, int bh, int bw,
                                                            int local_range, int q_slices, float sqrt_d,
                                                            float* __restrict__ probs, uint32_t* __restrict__ hist) {
    extern __shared__ float4 sm4[];
    uint32_t* shist = reinterpret_cast<uint32_t*>(sm4);  // [2][kBins1] pass-1 histograms of the CTA's first 2 slices
    float* sq = reinterpret_cast<float*>(shist + 2 * kBins1);  // [kQR][128]
    float* sk = sq + kQR * kD;                                  // [kKT][kKS]
    float* ss = sk + kKT * kKS;                                 // [kQR][nk]
    const int h = blockIdx.y;
    const int i0 = blockIdx.x * kQR;
    const int64_t ld = (int64_t)heads * kD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = bh * bw, half = local_range / 2;
    const int nqs = nq / q_slices;
    const int slice0 = i0 / nqs;

    for (int i = tid; i < 2 * kBins1; i += 256) shist[i] = 0;
    for (int idx = tid; idx < kQR * 32; idx += 256) {
        const int r = idx >> 5, e4 = idx & 31;
        const int i = i0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < nq) v = __ldg(reinterpret_cast<const float4*>(pq + i * ld + h * kD) + e4);
        reinterpret_cast<float4*>(sq)[idx] = v;
    }
    const int r0 = warp;  // one query block per warp
    const int i_0 = i0 + r0;
    const int qi = i_0 % s, qr_ = qi / bw, qc_ = qi % bw;

    for (int jt = 0; jt < nk; jt += kKT) {
        __syncthreads();
        for (int idx = tid; idx < kKT * 32; idx += 256) {
            const int kr = idx >> 5, e4 = idx & 31;
            const int j = jt + kr;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (j < nk) v = __ldg(reinterpret_cast<const float4*>(pk + (int64_t)kv_phys_block(pages, j) * ld + h * kD) + e4);
            *reinterpret_cast<float4*>(sk + kr * kKS + e4 * 4) = v;
        }
        __syncthreads();
        if (i_0 >= nq) continue;
        const float4* q0 = reinterpret_cast<const float4*>(sq + r0 * kD);
        const float4* k0 = reinterpret_cast<const float4*>(sk + lane * kKS);
        const float4* k1 = reinterpret_cast<const float4*>(sk + (lane + 32) * kKS);
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 8
        for (int e4 = 0; e4 < 32; ++e4) {
            const float4 x = q0[e4], y0 = k0[e4], y1 = k1[e4];
            a0 = __fmaf_rn(x.x, y0.x, a0);
            a0 = __fmaf_rn(x.y, y0.y, a0);
            a0 = __fmaf_rn(x.z, y0.z, a0);
            a0 = __fmaf_rn(x.w, y0.w, a0);
            a1 = __fmaf_rn(x.x, y1.x, a1);
            a1 = __fmaf_rn(x.y, y1.y, a1);
            a1 = __fmaf_rn(x.z, y1.z, a1);
            a1 = __fmaf_rn(x.w, y1.w, a1);
        }
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int j = jt + lane + 32 * cc;
            if (j >= nk) continue;
            const int kj = j % s, kr_ = kj / bw, kc_ = kj % bw;
            const bool allowed = kr_ >= qr_ - half && kr_ <= qr_ - half + local_range - 1 && kc_ >= qc_ - half &&
                                 kc_ <= qc_ - half + local_range - 1;
            ss[r0 * nk + j] = allowed ? __fdiv_rn(cc ? a1 : a0, sqrt_d) : -INFINITY;
        }
    }
    __syncthreads();
    if (i_0 < nq) {  // warp-uniform
        float* row = ss + r0 * nk;
        float m = -INFINITY;
        for (int j = lane; j < nk; j += 32) m = fmaxf(m, row[j]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float part = 0.0f;
        for (int j = lane; j < nk; j += 32) {
            const float e = fvsr_exp(__fsub_rn(row[j], m));
            row[j] = e;
            part = __fadd_rn(part, e);
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
        float* out = probs + ((int64_t)h * nq + i_0) * nk;
        const int sl = i_0 / nqs, local = sl - slice0;
        uint32_t* gh = hist + (int64_t)(h * q_slices + sl) * kHistPerRow;
        for (int j0 = 0; j0 < nk; j0 += 32) {
            const int j = j0 + lane;
            float p = 0.0f;
            if (j < nk) {
                p = __fdiv_rn(row[j], part);
                out[j] = p;
            }
            const uint32_t bin = __float_as_uint(p) >> 21;
            if (local < 2)
                hist_add(shist + local * kBins1, bin, j < nk);
            else if (j < nk)
                atomicAdd(gh + bin, 1u);
        }
    }
    __syncthreads();
    for (int i = tid; i < 2 * kBins1; i += 256) {
        const uint32_t c = shist[i];
        const int sl = slice0 + i / kBins1;
        if (c && sl < q_slices) atomicAdd(hist + (int64_t)(h * q_slices + sl) * kHistPerRow + (i % kBins1), c);
    }
}

// Passes 2 and 3 of the radix select: one CTA per kHistChunk entries of one (head, query slice) row.
__global__ void __launch_bounds__(256) select_hist_kernel(const float* __restrict__ probs, int nq, int nk, int q_slices,
                                                          int topk, uint32_t* __restrict__ hist, int pass) {
    __shared__ uint32_t sh[kBins2];
    const int row = blockIdx.y;
    const int h = row / q_slices, t = row % q_slices;
    const int nqs = nq / q_slices;
    const int64_t n = (int64_t)nqs * nk;
    const uint32_t rank0 = (uint32_t)((int64_t)topk < n - 1 ? (int64_t)topk : n - 1);
    uint32_t* hrow = hist + (int64_t)row * kHistPerRow;
    const int tid = threadIdx.x;
    for (int i = tid; i < kBins2; i += 256) sh[i] = 0;
    uint32_t prefix, pmask, rank;
    row_state(hrow, pass - 1, rank0, &prefix, &pmask, &rank);  // also synchronises the block
    const float* base = probs + ((int64_t)h * nq + (int64_t)t * nqs) * nk;
    const int64_t e0 = (int64_t)blockIdx.x * kHistChunk;
    const int64_t e1 = e0 + kHistChunk < n ? e0 + kHistChunk : n;
    for (int64_t b = e0 + (tid & ~31); b < e1; b += 256) {
        const int64_t idx = b + (tid & 31);
        uint32_t u = 0;
        bool valid = idx < e1;
        if (valid) {
            u = __float_as_uint(base[idx]);
            valid = (u & pmask) == prefix;
        }
        const uint32_t bin = pass == 2 ? (u >> 10) & (kBins2 - 1) : u & (kBins3 - 1);
        hist_add(sh, bin, valid);
    }
    __syncthreads();
    uint32_t* gh = hrow + (pass == 2 ? kBins1 : kBins1 + kBins2);
    const int nb = pass == 2 ? kBins2 : kBins3;
    for (int i = tid; i < nb; i += 256)
        if (sh[i]) atomicAdd(gh + i, sh[i]);
}

// Threshold = the exact (min(n−1, topk)+1)-th largest of the row; compaction of p > threshold into ascending kidx
// lists (the rest −1), kcnt, and the optional 0/1 mask. One CTA per kFinishRows query blocks of one row.
__global__ void __launch_bounds__(256) select_finish_kernel(const float* __restrict__ probs, int nq, int nk,
                                                            int q_slices, int topk, const uint32_t* __restrict__ hist,
                                                            int32_t* __restrict__ kidx, int32_t* __restrict__ kcnt,
                                                            uint8_t* __restrict__ mask) {
    const int row = blockIdx.y;
    const int h = row / q_slices, t = row % q_slices;
    const int nqs = nq / q_slices;
    const int64_t n = (int64_t)nqs * nk;
    const uint32_t rank0 = (uint32_t)((int64_t)topk < n - 1 ? (int64_t)topk : n - 1);
    uint32_t prefix, pmask, rank;
    row_state(hist + (int64_t)row * kHistPerRow, 3, rank0, &prefix, &pmask, &rank);
    const float thr = __uint_as_float(prefix);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ii = blockIdx.x * kFinishRows + warp;
    if (ii >= nqs) return;
    const int64_t qrow = (int64_t)h * nq + (int64_t)t * nqs + ii;
    const float* p = probs + qrow * nk;
    int32_t* lst = kidx + qrow * nk;
    int cnt = 0;
    for (int j0 = 0; j0 < nk; j0 += 32) {
        const int j = j0 + lane;
        const bool keep = j < nk && p[j] > thr;
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (keep) lst[cnt + __popc(bal & ((1u << lane) - 1u))] = j;
        if (mask && j < nk) mask[qrow * nk + j] = keep ? 1 : 0;
        cnt += __popc(bal);
    }
    for (int j = cnt + lane; j < nk; j += 32) lst[j] = -1;
    if (lane == 0) kcnt[qrow] = cnt;
}

__global__ void __launch_bounds__(256) mask_to_lists_kernel(const float* __restrict__ mask, int rows, int nk,
                                                            int32_t* __restrict__ kidx, int32_t* __restrict__ kcnt) {
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

size_t select_scores_smem_bytes(int nk) {
    return sizeof(uint32_t) * 2 * kBins1 + sizeof(float) * ((size_t)kQR * kD + (size_t)kKT * kKS + (size_t)kQR * nk);
}

size_t select_hist_bytes(int heads, int q_slices) { return sizeof(uint32_t) * (size_t)heads * q_slices * kHistPerRow; }

cudaError_t launch_select_scores(const float* pq, const float* pk, const KvPages& pk_pages, int heads, int nq, int nk,
                                 int bh, int bw, int local_range, int q_slices, float* probs, uint32_t* hist,
                                 cudaStream_t st) {
    const size_t smem = select_scores_smem_bytes(nk);
    cudaError_t e = cudaFuncSetAttribute(select_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(hist, 0, select_hist_bytes(heads, q_slices), st);
    if (e != cudaSuccess) return e;
    const float sqrt_d = sqrtf((float)kD);
    dim3 grid((nq + kQR - 1) / kQR, heads);
    select_scores_kernel<<<grid, 256, smem, st>>>(pq, pk, pk_pages, heads, nq, nk, bh, bw, local_range, q_slices, sqrt_d,
                                                  probs, hist);
    return cudaGetLastError();
}

cudaError_t launch_select_threshold(const float* probs, int heads, int nq, int nk, int q_slices, int topk,
                                    uint32_t* hist, int32_t* kidx, int32_t* kcnt, uint8_t* mask, cudaStream_t st) {
    const int rows = heads * q_slices;
    const int64_t n = (int64_t)(nq / q_slices) * nk;
    dim3 hgrid((unsigned)((n + kHistChunk - 1) / kHistChunk), rows);
    for (int pass = 2; pass <= 3; ++pass) {
        select_hist_kernel<<<hgrid, 256, 0, st>>>(probs, nq, nk, q_slices, topk, hist, pass);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    dim3 fgrid((nq / q_slices + kFinishRows - 1) / kFinishRows, rows);
    select_finish_kernel<<<fgrid, 256, 0, st>>>(probs, nq, nk, q_slices, topk, hist, kidx, kcnt, mask);
    return cudaGetLastError();
}

cudaError_t launch_mask_to_lists(const float* mask, int heads, int nq, int nk, int32_t* kidx, int32_t* kcnt,
                                 cudaStream_t st) {
    const int rows = heads * nq;
    mask_to_lists_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(mask, rows, nk, kidx, kcnt);
    return cudaGetLastError();
}

}  // namespace fvsr
