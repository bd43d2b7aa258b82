// select.cu — LCSA block selection (draftBlockMaskAndProbs, DiT.swift:158-174) on pooled fp32 Q/K.
//
// Two kernels:
//   select_scores_kernel    per (head, 16 query blocks): block scores pq·pk / sqrt(d) (fixed-order fmaf dot), the
//                           spatial locality mask (DiT.swift:130-145, computed from (bh, bw, R) instead of a table),
//                           and the softmax over key blocks, written to probs (H, Nq, Nk).
//   select_threshold_kernel per (head, query slice) row of n = (Nq/q_slices)·Nk probabilities: the exact
//                           (min(n−1, topk)+1)-th largest by an MSB-first 4×8-bit radix select on the fp32 bit patterns
//                           (probabilities are ≥ 0, so unsigned order = float order) — no sort — then compaction of
//                           p > threshold into ascending kidx lists, kcnt counts and the optional 0/1 mask.
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

constexpr int kQR = 16;   // query blocks per CTA (two per warp)
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

__global__ void __launch_bounds__(256) select_scores_kernel(const float* __restrict__ pq, const float* __restrict__ pk,
                                                            KvPages pages, int heads, int nq, int nk, int bh, int bw,
                                                            int local_range, float sqrt_d, float* __restrict__ probs) {
    extern __shared__ float4 sm4[];
    float* sq = reinterpret_cast<float*>(sm4);  // [kQR][128]
    float* sk = sq + kQR * kD;                   // [kKT][kKS]
    float* ss = sk + kKT * kKS;                  // [kQR][nk]
    const int h = blockIdx.y;
    const int i0 = blockIdx.x * kQR;
    const int64_t ld = (int64_t)heads * kD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = bh * bw, half = local_range / 2;

    for (int idx = tid; idx < kQR * 32; idx += 256) {
        const int r = idx >> 5, e4 = idx & 31;
        const int i = i0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < nq) v = __ldg(reinterpret_cast<const float4*>(pq + i * ld + h * kD) + e4);
        reinterpret_cast<float4*>(sq)[idx] = v;
    }
    const int r0 = 2 * warp, r1 = 2 * warp + 1;
    const int i_0 = i0 + r0, i_1 = i0 + r1;

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
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int c = lane + 32 * cc;
            const int j = jt + c;
            float a0 = 0.0f, a1 = 0.0f;
            const float4* q0 = reinterpret_cast<const float4*>(sq + r0 * kD);
            const float4* q1 = reinterpret_cast<const float4*>(sq + r1 * kD);
            const float4* kv = reinterpret_cast<const float4*>(sk + c * kKS);
#pragma unroll 8
            for (int e4 = 0; e4 < 32; ++e4) {
                const float4 x0 = q0[e4], x1 = q1[e4], y = kv[e4];
                a0 = __fmaf_rn(x0.x, y.x, a0);
                a0 = __fmaf_rn(x0.y, y.y, a0);
                a0 = __fmaf_rn(x0.z, y.z, a0);
                a0 = __fmaf_rn(x0.w, y.w, a0);
                a1 = __fmaf_rn(x1.x, y.x, a1);
                a1 = __fmaf_rn(x1.y, y.y, a1);
                a1 = __fmaf_rn(x1.z, y.z, a1);
                a1 = __fmaf_rn(x1.w, y.w, a1);
            }
            if (j < nk) {
                const int kj = j % s, kr_ = kj / bw, kc_ = kj % bw;
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int i = rr ? i_1 : i_0;
                    if (i >= nq) continue;
                    const int qi = i % s, qr_ = qi / bw, qc_ = qi % bw;
                    const bool allowed = kr_ >= qr_ - half && kr_ <= qr_ - half + local_range - 1 &&
                                         kc_ >= qc_ - half && kc_ <= qc_ - half + local_range - 1;
                    ss[(rr ? r1 : r0) * nk + j] = allowed ? __fdiv_rn(rr ? a1 : a0, sqrt_d) : -INFINITY;
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int r = rr ? r1 : r0;
        const int i = i0 + r;
        if (i >= nq) continue;  // warp-uniform
        float* row = ss + r * nk;
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
        float* out = probs + ((int64_t)h * nq + i) * nk;
        for (int j = lane; j < nk; j += 32) out[j] = __fdiv_rn(row[j], part);
    }
}

__global__ void __launch_bounds__(1024) select_threshold_kernel(const float* __restrict__ probs, int nq, int nk,
                                                                int q_slices, int topk, int32_t* __restrict__ kidx,
                                                                int32_t* __restrict__ kcnt, uint8_t* __restrict__ mask) {
    __shared__ uint32_t hist[32][256];
    __shared__ uint32_t total[256];
    __shared__ uint32_t s_prefix, s_pmask, s_rank;
    const int row = blockIdx.x;
    const int h = row / q_slices, t = row % q_slices;
    const int nqs = nq / q_slices;
    const int64_t n = (int64_t)nqs * nk;
    const float* base = probs + ((int64_t)h * nq + (int64_t)t * nqs) * nk;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t kk = (int64_t)topk < n - 1 ? (int64_t)topk : n - 1;
    if (tid == 0) {
        s_prefix = 0;
        s_pmask = 0;
        s_rank = (uint32_t)kk;
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 32 * 256; i += 1024) (&hist[0][0])[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, pmask = s_pmask;
        for (int64_t b0 = (int64_t)warp * 32; b0 < n; b0 += 1024) {
            const int64_t idx = b0 + lane;
            uint32_t key = 0xFFFFFFFFu;
            if (idx < n) {
                const uint32_t u = __float_as_uint(base[idx]);
                if ((u & pmask) == prefix) key = (u >> shift) & 0xFFu;
            }
            const uint32_t peers = __match_any_sync(0xffffffffu, key);
            if (key != 0xFFFFFFFFu && lane == __ffs(peers) - 1) atomicAdd(&hist[warp][key], (uint32_t)__popc(peers));
        }
        __syncthreads();
        if (tid < 256) {
            uint32_t s = 0;
#pragma unroll 8
            for (int w = 0; w < 32; ++w) s += hist[w][tid];
            total[tid] = s;
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t rank = s_rank, cum = 0;
            int chosen = 0;
            for (int bin = 255; bin >= 0; --bin) {
                if (rank < cum + total[bin]) {
                    chosen = bin;
                    break;
                }
                cum += total[bin];
            }
            s_rank = rank - cum;
            s_prefix = prefix | ((uint32_t)chosen << shift);
            s_pmask = pmask | (0xFFu << shift);
        }
        __syncthreads();
    }
    const float thr = __uint_as_float(s_prefix);
    for (int ii = warp; ii < nqs; ii += 32) {
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

size_t select_scores_smem_bytes(int nk) { return sizeof(float) * ((size_t)kQR * kD + (size_t)kKT * kKS + (size_t)kQR * nk); }

cudaError_t launch_select_scores(const float* pq, const float* pk, const KvPages& pk_pages, int heads, int nq, int nk,
                                 int bh, int bw, int local_range, float* probs, cudaStream_t st) {
    const size_t smem = select_scores_smem_bytes(nk);
    cudaError_t e = cudaFuncSetAttribute(select_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const float sqrt_d = sqrtf((float)kD);
    dim3 grid((nq + kQR - 1) / kQR, heads);
    select_scores_kernel<<<grid, 256, smem, st>>>(pq, pk, pk_pages, heads, nq, nk, bh, bw, local_range, sqrt_d, probs);
    return cudaGetLastError();
}

cudaError_t launch_select_threshold(const float* probs, int heads, int nq, int nk, int q_slices, int topk,
                                    int32_t* kidx, int32_t* kcnt, uint8_t* mask, cudaStream_t st) {
    select_threshold_kernel<<<heads * q_slices, 1024, 0, st>>>(probs, nq, nk, q_slices, topk, kidx, kcnt, mask);
    return cudaGetLastError();
}

cudaError_t launch_mask_to_lists(const float* mask, int heads, int nq, int nk, int32_t* kidx, int32_t* kcnt,
                                 cudaStream_t st) {
    const int rows = heads * nq;
    mask_to_lists_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(mask, rows, nk, kidx, kcnt);
    return cudaGetLastError();
}

}  // namespace fvsr
