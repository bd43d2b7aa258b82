// attn_f32.cu — fp32 block-sparse attention on the CUDA cores (the fp32 lane of kernelBlockAttention,
// SparseAttention.swift:169-187; DiT.swift:279-313 semantics).
//
// fp32 inputs must meet 1e-5 relative error against an fp32 reference, which tf32 tensor-core arithmetic cannot, so
// this lane runs plain fp32 FFMA. Four CTAs per (head, query block) item, each owning 32 of its 128 query rows, so a
// small problem (config 1: 96 items) still fills every SM (384 CTAs, four resident per SM). A CTA of 128 threads walks
// the item's kept key blocks in 16-key sub-tiles, K and V double-buffered in shared memory by cp.async (the next
// sub-tile is in flight while the current one is multiplied):
//   S  (32 rows × 16 keys): thread = (row pair, key pair) — rows 2·(t/8) + {0,1}, keys t%8 + {0, 8} — 2 × 2 scores
//       from float4 loads of Q and K rows (conflict-free: the 132-float row stride puts the warp's distinct rows on
//       distinct bank quads); row maximum and sum over the eight lanes of a row pair by shuffles; online softmax in
//       fp32 with accurate expf; P written transposed to shared memory with the row's rescale factor.
//   PV (32 rows × 128 dims): thread = (row quad, dim group) — rows 4·(t/16) + {0..3}, dims 4·(t%16) + {0..3} and
//       64 + 4·(t%16) + {0..3}: 32 fp32 accumulators, per key one float4 of P and two float4 of V (a warp reads
//       each V row as contiguous 256-byte halves).
// A query block with no kept key block writes zeros.
#include <math.h>

#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kRows = 32;        // query rows per CTA (four CTAs per item)
constexpr int kSplit = kBlock / kRows;
constexpr int kTK = 16;          // keys per sub-tile
constexpr int kSub = kBlock / kTK;
constexpr int kThreads = 128;
constexpr int kQS = 132;         // Q row stride (floats)
constexpr int kKS = 132;         // K row stride
constexpr int kVS = 128;         // V row stride (rows are read whole)
constexpr int kPS = 36;          // Pᵀ row stride: Pᵀ[key][row], 32 rows + pad (float4-aligned)

struct F32Smem {
    float q[kRows * kQS];
    float k[2][kTK * kKS];
    float v[2][kTK * kVS];
    float pt[kTK * kPS];
    float alpha[kRows];
    float linv[kRows];
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 4)
    attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, KvPages pages,
                    int heads, int nq, int nk, const int32_t* __restrict__ kidx, const int32_t* __restrict__ kcnt,
                    float* __restrict__ out, int item_begin, const int32_t* __restrict__ order, OutRows rows) {
    extern __shared__ float4 smem4[];
    F32Smem& sm = *reinterpret_cast<F32Smem*>(smem4);
    griddep_wait_then_release();
    const int slot = (int)(blockIdx.x / kSplit), part = (int)(blockIdx.x % kSplit);
    const int item = order ? order[slot] : item_begin + slot;
    const int h = item / nq, qb = item % nq;
    const int64_t ld = (int64_t)heads * kD;
    const int tid = threadIdx.x;
    const int row0 = part * kRows;  // this CTA's first row inside the query block
    int cnt = kcnt[item];
    cnt = cnt < 0 ? 0 : (cnt > nk ? nk : cnt);
    // PV / output mapping
    const int rq = tid >> 4, dg = tid & 15;
    if (cnt == 0) {  // SparseAttention.swift:47-53: a query block that selected nothing writes zeros
        for (int i = 0; i < 4; ++i) {
            float* orow = out + rows.row(qb, row0 + 4 * rq + i) * ld + h * kD;
            reinterpret_cast<float4*>(orow)[dg] = make_float4(0.f, 0.f, 0.f, 0.f);
            reinterpret_cast<float4*>(orow)[16 + dg] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        return;
    }
    const int32_t* lst = kidx + (int64_t)item * nk;
    const int steps = cnt * kSub;
    // the K and V rows of sub-tile `step` into buffer `b`: 16 keys × 32 float4 each, four of each per thread
    auto issue = [&](int step, int b) {
        int kb = __ldg(lst + step / kSub);
        kb = kb < 0 ? 0 : (kb >= nk ? nk - 1 : kb);
        const int64_t key0 = (int64_t)kv_phys_block(pages, kb) * kBlock + (step % kSub) * kTK;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = tid + kThreads * i, c = idx >> 5, e4 = idx & 31;
            const int64_t g = (key0 + c) * ld + h * kD + 4 * e4;
            cp_async16(sm.k[b] + c * kKS + 4 * e4, k + g);
            cp_async16(sm.v[b] + c * kVS + 4 * e4, v + g);
        }
    };
    {
        const float* qsrc = q + (rows.q_row(qb) + row0) * ld + h * kD;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = tid + kThreads * i, r = idx >> 5, e4 = idx & 31;
            cp_async16(sm.q + r * kQS + 4 * e4, qsrc + r * ld + 4 * e4);
        }
        issue(0, 0);
        cp_async_commit();
    }
    const float scale = 1.0f / sqrtf((float)kD);
    // S mapping: rows 2·rp + {0,1}, keys ks + {0, 8}
    const int rp = tid >> 3, ks = tid & 7;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    float o[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) o[i][j] = 0.0f;

    for (int step = 0; step < steps; ++step) {
        const int b = step & 1;
        cp_async_wait_all();
        __syncthreads();  // this sub-tile has landed everywhere, and every thread is done with buffer b ^ 1
        if (step + 1 < steps) {
            issue(step + 1, b ^ 1);
            cp_async_commit();
        }
        // ---- S = Q·Kᵀ for 2 rows × 2 keys ----
        float s[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        const float4* q0 = reinterpret_cast<const float4*>(sm.q + (2 * rp) * kQS);
        const float4* q1 = reinterpret_cast<const float4*>(sm.q + (2 * rp + 1) * kQS);
        const float4* k0 = reinterpret_cast<const float4*>(sm.k[b] + ks * kKS);
        const float4* k1 = reinterpret_cast<const float4*>(sm.k[b] + (ks + 8) * kKS);
#pragma unroll 8
        for (int e4 = 0; e4 < 32; ++e4) {
            const float4 a0 = q0[e4], a1 = q1[e4], b0 = k0[e4], b1 = k1[e4];
            s[0][0] = fmaf(a0.x, b0.x, s[0][0]); s[0][0] = fmaf(a0.y, b0.y, s[0][0]);
            s[0][0] = fmaf(a0.z, b0.z, s[0][0]); s[0][0] = fmaf(a0.w, b0.w, s[0][0]);
            s[0][1] = fmaf(a0.x, b1.x, s[0][1]); s[0][1] = fmaf(a0.y, b1.y, s[0][1]);
            s[0][1] = fmaf(a0.z, b1.z, s[0][1]); s[0][1] = fmaf(a0.w, b1.w, s[0][1]);
            s[1][0] = fmaf(a1.x, b0.x, s[1][0]); s[1][0] = fmaf(a1.y, b0.y, s[1][0]);
            s[1][0] = fmaf(a1.z, b0.z, s[1][0]); s[1][0] = fmaf(a1.w, b0.w, s[1][0]);
            s[1][1] = fmaf(a1.x, b1.x, s[1][1]); s[1][1] = fmaf(a1.y, b1.y, s[1][1]);
            s[1][1] = fmaf(a1.z, b1.z, s[1][1]); s[1][1] = fmaf(a1.w, b1.w, s[1][1]);
        }
        // ---- online softmax per row over the eight lanes of the row pair ----
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            s[j][0] *= scale;
            s[j][1] *= scale;
            float mx = fmaxf(s[j][0], s[j][1]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            const float mn = fmaxf(m[j], mx);
            const float p0 = expf(s[j][0] - mn), p1 = expf(s[j][1] - mn);
            float sum = p0 + p1;
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            const float al = expf(m[j] - mn);  // 0 on the first sub-tile (m = −inf)
            l[j] = l[j] * al + sum;
            m[j] = mn;
            sm.pt[ks * kPS + 2 * rp + j] = p0;
            sm.pt[(ks + 8) * kPS + 2 * rp + j] = p1;
            if (ks == 0) sm.alpha[2 * rp + j] = al;
        }
        __syncthreads();
        // ---- O = O·alpha + P·V for 4 rows × 8 dims ----
        {
            const float4 al = *reinterpret_cast<const float4*>(sm.alpha + 4 * rq);
            const float a4[4] = {al.x, al.y, al.z, al.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) o[i][j] *= a4[i];
            const float* vb = sm.v[b];
#pragma unroll 4
            for (int c = 0; c < kTK; ++c) {
                const float4 p = *reinterpret_cast<const float4*>(sm.pt + c * kPS + 4 * rq);
                const float4 v0 = reinterpret_cast<const float4*>(vb + c * kVS)[dg];
                const float4 v1 = reinterpret_cast<const float4*>(vb + c * kVS)[16 + dg];
                const float pp[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    o[i][0] = fmaf(pp[i], v0.x, o[i][0]);
                    o[i][1] = fmaf(pp[i], v0.y, o[i][1]);
                    o[i][2] = fmaf(pp[i], v0.z, o[i][2]);
                    o[i][3] = fmaf(pp[i], v0.w, o[i][3]);
                    o[i][4] = fmaf(pp[i], v1.x, o[i][4]);
                    o[i][5] = fmaf(pp[i], v1.y, o[i][5]);
                    o[i][6] = fmaf(pp[i], v1.z, o[i][6]);
                    o[i][7] = fmaf(pp[i], v1.w, o[i][7]);
                }
            }
        }
    }
    if (ks == 0) {
        sm.linv[2 * rp] = 1.0f / l[0];
        sm.linv[2 * rp + 1] = 1.0f / l[1];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float inv = sm.linv[4 * rq + i];
        float* orow = out + rows.row(qb, row0 + 4 * rq + i) * ld + h * kD;
        reinterpret_cast<float4*>(orow)[dg] = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
        reinterpret_cast<float4*>(orow)[16 + dg] =
            make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
    }
}

}  // namespace

cudaError_t launch_attn_f32(const float* q, const float* k, const float* v, const KvPages& pages, int heads, int nq,
                            int nk, const int32_t* kidx, const int32_t* kcnt, float* out, int item_begin,
                            int item_count, const int32_t* order, cudaStream_t st, OutRows rows) {
    if (item_count <= 0) return cudaSuccess;
    const int smem = (int)sizeof(F32Smem);
    cudaError_t e = cudaFuncSetAttribute(attn_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_f32_kernel, dim3((unsigned)item_count * kSplit), dim3(kThreads), (size_t)smem, st, q, k, v,
                      pages, heads, nq, nk, kidx, kcnt, out, item_begin, order, rows);
}

}  // namespace fvsr
