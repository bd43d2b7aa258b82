// attn_f32.cu — fp32 block-sparse attention on the CUDA cores (the fp32 lane of kernelBlockAttention,
// SparseAttention.swift:169-187; DiT.swift:279-313 semantics).
//
// fp32 inputs must meet 1e-5 relative error against an fp32 reference, which tf32 tensor-core arithmetic cannot, so
// this lane runs plain fp32 FFMA. One CTA per (head, query block); 256 threads, thread t owns query row t/2 and, in
// the interleaved split, keys c ≡ t (mod 2) of each 32-key tile for S and output dims [64·(t%2), 64·(t%2)+64) for O.
// Online softmax in fp32 with accurate expf. A query block with no kept key block writes zeros.
#include <math.h>

#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kTK = 32;    // keys per staged tile
constexpr int kQS = 132;   // padded Q row stride (floats)
constexpr int kKS = 132;   // padded K row stride
constexpr int kVS = 136;   // V row stride: dims [0,64) at 0, dims [64,128) at 68 (bank-split halves)

struct F32Smem {
    float q[kBlock * kQS];
    float k[kTK * kKS];
    float v[kTK * kVS];
};

__global__ void __launch_bounds__(256) attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                       const float* __restrict__ v, KvPages pages, int heads, int nq,
                                                       int nk, const int32_t* __restrict__ kidx,
                                                       const int32_t* __restrict__ kcnt, float* __restrict__ out,
                                                       int item_begin, const int32_t* __restrict__ order,
                                                       OutRows rows) {
    extern __shared__ float4 smem4[];
    F32Smem& sm = *reinterpret_cast<F32Smem*>(smem4);
    griddep_wait_then_release();
    const int item = order ? order[blockIdx.x] : item_begin + (int)blockIdx.x;
    const int h = item / nq, qb = item % nq;
    const int64_t ld = (int64_t)heads * kD;
    const int tid = threadIdx.x;
    const int r = tid >> 1, hf = tid & 1;
    int cnt = kcnt[item];
    cnt = cnt < 0 ? 0 : (cnt > nk ? nk : cnt);
    float* orow = out + rows.row(qb, r) * ld + h * kD + hf * 64;
    if (cnt == 0) {
        for (int i = 0; i < 16; ++i) reinterpret_cast<float4*>(orow)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    for (int idx = tid; idx < kBlock * 32; idx += 256) {
        const int rr = idx >> 5, e4 = idx & 31;
        *reinterpret_cast<float4*>(sm.q + rr * kQS + e4 * 4) =
            __ldg(reinterpret_cast<const float4*>(q + (rows.q_row(qb) + rr) * ld + h * kD) + e4);
    }
    const float scale = 1.0f / sqrtf((float)kD);
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.0f;
    float m = -INFINITY, l = 0.0f;
    const int32_t* lst = kidx + (int64_t)item * nk;
    for (int jj = 0; jj < cnt; ++jj) {
        int kb = lst[jj];
        kb = kb < 0 ? 0 : (kb >= nk ? nk - 1 : kb);
        const int64_t krow0 = (int64_t)kv_phys_block(pages, kb) * kBlock;
        for (int sub = 0; sub < kBlock / kTK; ++sub) {
            __syncthreads();
            for (int idx = tid; idx < kTK * 32; idx += 256) {
                const int c = idx >> 5, e4 = idx & 31;
                const int64_t g = (krow0 + sub * kTK + c) * ld + h * kD;
                *reinterpret_cast<float4*>(sm.k + c * kKS + e4 * 4) = __ldg(reinterpret_cast<const float4*>(k + g) + e4);
                *reinterpret_cast<float4*>(sm.v + c * kVS + e4 * 4 + (e4 >= 16 ? 4 : 0)) =
                    __ldg(reinterpret_cast<const float4*>(v + g) + e4);
            }
            __syncthreads();
            float s[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) s[i] = 0.0f;
            const float4* qr = reinterpret_cast<const float4*>(sm.q + r * kQS);
#pragma unroll 4
            for (int e4 = 0; e4 < 32; ++e4) {
                const float4 a = qr[e4];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float4 b = reinterpret_cast<const float4*>(sm.k + (2 * i + hf) * kKS)[e4];
                    s[i] = fmaf(a.x, b.x, s[i]);
                    s[i] = fmaf(a.y, b.y, s[i]);
                    s[i] = fmaf(a.z, b.z, s[i]);
                    s[i] = fmaf(a.w, b.w, s[i]);
                }
            }
            float mx = m;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                s[i] *= scale;
                mx = fmaxf(mx, s[i]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            const float alpha = expf(m - mx);
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                s[i] = expf(s[i] - mx);
                sum += s[i];
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            l = l * alpha + sum;
            m = mx;
#pragma unroll
            for (int i = 0; i < 64; ++i) o[i] *= alpha;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float other = __shfl_xor_sync(0xffffffffu, s[i], 1);
                const float p_even = hf ? other : s[i];  // key 2i
                const float p_odd = hf ? s[i] : other;   // key 2i + 1
                const float4* v0 = reinterpret_cast<const float4*>(sm.v + (2 * i) * kVS + hf * 68);
                const float4* v1 = reinterpret_cast<const float4*>(sm.v + (2 * i + 1) * kVS + hf * 68);
#pragma unroll
                for (int d4 = 0; d4 < 16; ++d4) {
                    const float4 a = v0[d4], b = v1[d4];
                    o[4 * d4 + 0] = fmaf(p_odd, b.x, fmaf(p_even, a.x, o[4 * d4 + 0]));
                    o[4 * d4 + 1] = fmaf(p_odd, b.y, fmaf(p_even, a.y, o[4 * d4 + 1]));
                    o[4 * d4 + 2] = fmaf(p_odd, b.z, fmaf(p_even, a.z, o[4 * d4 + 2]));
                    o[4 * d4 + 3] = fmaf(p_odd, b.w, fmaf(p_even, a.w, o[4 * d4 + 3]));
                }
            }
        }
    }
    const float inv = 1.0f / l;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        reinterpret_cast<float4*>(orow)[i] =
            make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
}

}  // namespace

cudaError_t launch_attn_f32(const float* q, const float* k, const float* v, const KvPages& pages, int heads, int nq,
                            int nk, const int32_t* kidx, const int32_t* kcnt, float* out, int item_begin,
                            int item_count, const int32_t* order, cudaStream_t st, OutRows rows) {
    if (item_count <= 0) return cudaSuccess;
    const int smem = (int)sizeof(F32Smem);
    cudaError_t e = cudaFuncSetAttribute(attn_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_f32_kernel, dim3(item_count), dim3(256), (size_t)smem, st, q, k, v, pages, heads, nq, nk,
                      kidx, kcnt, out, item_begin, order, rows);
}

}  // namespace fvsr
