// prepare.cu — the q/k/v side of one LCSA layer (blockForward, DiT.swift:497-506) in one pass over the three linear
// outputs, which arrive in token order (F, 8·bh, 8·bw):
//   q, k: WanRMSNorm (DiT.swift:34-47): x·rsqrt(mean(x²) + eps) in fp32, rounded to the storage type, times the
//         weight (rounded again); then ropeApply (DiT.swift:100-107): pairs (2j, 2j+1) of each head rotated by the
//         token's (cos, sin)_j in fp32, each product and sum rounded separately, then rounded to the storage type;
//   q, k, v: windowPartition (DiT.swift:113-118) — written in window order;
//   and the fp32 block means of the rotated q and k (DiT.swift:161-162) with pool_kernel's summation order, so the
//   selection sees exactly the pooled vectors that pooling the window-ordered outputs would give.
// K and V go to the arena blocks a KvPages table names: the pages of a window cache (the append of DiT.swift:508-511
// fused into this pass) or one contiguous window-ordered buffer.
//
// HBM-bound: algorithmic bytes per window = 3·128·C·elt read + 3·128·C·elt written + 2·128·64·8 rotation tables read
// (q and k) + 2·C·4 pooled written.
// Layout: CTA = one window of one tensor (blockIdx.y: 0 q, 1 k, 2 v); warp g walks tokens [32g, 32g + 32) of the
// window in window order; lane l holds channels 128·i + 4l .. 4l + 3 of every head i, so one token's sum of squares
// is a lane partial plus a five-step butterfly (every lane ends with the same value: a + b = b + a), both rotation
// pairs of a lane use the lane's two table entries j = 2l, 2l + 1, and a warp moves 256 contiguous bytes (bf16) of a
// head per instruction.
#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kPrepThreads = 128;
constexpr int kPrepMaxC = kPrepMaxHeads * kD;

template <int DT>
struct Lane4;  // four channels of one lane
template <>
struct Lane4<1> {
    using V = uint2;
};
template <>
struct Lane4<0> {
    using V = float4;
};

__device__ __forceinline__ void unpack4(const uint2& v, float f[4]) {
    f[0] = bf16_bits_to_float(v.x & 0xFFFFu);
    f[1] = bf16_bits_to_float(v.x >> 16);
    f[2] = bf16_bits_to_float(v.y & 0xFFFFu);
    f[3] = bf16_bits_to_float(v.y >> 16);
}
__device__ __forceinline__ void unpack4(const float4& v, float f[4]) {
    f[0] = v.x;
    f[1] = v.y;
    f[2] = v.z;
    f[3] = v.w;
}
// f holds values of the storage type already (to_t), so the bf16 packing keeps the high halves exactly.
__device__ __forceinline__ void pack4(const float f[4], uint2& v) {
    v.x = (__float_as_uint(f[0]) >> 16) | (__float_as_uint(f[1]) & 0xFFFF0000u);
    v.y = (__float_as_uint(f[2]) >> 16) | (__float_as_uint(f[3]) & 0xFFFF0000u);
}
__device__ __forceinline__ void pack4(const float f[4], float4& v) { v = make_float4(f[0], f[1], f[2], f[3]); }

template <int DT>
__device__ __forceinline__ float to_t(float x) {  // round to the storage type (nearest even)
    if constexpr (DT == 1)
        return __bfloat162float(__float2bfloat16_rn(x));
    else
        return x;
}

template <int DT, int NH>
__global__ void __launch_bounds__(kPrepThreads) prepare_kernel(const __grid_constant__ PrepArgs a) {
    using V = typename Lane4<DT>::V;
    __shared__ float part[4][kPrepMaxC];
    __shared__ float wsm[kPrepMaxC];
    griddep_wait_then_release();
    if (a.zero) {
        const size_t nb = (size_t)gridDim.x * gridDim.y, bid = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
        for (size_t w = bid * kPrepThreads + threadIdx.x; w < a.zero_words; w += nb * kPrepThreads) a.zero[w] = 0;
    }
    const int role = blockIdx.y, win = blockIdx.x;
    const int heads = a.heads, C = heads * kD, cv = C / 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const void* wt = role < 2 ? a.norm_w[role] : nullptr;
    const bool rope = role < 2 && a.cosv != nullptr;
    float* pooled = role < 2 ? a.pooled[role] : nullptr;
    if (wt) {  // CTA-uniform
        for (int c = threadIdx.x; c < C; c += kPrepThreads)
            wsm[c] = DT == 1 ? bf16_bits_to_float(static_cast<const uint16_t*>(wt)[c]) : static_cast<const float*>(wt)[c];
        __syncthreads();
    }
    const int64_t blk = role == 0 ? (int64_t)win : (int64_t)kv_phys_block(a.kv_pages, win);
    const V* src = static_cast<const V*>(a.x[role]);
    V* dst = static_cast<V*>(role == 0 ? a.q_out : a.kv_out[role - 1]) + blk * kBlock * cv;
    float acc[4 * NH];
#pragma unroll
    for (int i = 0; i < 4 * NH; ++i) acc[i] = 0.0f;

#pragma unroll 1
    for (int t = 0; t < 32; ++t) {
        const int r = 32 * warp + t;
        const int64_t tok = token_row(a.bh, a.bw, win, r);
        V raw[NH];
#pragma unroll
        for (int i = 0; i < NH; ++i)
            if (i < heads) raw[i] = __ldcs(src + tok * cv + 32 * i + lane);
        float2 cs = make_float2(1.0f, 1.0f), sn = make_float2(0.0f, 0.0f);
        if (rope) {
            cs = __ldg(reinterpret_cast<const float2*>(a.cosv + tok * 64) + lane);
            sn = __ldg(reinterpret_cast<const float2*>(a.sinv + tok * 64) + lane);
        }
        float inv = 1.0f;
        if (wt) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < NH; ++i)
                if (i < heads) {
                    float f[4];
                    unpack4(raw[i], f);
#pragma unroll
                    for (int e = 0; e < 4; ++e) ss = __fadd_rn(ss, __fmul_rn(f[e], f[e]));
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
            inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)C), a.eps));
        }
#pragma unroll
        for (int i = 0; i < NH; ++i)
            if (i < heads) {
                float f[4];
                unpack4(raw[i], f);
                if (wt) {
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        f[e] = to_t<DT>(__fmul_rn(to_t<DT>(__fmul_rn(f[e], inv)), wsm[kD * i + 4 * lane + e]));
                }
                if (rope) {
                    const float r0 = f[0], i0 = f[1], r1 = f[2], i1 = f[3];
                    f[0] = to_t<DT>(__fsub_rn(__fmul_rn(r0, cs.x), __fmul_rn(i0, sn.x)));
                    f[1] = to_t<DT>(__fadd_rn(__fmul_rn(r0, sn.x), __fmul_rn(i0, cs.x)));
                    f[2] = to_t<DT>(__fsub_rn(__fmul_rn(r1, cs.y), __fmul_rn(i1, sn.y)));
                    f[3] = to_t<DT>(__fadd_rn(__fmul_rn(r1, sn.y), __fmul_rn(i1, cs.y)));
                }
                if (pooled) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[4 * i + e] = __fadd_rn(acc[4 * i + e], f[e]);
                }
                V o;
                pack4(f, o);
                dst[(int64_t)r * cv + 32 * i + lane] = o;
            }
    }

    if (pooled) {  // CTA-uniform
#pragma unroll
        for (int i = 0; i < NH; ++i)
            if (i < heads) {
#pragma unroll
                for (int e = 0; e < 4; ++e) part[warp][kD * i + 4 * lane + e] = acc[4 * i + e];
            }
        __syncthreads();
        for (int c = threadIdx.x; c < C; c += kPrepThreads) {
            const float sum = __fadd_rn(__fadd_rn(part[0][c], part[1][c]), __fadd_rn(part[2][c], part[3][c]));
            pooled[blk * C + c] = __fmul_rn(sum, 0.0078125f);
        }
    }
}

template <int DT>
cudaError_t launch_prepare_t(const PrepArgs& a, cudaStream_t st) {
    const dim3 grid((unsigned)a.nq, 3), block(kPrepThreads);
    if (a.heads <= 4) return launch_pdl(prepare_kernel<DT, 4>, grid, block, 0, st, a);
    if (a.heads <= 8) return launch_pdl(prepare_kernel<DT, 8>, grid, block, 0, st, a);
    if (a.heads <= 12) return launch_pdl(prepare_kernel<DT, 12>, grid, block, 0, st, a);
    return launch_pdl(prepare_kernel<DT, 16>, grid, block, 0, st, a);
}

}  // namespace

cudaError_t launch_prepare(const PrepArgs& a, int dtype, cudaStream_t st) {
    if (a.nq <= 0) return cudaSuccess;
    if (a.heads < 1 || a.heads > kPrepMaxHeads) return cudaErrorInvalidValue;
    return dtype == 1 ? launch_prepare_t<1>(a, st) : launch_prepare_t<0>(a, st);
}

}  // namespace fvsr
