// norm.cu — the row normalisations of FlashVSR's DiT block around the path (DiT.swift:34-47, 371-377, 489-494, 543-546):
//   layernorm_kernel  LayerNorm over the channels (no affine, or affine), optionally followed by the block's
//                     modulation y·(1 + scale) + shift — norm1/norm2 with the MSA / MLP shift and scale, and norm3;
//   rmsnorm_kernel    WanRMSNorm (the cross-attention's normQ).
// One warp per row of C channels (C a multiple of 256, at most 2048), 8 bf16 per lane per 128-bit load; the row stays
// in registers between the passes. fp32 statistics; bf16 rounding points as the reference's ops leave them:
//   LayerNorm: mean = Σx / C, var = Σ(x − mean)² / C (two passes), n = (x − mean) / √(var + eps), rounded; affine:
//              round(n·w + b) from the unrounded n (one fused op); modulation: round(round(n·round(1 + scale)) + shift);
//   RMSNorm:   inv = 1 / √(Σx² / C + eps), round(round(x·inv)·w).
// Sums run as lane partials in channel order, then a xor butterfly (MLX's order is unspecified).
#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kMaxChunks = 8;  // 8 × 256 = 2048 channels

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ void load_row(const __nv_bfloat16* row, int nch, int lane, float (&x)[kMaxChunks * 8]) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c < nch) {
            const uint4 u = *reinterpret_cast<const uint4*>(row + 256 * c + 8 * lane);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                x[8 * c + 2 * i] = bf16_bits_to_float(w[i] & 0xFFFFu);
                x[8 * c + 2 * i + 1] = bf16_bits_to_float(w[i] >> 16);
            }
        }
    }
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float ldb(const __nv_bfloat16* p, int i) { return __bfloat162float(p[i]); }

__global__ void __launch_bounds__(256) layernorm_kernel(int m, int ch, const __nv_bfloat16* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ weight,
                                                        const __nv_bfloat16* __restrict__ bias,
                                                        const __nv_bfloat16* __restrict__ shift,
                                                        const __nv_bfloat16* __restrict__ scale, float eps,
                                                        __nv_bfloat16* __restrict__ out) {
    griddep_wait_then_release();
    const int warp = (int)(blockIdx.x * 8 + (threadIdx.x >> 5)), lane = threadIdx.x & 31;
    if (warp >= m) return;
    const int nch = ch / 256;
    const __nv_bfloat16* row = x + (int64_t)warp * ch;
    float v[kMaxChunks * 8];
    load_row(row, nch, lane, v);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxChunks * 8; ++i)
        if (i < nch * 8) s = __fadd_rn(s, v[i]);
    const float mean = __fdiv_rn(warp_sum(s), (float)ch);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxChunks * 8; ++i)
        if (i < nch * 8) {
            const float d = __fsub_rn(v[i], mean);
            q = __fmaf_rn(d, d, q);
        }
    const float var = __fdiv_rn(warp_sum(q), (float)ch);
    const float rstd = __frcp_rn(__fsqrt_rn(__fadd_rn(var, eps)));
    __nv_bfloat16* orow = out + (int64_t)warp * ch;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c >= nch) continue;
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            float y[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int col = 256 * c + 8 * lane + i + u;
                float n = __fmul_rn(__fsub_rn(v[8 * c + i + u], mean), rstd);
                if (weight) n = __fmaf_rn(n, ldb(weight, col), bias ? ldb(bias, col) : 0.0f);
                n = bf(n);
                if (scale) n = bf(__fadd_rn(bf(__fmul_rn(n, bf(__fadd_rn(1.0f, ldb(scale, col))))), ldb(shift, col)));
                y[u] = n;
            }
            w[i >> 1] = pack2(y[0], y[1]);
        }
        *reinterpret_cast<uint4*>(orow + 256 * c + 8 * lane) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(int m, int ch, const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ weight, float eps,
                                                      __nv_bfloat16* __restrict__ out) {
    griddep_wait_then_release();
    const int warp = (int)(blockIdx.x * 8 + (threadIdx.x >> 5)), lane = threadIdx.x & 31;
    if (warp >= m) return;
    const int nch = ch / 256;
    float v[kMaxChunks * 8];
    load_row(x + (int64_t)warp * ch, nch, lane, v);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxChunks * 8; ++i)
        if (i < nch * 8) s = __fmaf_rn(v[i], v[i], s);
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(s), (float)ch), eps)));
    __nv_bfloat16* orow = out + (int64_t)warp * ch;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
        if (c >= nch) continue;
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            const int col = 256 * c + 8 * lane + i;
            const float y0 = bf(__fmul_rn(bf(__fmul_rn(v[8 * c + i], inv)), ldb(weight, col)));
            const float y1 = bf(__fmul_rn(bf(__fmul_rn(v[8 * c + i + 1], inv)), ldb(weight, col + 1)));
            w[i >> 1] = pack2(y0, y1);
        }
        *reinterpret_cast<uint4*>(orow + 256 * c + 8 * lane) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace

cudaError_t launch_layernorm(int m, int ch, const void* x, const void* weight, const void* bias, const void* shift,
                             const void* scale, float eps, void* out, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    return launch_pdl(layernorm_kernel, dim3((m + 7) / 8), dim3(256), 0, st, m, ch,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
                      static_cast<const __nv_bfloat16*>(bias), static_cast<const __nv_bfloat16*>(shift),
                      static_cast<const __nv_bfloat16*>(scale), eps, static_cast<__nv_bfloat16*>(out));
}

cudaError_t launch_rmsnorm(int m, int ch, const void* x, const void* weight, float eps, void* out, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    return launch_pdl(rmsnorm_kernel, dim3((m + 7) / 8), dim3(256), 0, st, m, ch,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight), eps,
                      static_cast<__nv_bfloat16*>(out));
}

}  // namespace fvsr
