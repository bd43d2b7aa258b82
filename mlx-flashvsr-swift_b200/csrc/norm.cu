// norm.cu — the row normalisations of FlashVSR's DiT block around the path (DiT.swift:34-47, 371-377, 489-494, 543-546):
//   layernorm_kernel  LayerNorm over the channels (no affine, or affine), optionally followed by the block's
//                     modulation y·(1 + scale) + shift — norm1/norm2 with the MSA / MLP shift and scale, and norm3;
//   rmsnorm_kernel    WanRMSNorm (the cross-attention's normQ).
// A CTA of 8 warps stages the per-channel vectors (weight, bias, shift, round(1 + scale)) once in shared memory as fp32,
// then each warp walks rows (C channels, C a multiple of 256, at most 2048), 8 bf16 per lane per 128-bit load; the
// row stays in registers between the passes. The grid is a few CTAs per SM, so the staging is paid a few times per SM
// rather than once per 8 rows. fp32 statistics; bf16 rounding points as the reference's ops leave them:
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

// Shared-memory vectors of a CTA: [kVecs][ch] fp32.
enum { kVW = 0, kVB = 1, kVShift = 2, kVScale1 = 3, kVecs = 4 };

template <int NCH>
__global__ void __launch_bounds__(256, 2) layernorm_kernel(int m, int ch, const __nv_bfloat16* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ weight,
                                                        const __nv_bfloat16* __restrict__ bias,
                                                        const __nv_bfloat16* __restrict__ shift,
                                                        const __nv_bfloat16* __restrict__ scale, float eps,
                                                        __nv_bfloat16* __restrict__ out) {
    extern __shared__ float vec[];
    griddep_wait_then_release();
    for (int i = threadIdx.x; i < ch; i += blockDim.x) {
        vec[kVW * ch + i] = weight ? ldb(weight, i) : 1.0f;
        vec[kVB * ch + i] = bias ? ldb(bias, i) : 0.0f;
        vec[kVShift * ch + i] = shift ? ldb(shift, i) : 0.0f;
        vec[kVScale1 * ch + i] = scale ? bf(__fadd_rn(1.0f, ldb(scale, i))) : 1.0f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    constexpr int nch = NCH;
    const bool affine = weight != nullptr, modulate = scale != nullptr;
    for (int rowi = (int)(blockIdx.x * 8 + (threadIdx.x >> 5)); rowi < m; rowi += (int)gridDim.x * 8) {
        const __nv_bfloat16* row = x + (int64_t)rowi * ch;
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
        __nv_bfloat16* orow = out + (int64_t)rowi * ch;
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) {
            if (c >= nch) continue;
            const int col0 = 256 * c + 8 * lane;
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                float y[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int col = col0 + i + u;
                    float n = __fmul_rn(__fsub_rn(v[8 * c + i + u], mean), rstd);
                    if (affine) n = __fmaf_rn(n, vec[kVW * ch + col], vec[kVB * ch + col]);
                    n = bf(n);
                    if (modulate) n = bf(__fadd_rn(bf(__fmul_rn(n, vec[kVScale1 * ch + col])), vec[kVShift * ch + col]));
                    y[u] = n;
                }
                w[i >> 1] = pack2(y[0], y[1]);
            }
            *reinterpret_cast<uint4*>(orow + col0) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

template <int NCH>
__global__ void __launch_bounds__(256, 2) rmsnorm_kernel(int m, int ch, const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ weight, float eps,
                                                      __nv_bfloat16* __restrict__ out) {
    extern __shared__ float vec[];
    griddep_wait_then_release();
    for (int i = threadIdx.x; i < ch; i += blockDim.x) vec[i] = ldb(weight, i);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    constexpr int nch = NCH;
    for (int rowi = (int)(blockIdx.x * 8 + (threadIdx.x >> 5)); rowi < m; rowi += (int)gridDim.x * 8) {
        float v[kMaxChunks * 8];
        load_row(x + (int64_t)rowi * ch, nch, lane, v);
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxChunks * 8; ++i)
            if (i < nch * 8) s = __fmaf_rn(v[i], v[i], s);
        const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(warp_sum(s), (float)ch), eps)));
        __nv_bfloat16* orow = out + (int64_t)rowi * ch;
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) {
            if (c >= nch) continue;
            const int col0 = 256 * c + 8 * lane;
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const float y0 = bf(__fmul_rn(bf(__fmul_rn(v[8 * c + i], inv)), vec[col0 + i]));
                const float y1 = bf(__fmul_rn(bf(__fmul_rn(v[8 * c + i + 1], inv)), vec[col0 + i + 1]));
                w[i >> 1] = pack2(y0, y1);
            }
            *reinterpret_cast<uint4*>(orow + col0) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// As many CTAs as fit on the SMs at once (one wave; the row loop does the rest), never more than 8-row groups.
template <typename Kernel>
int norm_grid(Kernel kernel, size_t smem, int m) {
    int dev = 0, nsm = 148, per_sm = 2;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const int groups = (m + 7) / 8;
    return groups < per_sm * nsm ? groups : per_sm * nsm;
}

template <int NCH>
cudaError_t layernorm_nch(int m, int ch, const void* x, const void* weight, const void* bias, const void* shift,
                          const void* scale, float eps, void* out, cudaStream_t st) {
    const size_t smem = (size_t)kVecs * ch * sizeof(float);
    return launch_pdl(layernorm_kernel<NCH>, dim3(norm_grid(layernorm_kernel<NCH>, smem, m)), dim3(256), smem, st, m,
                      ch, static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
                      static_cast<const __nv_bfloat16*>(bias), static_cast<const __nv_bfloat16*>(shift),
                      static_cast<const __nv_bfloat16*>(scale), eps, static_cast<__nv_bfloat16*>(out));
}

template <int NCH>
cudaError_t rmsnorm_nch(int m, int ch, const void* x, const void* weight, float eps, void* out, cudaStream_t st) {
    const size_t smem = (size_t)ch * sizeof(float);
    return launch_pdl(rmsnorm_kernel<NCH>, dim3(norm_grid(rmsnorm_kernel<NCH>, smem, m)), dim3(256), smem, st, m, ch,
                      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight), eps,
                      static_cast<__nv_bfloat16*>(out));
}

}  // namespace

cudaError_t launch_layernorm(int m, int ch, const void* x, const void* weight, const void* bias, const void* shift,
                             const void* scale, float eps, void* out, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    switch (ch / 256) {
        case 1: return layernorm_nch<1>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        case 2: return layernorm_nch<2>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        case 3: return layernorm_nch<3>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        case 4: return layernorm_nch<4>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        case 5: return layernorm_nch<5>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        case 6: return layernorm_nch<6>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        case 7: return layernorm_nch<7>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        case 8: return layernorm_nch<8>(m, ch, x, weight, bias, shift, scale, eps, out, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_rmsnorm(int m, int ch, const void* x, const void* weight, float eps, void* out, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    switch (ch / 256) {
        case 1: return rmsnorm_nch<1>(m, ch, x, weight, eps, out, st);
        case 2: return rmsnorm_nch<2>(m, ch, x, weight, eps, out, st);
        case 3: return rmsnorm_nch<3>(m, ch, x, weight, eps, out, st);
        case 4: return rmsnorm_nch<4>(m, ch, x, weight, eps, out, st);
        case 5: return rmsnorm_nch<5>(m, ch, x, weight, eps, out, st);
        case 6: return rmsnorm_nch<6>(m, ch, x, weight, eps, out, st);
        case 7: return rmsnorm_nch<7>(m, ch, x, weight, eps, out, st);
        case 8: return rmsnorm_nch<8>(m, ch, x, weight, eps, out, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace fvsr
