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
#include "sm100.cuh"

namespace fvsr {

namespace {

using namespace sm100;

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

__device__ __forceinline__ float ldb(const __nv_bfloat16* p, int i) { return __bfloat162float(p[i]); }

// Shared-memory vectors of a CTA: [kVecs][ch] fp32, each stored so that the eight columns a lane owns in a 256-column
// chunk (256c + 8·lane + 0..7) are two float4 at ((2c + h)·32 + lane)·4, h = 0, 1: a warp's float4 reads are
// consecutive 16-byte words (no bank conflicts; the natural layout gives 8-way conflicts on scalar reads).
enum { kVW = 0, kVB = 1, kVShift = 2, kVScale1 = 3, kVecs = 4 };
__device__ __forceinline__ int vec_pos(int col) {
    const int c = col >> 8, lane = (col >> 3) & 31, i = col & 7;
    return (((c << 1) + (i >> 2)) * 32 + lane) * 4 + (i & 3);
}
// The eight vector values of a lane's columns in chunk c.
__device__ __forceinline__ void vec8(const float* v, int c, int lane, float (&out)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(v + ((2 * c) * 32 + lane) * 4);
    const float4 b = *reinterpret_cast<const float4*>(v + ((2 * c + 1) * 32 + lane) * 4);
    out[0] = a.x, out[1] = a.y, out[2] = a.z, out[3] = a.w, out[4] = b.x, out[5] = b.y, out[6] = b.z, out[7] = b.w;
}

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
        const int pos = vec_pos(i);
        vec[kVW * ch + pos] = weight ? ldb(weight, i) : 1.0f;
        vec[kVB * ch + pos] = bias ? ldb(bias, i) : 0.0f;
        vec[kVShift * ch + pos] = shift ? ldb(shift, i) : 0.0f;
        vec[kVScale1 * ch + pos] = scale ? bf(__fadd_rn(1.0f, ldb(scale, i))) : 1.0f;
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
        const uint64_t negmean2 = f2(-mean, -mean), rstd2 = f2(rstd, rstd);
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) {
            if (c >= nch) continue;
            const int col0 = 256 * c + 8 * lane;
            float wv[8], bv[8], s1[8], sh[8];
            if (affine) {
                vec8(vec + kVW * ch, c, lane, wv);
                vec8(vec + kVB * ch, c, lane, bv);
            }
            if (modulate) {
                vec8(vec + kVScale1 * ch, c, lane, s1);
                vec8(vec + kVShift * ch, c, lane, sh);
            }
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                // n = (x − mean)·rstd, two columns per packed op, each rounded as the scalar ops would be
                uint64_t n2 = fmul2(fadd2(f2(v[8 * c + i], v[8 * c + i + 1]), negmean2), rstd2);
                if (affine) n2 = ffma2(n2, f2(wv[i], wv[i + 1]), f2(bv[i], bv[i + 1]));
                float n0, n1;
                uf2(n2, n0, n1);
                uint32_t p = pack_bf16x2(n0, n1);
                if (modulate) {  // round(round(n·round(1 + scale)) + shift)
                    bf2_to_f(p, n0, n1);
                    uf2(fmul2(f2(n0, n1), f2(s1[i], s1[i + 1])), n0, n1);
                    bf2_to_f(pack_bf16x2(n0, n1), n0, n1);
                    uf2(fadd2(f2(n0, n1), f2(sh[i], sh[i + 1])), n0, n1);
                    p = pack_bf16x2(n0, n1);
                }
                w[i >> 1] = p;
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
    for (int i = threadIdx.x; i < ch; i += blockDim.x) vec[vec_pos(i)] = ldb(weight, i);
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
        const uint64_t inv2 = f2(inv, inv);
        __nv_bfloat16* orow = out + (int64_t)rowi * ch;
#pragma unroll
        for (int c = 0; c < kMaxChunks; ++c) {
            if (c >= nch) continue;
            const int col0 = 256 * c + 8 * lane;
            float wv[8];
            vec8(vec, c, lane, wv);
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {  // round(round(x·inv)·w), two columns per packed op
                float y0, y1;
                uf2(fmul2(f2(v[8 * c + i], v[8 * c + i + 1]), inv2), y0, y1);
                bf2_to_f(pack_bf16x2(y0, y1), y0, y1);
                uf2(fmul2(f2(y0, y1), f2(wv[i], wv[i + 1])), y0, y1);
                w[i >> 1] = pack_bf16x2(y0, y1);
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
