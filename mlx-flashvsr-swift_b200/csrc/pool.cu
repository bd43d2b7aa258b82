// pool.cu — fp32 block means of window-ordered tokens (DiT.swift:161-162), optionally fused with the in-place copy
// of the same rows into a KV-cache page (the cache append of DiT.swift:508-511 reads each key row once).
//
// HBM-bound: algorithmic bytes = nblocks·128·C·elt read (+ the same written when copying) + nblocks·C·4 written.
// The inputs are read with evict-first (streaming) loads, so the pass does not push the pooled rows it writes — which
// the selection reads next — out of L2. Layout: one CTA covers one 128-token block × 512 channels; 4 token groups × 64 channel lanes, 8 channels per lane
// (one 128-bit load per token for bf16), so a warp reads 512 contiguous bytes of a token row per load. With at most
// 256 channels (the one or two heads of a sharded rank) the 64 lanes are split into bpc = 64 / lanes groups that
// pool bpc consecutive blocks at once, each block with exactly the arithmetic of the one-block layout.
#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kPoolLanes = 64;               // channel lanes per CTA
constexpr int kPoolChannels = kPoolLanes * 8;  // 512 channels per CTA

// Blocks [0, n1) pool x into out (and copy to copy_dst); blocks [n1, gridDim.y) pool x2 into out2, so the query and
// key pools of one selection share a launch.
template <int DT>
__global__ void __launch_bounds__(256) pool_kernel(const void* __restrict__ x, int channels, float* __restrict__ out,
                                                   void* __restrict__ copy_dst, int n1, const void* __restrict__ x2,
                                                   float* __restrict__ out2, uint32_t* __restrict__ zero,
                                                   size_t zero_words, int lanes, int nblocks) {
    __shared__ float part[4][kPoolChannels];
    griddep_wait_then_release();
    if (zero) {
        const size_t nb = (size_t)gridDim.x * gridDim.y, bid = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
        for (size_t w = bid * 256 + threadIdx.x; w < zero_words; w += nb * 256) zero[w] = 0;
    }
    const int lane = threadIdx.x & (kPoolLanes - 1);
    const int g = threadIdx.x / kPoolLanes;  // token group: tokens [32g, 32g + 32)
    const int sub = lane / lanes, cl = lane % lanes;  // block within the CTA, channel lane within the block
    const int c0 = blockIdx.x * kPoolChannels + cl * 8;
    int64_t b = (int64_t)blockIdx.y * (kPoolLanes / lanes) + sub;
    const bool live = b < nblocks;
    if (b >= n1) {
        b -= n1;
        x = x2;
        out = out2;
        copy_dst = nullptr;
    }
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    if (live && c0 < channels) {
        // 8 tokens per batch: all 8 loads are issued before their sums (which stay in token order)
        for (int t0 = 32 * g; t0 < 32 * g + 32; t0 += 8) {
            if (DT == 1) {
                uint4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    v[u] = __ldcs(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) +
                                                               (b * kBlock + t0 + u) * (int64_t)channels + c0));
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (copy_dst)
                        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(copy_dst) +
                                                  (b * kBlock + t0 + u) * (int64_t)channels + c0) = v[u];
                    const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        acc[2 * i] = __fadd_rn(acc[2 * i], bf16_bits_to_float(w[i] & 0xFFFFu));
                        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_bits_to_float(w[i] >> 16));
                    }
                }
            } else {
                float4 v[8][2];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(x) +
                                                                        (b * kBlock + t0 + u) * (int64_t)channels + c0);
                    v[u][0] = __ldcs(src);
                    v[u][1] = __ldcs(src + 1);
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (copy_dst) {
                        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(copy_dst) +
                                                                (b * kBlock + t0 + u) * (int64_t)channels + c0);
                        dst[0] = v[u][0];
                        dst[1] = v[u][1];
                    }
                    const float w[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                                        v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], w[i]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) part[g][lane * 8 + i] = acc[i];
    __syncthreads();
    if (g == 0 && live && c0 < channels) {
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = lane * 8 + i;
            const float s = __fadd_rn(__fadd_rn(part[0][c], part[1][c]), __fadd_rn(part[2][c], part[3][c]));
            r[i] = __fmul_rn(s, 0.0078125f);
        }
        float4* o = reinterpret_cast<float4*>(out + b * channels + c0);
        o[0] = make_float4(r[0], r[1], r[2], r[3]);
        o[1] = make_float4(r[4], r[5], r[6], r[7]);
    }
}

// The cache append of DiT.swift:508-511 in one launch: new key block b (of nblocks = slices·s) is pooled into the pooled
// key arena and copied, with value block b, into arena block dst.page_block[b / s] + b % s. The pooling arithmetic is
// the one above (token order within each group of 32, groups combined (g0+g1)+(g2+g3)), so the pooled keys are
// bit-identical to pool_kernel's. Key and value rows of a batch of U tokens are all loaded before any is stored.
// Algorithmic bytes: 2·nblocks·128·C·elt read + the same written + nblocks·C·4 written.
template <int DT>
__global__ void __launch_bounds__(256, 4) append_kernel(const void* __restrict__ k_new, const void* __restrict__ v_new,
                                                     int channels, int nblocks, const __grid_constant__ KvPages dst,
                                                     void* __restrict__ k_arena,
                                                     void* __restrict__ v_arena, float* __restrict__ pk_arena,
                                                     int lanes) {
    constexpr int U = DT == 1 ? 4 : 2;               // tokens per batch (64 registers: 4 CTAs per SM)
    constexpr int W = DT == 1 ? 1 : 2;               // uint4 words per 8 channels
    __shared__ float part[4][kPoolChannels];
    griddep_wait_then_release();
    const int lane = threadIdx.x & (kPoolLanes - 1);
    const int g = threadIdx.x / kPoolLanes;
    const int sub = lane / lanes, cl = lane % lanes;
    const int c0 = blockIdx.x * kPoolChannels + cl * 8;
    const int64_t b = (int64_t)blockIdx.y * (kPoolLanes / lanes) + sub;
    const bool live = b < nblocks && c0 < channels;
    const int64_t pb = live ? (int64_t)dst.page_block[b / dst.s] + b % dst.s : 0;  // arena block
    const int row_words = channels * (DT == 1 ? 2 : 4) / 16;                       // uint4 words per token row
    const int64_t cw = (int64_t)c0 * (DT == 1 ? 2 : 4) / 16;
    const int64_t first = (b * kBlock + 32 * g) * row_words + cw;            // this thread's first token row
    const int64_t first_dst = (pb * kBlock + 32 * g) * row_words + cw;
    const uint4* ks = static_cast<const uint4*>(k_new) + first;
    const uint4* vs = static_cast<const uint4*>(v_new) + first;
    uint4* kd = static_cast<uint4*>(k_arena) + first_dst;
    uint4* vd = static_cast<uint4*>(v_arena) + first_dst;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    if (live) {
#pragma unroll 1
        for (int t = 0; t < 32; t += U) {
            uint4 kv[U][W], vv[U][W];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int w = 0; w < W; ++w) {
                    kv[u][w] = __ldcs(ks + u * row_words + w);
                    vv[u][w] = __ldcs(vs + u * row_words + w);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
#pragma unroll
                for (int w = 0; w < W; ++w) {
                    kd[u * row_words + w] = kv[u][w];
                    vd[u * row_words + w] = vv[u][w];
                }
                if constexpr (DT == 1) {
                    const uint32_t x[4] = {kv[u][0].x, kv[u][0].y, kv[u][0].z, kv[u][0].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        acc[2 * i] = __fadd_rn(acc[2 * i], bf16_bits_to_float(x[i] & 0xFFFFu));
                        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_bits_to_float(x[i] >> 16));
                    }
                } else {
                    const uint32_t x[8] = {kv[u][0].x, kv[u][0].y, kv[u][0].z, kv[u][0].w,
                                           kv[u][W - 1].x, kv[u][W - 1].y, kv[u][W - 1].z, kv[u][W - 1].w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __uint_as_float(x[i]));
                }
            }
            ks += U * row_words;
            vs += U * row_words;
            kd += U * row_words;
            vd += U * row_words;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) part[g][lane * 8 + i] = acc[i];
    __syncthreads();
    if (g == 0 && live) {
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = lane * 8 + i;
            const float sum = __fadd_rn(__fadd_rn(part[0][c], part[1][c]), __fadd_rn(part[2][c], part[3][c]));
            r[i] = __fmul_rn(sum, 0.0078125f);
        }
        float4* o = reinterpret_cast<float4*>(pk_arena + pb * channels + c0);
        o[0] = make_float4(r[0], r[1], r[2], r[3]);
        o[1] = make_float4(r[4], r[5], r[6], r[7]);
    }
}

}  // namespace

cudaError_t launch_append(const void* k_new, const void* v_new, int dtype, int64_t nblocks, int channels,
                          const KvPages& dst, void* k_arena, void* v_arena, float* pk_arena, cudaStream_t st) {
    if (nblocks == 0) return cudaSuccess;
    int lanes = 1;
    while (lanes < kPoolLanes && lanes * 8 < channels) lanes <<= 1;
    const int bpc = kPoolLanes / lanes;
    dim3 grid((channels + kPoolChannels - 1) / kPoolChannels, (unsigned)((nblocks + bpc - 1) / bpc));
    if (dtype == 1)
        return launch_pdl(append_kernel<1>, grid, dim3(256), 0, st, k_new, v_new, channels, (int)nblocks, dst, k_arena,
                          v_arena, pk_arena, lanes);
    return launch_pdl(append_kernel<0>, grid, dim3(256), 0, st, k_new, v_new, channels, (int)nblocks, dst, k_arena,
                      v_arena, pk_arena, lanes);
}

cudaError_t launch_pool(const void* x, int dtype, int64_t nblocks, int channels, float* out, void* copy_dst,
                        cudaStream_t st) {
    return launch_pool2(x, nblocks, out, copy_dst, nullptr, 0, nullptr, dtype, channels, st);
}

cudaError_t launch_pool2(const void* x1, int64_t n1, float* out1, void* copy_dst, const void* x2, int64_t n2,
                         float* out2, int dtype, int channels, cudaStream_t st, uint32_t* zero, size_t zero_words) {
    if (n1 + n2 == 0) return cudaSuccess;
    // channel lanes one block needs (a power of two ≤ 64); the rest of the 64 pool further blocks
    int lanes = 1;
    while (lanes < kPoolLanes && lanes * 8 < channels) lanes <<= 1;
    const int bpc = kPoolLanes / lanes;
    const int64_t nb = n1 + n2;
    dim3 grid((channels + kPoolChannels - 1) / kPoolChannels, (unsigned)((nb + bpc - 1) / bpc));
    if (dtype == 1)
        return launch_pdl(pool_kernel<1>, grid, dim3(256), 0, st, x1, channels, out1, copy_dst, (int)n1, x2, out2, zero,
                          zero_words, lanes, (int)nb);
    return launch_pdl(pool_kernel<0>, grid, dim3(256), 0, st, x1, channels, out1, copy_dst, (int)n1, x2, out2, zero,
                      zero_words, lanes, (int)nb);
}

}  // namespace fvsr
