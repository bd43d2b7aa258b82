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
// HBM-bound in bytes: per window 3·128·C·elt read + 3·128·C·elt written + 128·64·8 rotation-table bytes (read by the
// q and the k CTA) + 2·C·4 pooled written. With few windows (135 at 1920×1152) it is latency-bound instead: 4 warps per
// CTA, each walking its tokens in order.
// Layout: CTA = one window of one tensor (blockIdx.y: 0 q, 1 k, 2 v); warp g walks tokens [32g, 32g + 32) of the
// window in window order, loading the next token's row while it computes the current one; lane l holds channels
// 128·i + 4l + e (e = 0..3) of every head i, so one token's sum of squares is a lane partial — four chains s_e over
// the heads, combined (s0 + s1) + (s2 + s3) — plus a five-step butterfly (every lane ends with the same value:
// a + b = b + a), both rotation pairs of a lane use the lane's two table entries j = 2l, 2l + 1, and a warp moves 256
// contiguous bytes (bf16) of a head per instruction.
#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kPrepThreads = 128;
constexpr int kPrepMaxC = kPrepMaxHeads * kD;

// Applies norm (inv, weights) and rotation (cs, sn) to one lane's four channels of head i; returns the packed output
// and adds the output values to acc. bf16: the weight multiply is one bf16x2 multiply — round(n·w) of the exact
// product, which equals rounding the fp32 product (exact for two bf16 values) — and conversions pack pairs.
template <int DT>
struct LaneOps;

template <>
struct LaneOps<1> {
    using V = uint2;
    static __device__ __forceinline__ void load_w(const void* wt, uint32_t* wsm, int C) {
        for (int c = threadIdx.x; c < C / 2; c += kPrepThreads) wsm[c] = static_cast<const uint32_t*>(wt)[c];
    }
    static __device__ __forceinline__ float2 unpack2(uint32_t w) {  // bf16 pair → (low, high) as fp32
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    }
    static __device__ __forceinline__ uint32_t pack2(float2 f) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    static __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
        const __nv_bfloat162 h = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                         *reinterpret_cast<const __nv_bfloat162*>(&b));
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    // the lane's four channel chains (s0, s1) and (s2, s3), each adding this head's square as fp32x2 operations. The
    // compiler may fuse such a product and sum into one fp32x2 FMA; the square of a bf16 value is exact in fp32, so
    // fused or not the sum rounds the same.
    static __device__ __forceinline__ void sumsq(const V& v, float2& s01, float2& s23) {
        const float2 x01 = unpack2(v.x), x23 = unpack2(v.y);
        s01 = __fadd2_rn(s01, __fmul2_rn(x01, x01));
        s23 = __fadd2_rn(s23, __fmul2_rn(x23, x23));
    }
    // one rotation pair: (re·c − im·s, re·s + im·c) with every product and sum rounded to fp32
    static __device__ __forceinline__ float2 rotate(float2 x, float c, float s) {
        const float2 a = __fmul2_rn(x, make_float2(c, s)), b = __fmul2_rn(x, make_float2(s, c));
        return make_float2(__fsub_rn(a.x, a.y), __fadd_rn(b.x, b.y));
    }
    static __device__ __forceinline__ V apply(V v, bool norm, float inv, const uint32_t* wsm, int wbase, bool rope,
                                              float2 cs, float2 sn, bool pool, float* acc) {
        if (norm) {
            const uint2 w = *reinterpret_cast<const uint2*>(wsm + wbase / 2);
            const float2 iv = make_float2(inv, inv);
            v.x = mul2(pack2(__fmul2_rn(unpack2(v.x), iv)), w.x);
            v.y = mul2(pack2(__fmul2_rn(unpack2(v.y), iv)), w.y);
        }
        if (rope) {
            v.x = pack2(rotate(unpack2(v.x), cs.x, sn.x));
            v.y = pack2(rotate(unpack2(v.y), cs.y, sn.y));
        }
        if (pool) {
            float2* a2 = reinterpret_cast<float2*>(acc);
            a2[0] = __fadd2_rn(a2[0], unpack2(v.x));
            a2[1] = __fadd2_rn(a2[1], unpack2(v.y));
        }
        return v;
    }
};

template <>
struct LaneOps<0> {
    using V = float4;
    static __device__ __forceinline__ void load_w(const void* wt, uint32_t* wsm, int C) {
        for (int c = threadIdx.x; c < C; c += kPrepThreads) wsm[c] = static_cast<const uint32_t*>(wt)[c];
    }
    // fp32 squares are not exact: scalar multiply and add, which are never fused
    static __device__ __forceinline__ void sumsq(const V& v, float2& s01, float2& s23) {
        s01.x = __fadd_rn(s01.x, __fmul_rn(v.x, v.x));
        s01.y = __fadd_rn(s01.y, __fmul_rn(v.y, v.y));
        s23.x = __fadd_rn(s23.x, __fmul_rn(v.z, v.z));
        s23.y = __fadd_rn(s23.y, __fmul_rn(v.w, v.w));
    }
    static __device__ __forceinline__ V apply(V v, bool norm, float inv, const uint32_t* wsm, int wbase, bool rope,
                                              float2 cs, float2 sn, bool pool, float* acc) {
        if (norm) {
            const float4 w = *reinterpret_cast<const float4*>(wsm + wbase);
            v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
        }
        if (rope) {
            const float r0 = v.x, i0 = v.y, r1 = v.z, i1 = v.w;
            v.x = __fsub_rn(__fmul_rn(r0, cs.x), __fmul_rn(i0, sn.x));
            v.y = __fadd_rn(__fmul_rn(r0, sn.x), __fmul_rn(i0, cs.x));
            v.z = __fsub_rn(__fmul_rn(r1, cs.y), __fmul_rn(i1, sn.y));
            v.w = __fadd_rn(__fmul_rn(r1, sn.y), __fmul_rn(i1, cs.y));
        }
        if (pool) {
            acc[0] = __fadd_rn(acc[0], v.x);
            acc[1] = __fadd_rn(acc[1], v.y);
            acc[2] = __fadd_rn(acc[2], v.z);
            acc[3] = __fadd_rn(acc[3], v.w);
        }
        return v;
    }
};

template <int DT, int NH>
__global__ void __launch_bounds__(kPrepThreads) prepare_kernel(const __grid_constant__ PrepArgs a) {
    using Ops = LaneOps<DT>;
    using V = typename Ops::V;
    __shared__ float part[4][kPrepMaxC];
    __shared__ __align__(16) uint32_t wsm[kPrepMaxC];
    griddep_wait_then_release();
    if (a.zero) {
        const size_t nb = (size_t)gridDim.x * gridDim.y, bid = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
        for (size_t w = bid * kPrepThreads + threadIdx.x; w < a.zero_words; w += nb * kPrepThreads) a.zero[w] = 0;
    }
    const int role = blockIdx.y, win = blockIdx.x;
    const int heads = a.heads, C = heads * kD, cv = C / 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const void* wt = role < 2 ? a.norm_w[role] : nullptr;
    const bool norm = wt != nullptr;
    const bool rope = role < 2 && a.cosv != nullptr;
    float* pooled = role < 2 ? a.pooled[role] : nullptr;
    if (norm) {  // CTA-uniform
        Ops::load_w(wt, wsm, C);
        __syncthreads();
    }
    const int64_t blk = role == 0 ? (int64_t)win : (int64_t)kv_phys_block(a.kv_pages, win);
    const V* src = static_cast<const V*>(a.x[role]) + lane;
    V* dst = static_cast<V*>(role == 0 ? a.q_out : a.kv_out[role - 1]) + blk * kBlock * cv + lane;
    float acc[4 * NH];
#pragma unroll
    for (int i = 0; i < 4 * NH; ++i) acc[i] = 0.0f;

    // software pipeline: the next token's row and table entries load while this token is computed
    V nxt[NH];
    float2 ncs = make_float2(1.0f, 1.0f), nsn = make_float2(0.0f, 0.0f);
    auto load = [&](int t) {
        const int64_t tok = token_row(a.bh, a.bw, win, 32 * warp + t);
#pragma unroll
        for (int i = 0; i < NH; ++i)
            if (i < heads) nxt[i] = __ldcs(src + tok * cv + 32 * i);
        if (rope) {
            ncs = __ldg(reinterpret_cast<const float2*>(a.cosv + tok * 64) + lane);
            nsn = __ldg(reinterpret_cast<const float2*>(a.sinv + tok * 64) + lane);
        }
    };
    load(0);
#pragma unroll 1
    for (int t = 0; t < 32; ++t) {
        V cur[NH];
#pragma unroll
        for (int i = 0; i < NH; ++i) cur[i] = nxt[i];
        const float2 cs = ncs, sn = nsn;
        if (t + 1 < 32) load(t + 1);
        float inv = 1.0f;
        if (norm) {
            float2 s01 = make_float2(0.0f, 0.0f), s23 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < NH; ++i)
                if (i < heads) Ops::sumsq(cur[i], s01, s23);
            float ss = __fadd_rn(__fadd_rn(s01.x, s01.y), __fadd_rn(s23.x, s23.y));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
            inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)C), a.eps));
        }
        V* drow = dst + (int64_t)(32 * warp + t) * cv;
#pragma unroll
        for (int i = 0; i < NH; ++i)
            if (i < heads)
                drow[32 * i] = Ops::apply(cur[i], norm, inv, wsm, kD * i + 4 * lane, rope, cs, sn, pooled != nullptr,
                                          acc + 4 * i);
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
