// gemm.cu — bf16 GEMM on the 5th-generation tensor cores for the linear layers around the LCSA path:
// out = epilogue(A · Bᵀ + bias), A (M, K) activations and B (N, K) weights (nn.Linear layout), both K-major bf16,
// fp32 accumulation in TMEM. Replaces MLX's Linear (x·Wᵀ + b) of FlashVSR's DiT block (DiT.swift:318-381, 486-549):
// the q/k/v projections of the self-attention, its output projection `sa.o`, the feed-forward pair with GELU(tanh)
// between, and the gated residual adds `tok + gate · f(x)`.
//
// Persistent kernel, one CTA per SM walking 128 × 256 output tiles (consecutive tiles share the A rows, all of B sits
// in L2). (A 256 × 256 tile, two M-128 MMAs per K step and one accumulator pair, measured slower: its epilogue cannot
// overlap the next tile.) Warp roles (320 threads):
//   warp 0      TMA producer: per 64-wide K step one A box (128 × 64) and one B box (256 × 64) into a 4-stage ring;
//   warp 1      TMEM owner + single-thread MMA issuer: 4 × tcgen05.mma (M 128, N 256, K 16) per K step into one of
//               two TMEM accumulators (256 columns each), so the next tile's MMAs run while the epilogue drains;
//   warps 2..9  epilogue, two warps per TMEM lane quarter (a warp reaches only lanes 32·(warp % 4) + 0..31), each of
//               the pair taking 128 of the tile's 256 columns: thread = output row = TMEM lane, 32 columns per
//               tcgen05.ld with the next load in flight while the current chunk is converted, the epilogue arithmetic
//               in fp32 with the reference's bf16 rounding points, 64-byte loads of the residual row and 64-byte
//               stores; the tile's bias and gate columns are staged once in shared memory (one column per thread).
// With K = 1536 a tile's MMAs take ~9 µs, so the epilogue (GELU included) has to fit in that to stay hidden.
// Every wait is bounded (4 s, %globaltimer); on expiry the kernel raises its abort and device timeout words and
// returns, and fvsr_device_check reports FVSR_ETIMEOUT.
#include <math.h>

#include "common.cuh"
#include "sm100.cuh"

namespace fvsr {

__device__ int g_gemm_timeout = 0;

namespace {

using namespace sm100;

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr uint32_t kABytes = kBM * kBK * 2;   // 16 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;   // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 320;
constexpr int kEpiThreads = 256;    // warps 2..9
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, kBN, 0, 0);
// barriers: full[s], empty[s], acc_full[2], acc_empty[2]
constexpr int kBarFull = 0, kBarEmpty = kStages, kBarAccFull = 2 * kStages, kBarAccEmpty = 2 * kStages + 2,
              kNumBars = 2 * kStages + 4;
constexpr uint32_t kOffBar = kStages * kStageBytes;
constexpr uint32_t kOffTmemSlot = kOffBar + 8 * kNumBars;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffCols = kOffAbort + 12;                    // 16-byte aligned: bias[256], gate[256] as fp32
constexpr uint32_t kSmemBytes = 1024 + kOffCols + 2 * kBN * 4;

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// GELU with the tanh approximation, as MLX's GELU(approximation: .tanh): 0.5·x·(1 + tanh(√(2/π)·(x + 0.044715·x³))),
// with tanh(y) = 1 − 2 / (e^(2y) + 1) from the fast exponential (relative error ~1e-6, far below a bf16 step; e^(2y)
// overflowing to +inf gives 1, underflowing to 0 gives −1).
__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    const float y = k0 * (x + k1 * x * x * x);
    const float t = 1.0f - __fdividef(2.0f, __expf(2.0f * y) + 1.0f);
    return 0.5f * x * (1.0f + t);
}

// 32 consecutive output columns of one row: v = the fp32 accumulators, bias / gate = the columns' fp32 values in
// shared memory (broadcast reads), resid / out = the row's bf16 columns in global memory (64 bytes each).
__device__ __forceinline__ void epilogue_chunk(const uint32_t* v, int mode, const float* bias, const float* gate,
                                               const __nv_bfloat16* resid, __nv_bfloat16* out) {
    uint32_t rv[16];
    if (mode == kGemmGatedResidual) {
        const uint4* rp = reinterpret_cast<const uint4*>(resid);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 q = rp[i];
            rv[4 * i] = q.x, rv[4 * i + 1] = q.y, rv[4 * i + 2] = q.z, rv[4 * i + 3] = q.w;
        }
    }
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        float y[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float x = bf16_round(__uint_as_float(v[i + u]) + bias[i + u]);  // the Linear's output
            if (mode == kGemmGelu) x = bf16_round(gelu_tanh(x));
            if (mode == kGemmGatedResidual) {                                // tok + gate · f(x)
                const uint32_t rw = rv[(i + u) >> 1];
                const float rx = __uint_as_float(((i + u) & 1) ? (rw & 0xffff0000u) : (rw << 16));
                x = bf16_round(rx + bf16_round(gate[i + u] * x));
            }
            y[u] = x;
        }
        w[i >> 1] = pack_bf16x2(y[0], y[1]);
    }
    uint4* dst = reinterpret_cast<uint4*>(out);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    griddep_wait_then_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = a.M / kBM, nt = a.N / kBN, kt = a.K / kBK;
    const int tiles = mt * nt;
    volatile uint32_t* abort_word = reinterpret_cast<volatile uint32_t*>(smem + kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);
    auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
    auto wait = [&](int b, uint32_t parity) {
        return mbar_wait(bar(b), parity & 1u, abort_word, &g_gemm_timeout, kWaitLimitNs);
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar(kBarFull + s), 1);
            mbar_init(bar(kBarEmpty + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(kBarAccFull + b), 1);
            mbar_init(bar(kBarAccEmpty + b), kEpiThreads);
        }
        *abort_word = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t it = 0;  // K steps issued by this CTA over all its tiles
            bool ok = true;
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
                const int m0 = (t / nt) * kBM, n0 = (t % nt) * kBN;
                for (int kb = 0; kb < kt; ++kb, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages && !(ok = wait(kBarEmpty + s, (it / kStages - 1)))) break;
                    const uint32_t dst = sbase + (uint32_t)s * kStageBytes;
                    mbar_expect_tx(bar(kBarFull + s), kStageBytes);
                    tma_load_2d(dst, &tmA, kb * kBK, m0, bar(kBarFull + s));
                    tma_load_2d(dst + kABytes, &tmB, kb * kBK, n0, bar(kBarFull + s));
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread) ----------------
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            int lt = 0;  // tiles of this CTA so far
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++lt) {
                const int acc = lt & 1;
                // the epilogue drained this accumulator two tiles ago
                if (lt >= 2 && !(ok = wait(kBarAccEmpty + acc, (uint32_t)((lt >> 1) - 1)))) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)acc * kBN;
                for (int kb = 0; kb < kt; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!(ok = wait(kBarFull + s, it / kStages))) break;
                    tc_fence_after();
                    const uint32_t sa = sbase + (uint32_t)s * kStageBytes;
                    const uint64_t ad = smem_desc(sa, 16, 1024);
                    const uint64_t bd = smem_desc(sa + kABytes, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_ss(d, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    mma_commit(bar(kBarEmpty + s));  // the stage is free once these MMAs have read it
                }
                if (ok) mma_commit(bar(kBarAccFull + acc));
            }
        }
    } else {
        // ---------------- epilogue: thread = row = TMEM lane, half = which 128 columns ----------------
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;
        const int et = threadIdx.x - 64;  // 0..255: the tile column this thread stages
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * (kBN / 2));
        float* bias_s = reinterpret_cast<float*>(smem + kOffCols);
        float* gate_s = bias_s + kBN;
        int lt = 0;
        bool ok = true;
        // Every epilogue warp runs every tile of the CTA, so the two named barriers per tile always meet; after a
        // timed-out wait (ok false, the abort word raised) a warp only keeps those barriers and skips the tile.
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++lt) {
            const int acc = lt & 1;
            const int m0 = (t / nt) * kBM, n0 = (t % nt) * kBN;
            named_barrier_sync(1, kEpiThreads);  // every epilogue thread is done with the previous tile's columns
            bias_s[et] = a.bias ? __bfloat162float(a.bias[n0 + et]) : 0.0f;
            gate_s[et] = a.mode == kGemmGatedResidual ? __bfloat162float(a.gate[n0 + et]) : 0.0f;
            named_barrier_sync(1, kEpiThreads);
            if (ok) ok = __all_sync(0xffffffffu, wait(kBarAccFull + acc, (uint32_t)(lt >> 1)));
            if (!ok) continue;
            tc_fence_after();
            const int j = a.split > 0 ? n0 / a.split : 0;
            const int c0 = (a.split > 0 ? n0 - j * a.split : n0) + half * (kBN / 2);
            const int64_t row = (int64_t)(m0 + r);
            void* const ob = j == 0 ? a.out[0] : (j == 1 ? a.out[1] : a.out[2]);  // no dynamic index into the params
            __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(ob) + row * a.ldo + c0;
            const __nv_bfloat16* rrow = a.resid ? a.resid + row * a.ldo + c0 : nullptr;
            const float* bcol = bias_s + half * (kBN / 2);
            const float* gcol = gate_s + half * (kBN / 2);
            const uint32_t tbase = lane_base + (uint32_t)acc * kBN;
            uint32_t va[32], vb[32];
            tmem_ld32(tbase, va);
            tmem_ld_wait(va);
#pragma unroll
            for (int c = 0; c < kBN / 64; c += 2) {
                tmem_ld32(tbase + 32u * (c + 1), vb);
                epilogue_chunk(va, a.mode, bcol + 32 * c, gcol + 32 * c, rrow ? rrow + 32 * c : nullptr, orow + 32 * c);
                tmem_ld_wait(vb);
                if (c + 2 < kBN / 64) tmem_ld32(tbase + 32u * (c + 2), va);
                epilogue_chunk(vb, a.mode, bcol + 32 * (c + 1), gcol + 32 * (c + 1),
                               rrow ? rrow + 32 * (c + 1) : nullptr, orow + 32 * (c + 1));
                if (c + 2 < kBN / 64) tmem_ld_wait(va);
            }
            tc_fence_before();
            mbar_arrive(bar(kBarAccEmpty + acc));  // the MMA thread may now reuse this accumulator
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

size_t gemm_smem_bytes() { return kSmemBytes; }

cudaError_t launch_gemm_bf16(const GemmArgs& args, const void* A, const void* B, cudaStream_t st) {
    if (args.M % kBM || args.N % kBN || args.K % kBK || args.M <= 0 || args.N <= 0 || args.K <= 0)
        return cudaErrorInvalidValue;
    CUtensorMap ma, mb;
    if (!make_tile_map_box(&ma, A, args.M, args.K, kBM) || !make_tile_map_box(&mb, B, args.N, args.K, kBN))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    int dev = 0, nsm = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const int tiles = (args.M / kBM) * (args.N / kBN);
    const int grid = tiles < nsm ? tiles : nsm;
    return launch_pdl(gemm_bf16_sm100_kernel, dim3(grid), dim3(kThreads), (size_t)kSmemBytes, st, ma, mb, args);
}

cudaError_t read_and_clear_gemm_error(int* flag) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemm_timeout, sizeof(int));
    if (e != cudaSuccess) return e;
    if (v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_gemm_timeout, &zero, sizeof(int));
    }
    *flag = v;
    return e;
}

}  // namespace fvsr
