// gemm.cu — bf16 GEMM on the 5th-generation tensor cores for the linear layers around the LCSA path:
// out = epilogue(A · Bᵀ + bias), A (M, K) activations and B (N, K) weights (nn.Linear layout), both K-major bf16,
// fp32 accumulation in TMEM. Replaces MLX's Linear (x·Wᵀ + b) of FlashVSR's DiT block (DiT.swift:318-381, 486-549):
// the q/k/v projections of the self-attention, its output projection `sa.o`, the feed-forward pair with GELU(tanh)
// between, and the gated residual adds `tok + gate · f(x)`.
//
// Persistent kernel over CTA pairs: a cluster of two CTAs (one TPC) walks 256 × 256 output tiles (consecutive tiles of
// a pair share the A rows; B sits in L2) with tcgen05 cta_group::2 MMAs (M 256, N 256, K 16). CTA r of the pair loads
// rows [m0 + 128·r, +128) of A and rows [n0 + 128·r, +128) of B per 64-wide K step (32 KB per stage, 6 stages), the
// even CTA's single MMA thread drives both tensor cores, and each CTA's TMEM receives its own 128 rows × 256 columns.
// Against one CTA per 128 × 256 tile this halves B per SM: 8 KB of shared-memory operand reads and 32 KB of L2 → SM
// traffic per 128 × 256 × 64 of work instead of 12 KB and 48 KB (measured: K = 8960 1209 → 1354 TFLOP/s).
// Warp roles (320 threads per CTA):
//   warp 0      TMA producer of this CTA's halves;
//   warp 1      TMEM owner (pair allocation, 512 columns = two accumulators) and, in the even CTA, the MMA issuer:
//               the next tile's MMAs run while the epilogue drains the other accumulator;
//   warps 2..9  epilogue, two warps per TMEM lane quarter (a warp reaches only lanes 32·(warp % 4) + 0..31), each of
//               the pair taking 128 of the tile's 256 columns: thread = output row = TMEM lane, 32 columns per
//               tcgen05.ld with the next load in flight while the current chunk is converted, the epilogue arithmetic
//               in fp32 with the reference's bf16 rounding points, 64-byte loads of the residual row and 64-byte
//               stores; the tile's bias and gate columns are staged once in shared memory (one column per thread).
// Synchronisation: stage s is full when the even CTA's full[s] has both CTAs' 64 KB (the odd CTA's loads signal it
// through its cluster address; only the even producer arrives, with the expected byte count); the MMA commits free
// stage s in both CTAs (empty[s] of each) and announce an accumulator in both (acc_full of each); each epilogue warp of
// either CTA arrives once on the even CTA's acc_empty (16 arrivals per tile). Both CTAs walk the same tiles and meet at
// cluster barriers after set-up and before TMEM is freed. Each CTA loads only its own operands, with plain tile loads.
// Every wait is bounded (4 s, %globaltimer); on expiry the kernel raises its abort and device timeout words and skips
// the rest of its work, and fvsr_device_check reports FVSR_ETIMEOUT.
#include <math.h>

#include "common.cuh"
#include "sm100.cuh"

namespace fvsr {

__device__ int g_gemm_timeout = 0;

namespace {

using namespace sm100;

constexpr int kBM = 256, kBN = 256, kBK = 64, kStages = 6;   // pair tile M × N, K step, ring depth
constexpr uint32_t kHalfBytes = 128 * kBK * 2;                 // 16 KB: one CTA's A rows or B rows per K step
constexpr uint32_t kStageBytes = 2 * kHalfBytes;               // A then B
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8, kEpiThreads = 32 * kEpiWarps;     // warps 2..9
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, kBN, 0, 0);
// barriers: full[s], empty[s], acc_full[2], acc_empty[2]
constexpr int kBarFull = 0, kBarEmpty = kStages, kBarAccFull = 2 * kStages, kBarAccEmpty = 2 * kStages + 2,
              kNumBars = 2 * kStages + 4;
constexpr uint32_t kOffBar = kStages * kStageBytes;
constexpr uint32_t kOffTmemSlot = kOffBar + 8 * kNumBars;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffCols = (kOffAbort + 4 + 15) & ~15u;     // bias[256], gate[256] as fp32
constexpr uint32_t kSmemBytes = 1024 + kOffCols + 2 * kBN * 4;
static_assert(kSmemBytes <= 232448, "shared memory");

// GELU with the tanh approximation, as MLX's GELU(approximation: .tanh): 0.5·x·(1 + tanh(y)), y = √(2/π)·(x +
// 0.044715·x³), evaluated through 0.5·(1 + tanh(y)) = 1 / (1 + e^(−2y)) as x / (1 + 2^z), z = x·(c0 + c1·x²) with
// c0 = −2·√(2/π)·log2(e), c1 = 0.044715·c0 (relative error ~1e-6, far below a bf16 step; 2^z overflowing to +inf gives
// 0, underflowing to 0 gives x). Two outputs per call, packed arithmetic except the two exponentials and reciprocals.
__device__ __forceinline__ void gelu_tanh2(float& x0, float& x1) {
    constexpr float c0 = -2.0f * 0.7978845608028654f * 1.4426950408889634f, c1 = 0.044715f * c0;
    const uint64_t x = f2(x0, x1);
    float z0, z1;
    uf2(fmul2(x, ffma2(fmul2(x, x), f2(c1, c1), f2(c0, c0))), z0, z1);
    float d0, d1;
    uf2(fadd2(f2(ex2_approx(z0), ex2_approx(z1)), f2(1.0f, 1.0f)), d0, d1);
    uf2(fmul2(x, f2(rcp_approx(d0), rcp_approx(d1))), x0, x1);
}

// 32 consecutive output columns of one row: v = the fp32 accumulators, bias / gate = the columns' fp32 values in
// shared memory (broadcast reads), rv = the residual's bf16 pairs (gated residual only), out = the row's bf16 columns
// in global memory (64 bytes). Rounding
// points as the reference's ops: Linear = round(acc + bias); GELU = round(gelu(Linear)); gated residual =
// round(resid + round(gate · Linear)).
// The 32 bf16 residual values of a chunk (64 bytes of one row), loaded ahead of their use.
__device__ __forceinline__ void load_resid(const __nv_bfloat16* resid, uint32_t* rv) {
    const uint4* rp = reinterpret_cast<const uint4*>(resid);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 q = rp[i];
        rv[4 * i] = q.x, rv[4 * i + 1] = q.y, rv[4 * i + 2] = q.z, rv[4 * i + 3] = q.w;
    }
}

template <int kMode>
__device__ __forceinline__ void epilogue_chunk(const uint32_t* v, const float* bias, const float* gate,
                                               const uint32_t* rv, __nv_bfloat16* out) {
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        const float4 b = *reinterpret_cast<const float4*>(bias + i);
        float x[4];
        uf2(fadd2(f2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), f2(b.x, b.y)), x[0], x[1]);
        uf2(fadd2(f2(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3])), f2(b.z, b.w)), x[2], x[3]);
#pragma unroll
        for (int u = 0; u < 4; u += 2) {
            uint32_t p = pack_bf16x2(x[u], x[u + 1]);  // the Linear's output
            if (kMode == kGemmGelu) {
                float y0, y1;
                bf2_to_f(p, y0, y1);
                gelu_tanh2(y0, y1);
                p = pack_bf16x2(y0, y1);
            } else if (kMode == kGemmGatedResidual) {  // tok + gate · f(x)
                float y0, y1, r0, r1, g0, g1;
                bf2_to_f(p, y0, y1);
                const float2 g = *reinterpret_cast<const float2*>(gate + i + u);
                uf2(fmul2(f2(g.x, g.y), f2(y0, y1)), g0, g1);
                bf2_to_f(pack_bf16x2(g0, g1), g0, g1);
                bf2_to_f(rv[(i + u) >> 1], r0, r1);
                uf2(fadd2(f2(r0, r1), f2(g0, g1)), y0, y1);
                p = pack_bf16x2(y0, y1);
            }
            w[(i + u) >> 1] = p;
        }
    }
    uint4* dst = reinterpret_cast<uint4*>(out);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

template <int kMode>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_bf16_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    griddep_wait_then_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const int mt = (a.M + kBM - 1) / kBM, nt = a.N / kBN, kt = a.K / kBK;
    const int tiles = mt * nt;
    volatile uint32_t* abort_word = reinterpret_cast<volatile uint32_t*>(smem + kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);
    auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
    auto wait = [&](int b, uint32_t parity) {
        return mbar_wait(bar(b), parity & 1u, abort_word, &g_gemm_timeout, kWaitLimitNs);
    };
    if (threadIdx.x == 0) {
        for (int st = 0; st < kStages; ++st) {
            mbar_init(bar(kBarFull + st), 1);
            mbar_init(bar(kBarEmpty + st), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(kBarAccFull + b), 1);
            mbar_init(bar(kBarAccEmpty + b), 2 * kEpiWarps);
        }
        *abort_word = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers are initialised and their TMEM allocated before any remote signal
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer of this CTA's halves ----------------
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = pair; ok && t < tiles; t += npairs) {
                int m0 = (t / nt) * kBM + 128 * (int)rank;
                const int n0 = (t % nt) * kBN + 128 * (int)rank;
                if (m0 >= a.M) m0 -= 128;  // past M (odd CTA, last tile row): reload the even rows, stored by no one
                for (int kb = 0; kb < kt; ++kb, ++it) {
                    const int st = (int)(it % kStages);
                    if (it >= kStages && !(ok = wait(kBarEmpty + st, it / kStages - 1))) break;
                    const uint32_t dst = sbase + (uint32_t)st * kStageBytes;
                    const uint32_t full0 = mapa_shared(bar(kBarFull + st), 0);
                    if (rank == 0) mbar_expect_tx(bar(kBarFull + st), 2 * kStageBytes);
                    tma_load_2d_pair(dst, &tmA, kb * kBK, m0, full0);
                    tma_load_2d_pair(dst + kHalfBytes, &tmB, kb * kBK, n0, full0);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: one thread of the even CTA ----------------
        if (lane == 0 && rank == 0) {
            uint32_t it = 0;
            bool ok = true;
            int lt = 0;
            for (int t = pair; ok && t < tiles; t += npairs, ++lt) {
                const int acc = lt & 1;
                if (lt >= 2 && !(ok = wait(kBarAccEmpty + acc, (uint32_t)((lt >> 1) - 1)))) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)acc * kBN;
                for (int kb = 0; kb < kt; ++kb, ++it) {
                    const int st = (int)(it % kStages);
                    if (!(ok = wait(kBarFull + st, it / kStages))) break;
                    tc_fence_after();
                    const uint32_t sa = sbase + (uint32_t)st * kStageBytes;
                    const uint64_t ad = smem_desc(sa, 16, 1024);
                    const uint64_t bd = smem_desc(sa + kHalfBytes, 16, 1024);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_ss_pair(d, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), kIdesc,
                                    (kb > 0 || kk > 0) ? 1u : 0u);
                    mma_commit_pair(bar(kBarEmpty + st));
                    mma_commit_pair(mapa_shared(bar(kBarEmpty + st), 1));
                }
                if (ok) {
                    mma_commit_pair(bar(kBarAccFull + acc));
                    mma_commit_pair(mapa_shared(bar(kBarAccFull + acc), 1));
                }
            }
        }
    } else {
        // ---------------- epilogue: this CTA's 128 rows; thread = row = TMEM lane, half = which 128 columns ----------------
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;
        const int et = threadIdx.x - 64;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * (kBN / 2));
        float* bias_s = reinterpret_cast<float*>(smem + kOffCols);
        float* gate_s = bias_s + kBN;
        const uint32_t acc_empty0 = mapa_shared(bar(kBarAccEmpty), 0);
        int lt = 0;
        bool ok = true;
        for (int t = pair; t < tiles; t += npairs, ++lt) {
            const int acc = lt & 1;
            const int m0 = (t / nt) * kBM + 128 * (int)rank, n0 = (t % nt) * kBN;
            named_barrier_sync(1, kEpiThreads);
            bias_s[et] = a.bias ? __bfloat162float(a.bias[n0 + et]) : 0.0f;
            gate_s[et] = kMode == kGemmGatedResidual ? __bfloat162float(a.gate[n0 + et]) : 0.0f;
            named_barrier_sync(1, kEpiThreads);
            const bool live = m0 < a.M;  // the odd CTA of the last row of tiles may lie wholly past M
            const int j = a.split > 0 ? n0 / a.split : 0;
            const int c0 = (a.split > 0 ? n0 - j * a.split : n0) + half * (kBN / 2);
            const int64_t row = (int64_t)(m0 + r);
            const __nv_bfloat16* rrow = a.resid ? a.resid + row * a.ldo + c0 : nullptr;
            uint32_t ra[16], rb[16];
            if (kMode == kGemmGatedResidual && ok && live) load_resid(rrow, ra);  // in flight during the wait
            if (ok) ok = __all_sync(0xffffffffu, wait(kBarAccFull + acc, (uint32_t)(lt >> 1)));
            if (!ok) continue;
            tc_fence_after();
            if (live) {
                void* const ob = j == 0 ? a.out[0] : (j == 1 ? a.out[1] : a.out[2]);
                __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(ob) + row * a.ldo + c0;
                const float* bcol = bias_s + half * (kBN / 2);
                const float* gcol = gate_s + half * (kBN / 2);
                const uint32_t tbase = lane_base + (uint32_t)acc * kBN;
                uint32_t va[32], vb[32];
                tmem_ld32(tbase, va);
                tmem_ld_wait(va);
#pragma unroll
                for (int c = 0; c < kBN / 64; c += 2) {
                    tmem_ld32(tbase + 32u * (c + 1), vb);
                    if (kMode == kGemmGatedResidual) load_resid(rrow + 32 * (c + 1), rb);
                    epilogue_chunk<kMode>(va, bcol + 32 * c, gcol + 32 * c, ra, orow + 32 * c);
                    tmem_ld_wait(vb);
                    if (c + 2 < kBN / 64) {
                        tmem_ld32(tbase + 32u * (c + 2), va);
                        if (kMode == kGemmGatedResidual) load_resid(rrow + 32 * (c + 2), ra);
                    }
                    epilogue_chunk<kMode>(vb, bcol + 32 * (c + 1), gcol + 32 * (c + 1), rb, orow + 32 * (c + 1));
                    if (c + 2 < kBN / 64) tmem_ld_wait(va);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8u * (uint32_t)acc);  // the even CTA's acc_empty[acc]
        }
    }
    tc_fence_before();
    cluster_sync();  // no signal to the other CTA and no MMA on this CTA's shared memory is still in flight
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

template <int kMode>
cudaError_t launch_gemm_mode(const GemmArgs& args, const CUtensorMap& ma, const CUtensorMap& mb, cudaStream_t st) {
    auto kernel = gemm_bf16_sm100_kernel<kMode>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    int dev = 0, nsm = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    const int tiles = ((args.M + kBM - 1) / kBM) * (args.N / kBN);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    int resident = 0;  // pairs that fit on the GPU at once (one CTA per SM, both SMs of a pair on one TPC)
    cfg.gridDim = dim3(nsm & ~1);
    if (cudaOccupancyMaxActiveClusters(&resident, kernel, &cfg) != cudaSuccess || resident < 1) resident = nsm / 2;
    const int pairs = tiles < resident ? tiles : resident;
    cfg.gridDim = dim3(2 * pairs);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, ma, mb, args);
}

}  // namespace

size_t gemm_smem_bytes() { return kSmemBytes; }

cudaError_t launch_gemm_bf16(const GemmArgs& args, const void* A, const void* B, cudaStream_t st) {
    if (args.M % 128 || args.N % kBN || args.K % kBK || args.M <= 0 || args.N <= 0 || args.K <= 0)
        return cudaErrorInvalidValue;
    CUtensorMap ma, mb;
    if (!make_tile_map_box(&ma, A, args.M, args.K, 128) || !make_tile_map_box(&mb, B, args.N, args.K, 128))
        return cudaErrorInvalidValue;
    switch (args.mode) {
        case kGemmPlain: return launch_gemm_mode<kGemmPlain>(args, ma, mb, st);
        case kGemmGelu: return launch_gemm_mode<kGemmGelu>(args, ma, mb, st);
        case kGemmGatedResidual: return launch_gemm_mode<kGemmGatedResidual>(args, ma, mb, st);
        default: return cudaErrorInvalidValue;
    }
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
