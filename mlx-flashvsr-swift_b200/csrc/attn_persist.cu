// attn_persist.cu — persistent bf16 block-sparse attention over an equal-work schedule (schedule.cu).
//
// Same per-item semantics as attn_sm100.cu (SparseAttention.swift:17-153: one query block's online softmax over its
// selected key blocks), but one CTA per SM walks a fixed share of the range's kept key blocks as a sequence of
// segments (item, first list position, length, partial slot): the pipelines run on across segment boundaries, so the
// next item's Q and first K/V tiles load while the current one finishes, and every CTA does the same number of key
// blocks. Segment σ (counted within the CTA) uses Q slot σ%2; global block j (over the CTA's segments) uses K/V slot
// j%2 and S/P buffer j%3, so one phase sequence per barrier covers the whole walk. O is single: a segment's first
// PV waits until the previous segment's epilogue has read it (its S MMAs already run ahead).
//
// Warp roles (320 threads): warp 0 TMA producer (Q of each segment, then its K and V tiles), warp 1 TMEM owner and
// single-thread MMA issuer (S_j = Q·K_jᵀ two blocks ahead of O += P_j·V_j), warps 2..9 two softmax sets of four warps
// (set st takes the blocks j ≡ st mod 2; thread = query row = TMEM lane), which also run each segment's epilogue:
// combine the two sets' row sums, read O, write the bf16 rows (or, for a piece of a cut item, fp32 O and (m, l)).
// TMEM (512 columns): O [0,128), S0/P0 [128,256), S1/P1 [256,384), S2/P2 [384,512).
// Shared memory: Q 2 × 32 KB, K 2 × 32 KB, V 2 × 32 KB (128-byte swizzled, two 128 × 64 boxes each).
// Every wait is bounded (4 s); on expiry the kernel raises the device timeout word that fvsr_device_check reports.
#include "common.cuh"
#include "sm100.cuh"

namespace fvsr {

// Raised when a wait of this kernel gives up (its own word: device variables are per translation unit here).
__device__ int g_fvsr_timeout_persist = 0;

namespace {

using namespace sm100;

constexpr uint32_t kTile = kBlock * kD * 2;  // 32 KB bf16 tile
constexpr uint32_t kBox = kTile / 2;
constexpr int kThreadsP = 320;
constexpr uint64_t kLimitNs = 4000000000ull;
constexpr float kThreshold = 8.0f;  // lazy rescaling (log2 units), as in attn_sm100.cu
constexpr uint32_t kColO = 0, kColS = 128, kCols = 512;
constexpr uint32_t kIdS = idesc_bf16_f32(128, 128, 0, 0);   // A = Q, B = K (K-major shared memory)
constexpr uint32_t kIdPV = idesc_bf16_f32(128, 128, 0, 1);  // A = P (TMEM), B = V (MN-major shared memory)

constexpr uint32_t kOffQ = 0, kOffK = 2 * kTile, kOffV = 4 * kTile, kOffBar = 6 * kTile;
// barriers (index = slot, buffer or parity): Q full/empty [2], K full [2], V full [2], S full [3], P full [3],
// PV done [2], max hand-off [2], O drained, segment-end exchange
enum { bQF = 0, bQE = 2, bKF = 4, bVF = 6, bSF = 8, bPF = 11, bPV = 14, bM = 16, bOE = 18, bFin = 19, kNumBars = 20 };
constexpr uint32_t kOffTmem = kOffBar + 8 * kNumBars;
constexpr uint32_t kOffAbort = kOffTmem + 4;
constexpr uint32_t kOffMx = (kOffAbort + 4 + 15) & ~15u;  // running max hand-off [2][128] f32
constexpr uint32_t kOffFin = kOffMx + 2 * 128 * 4;        // (l, m) per segment parity, set, row: [2][2][2][128] f32
constexpr uint32_t kOffRows = kOffFin + 2 * 2 * 2 * 128 * 4;  // K/V tile row of each block of the walk
constexpr int kRowsCap = 6144;                                     // blocks staged; a longer walk reads kidx directly
constexpr uint32_t kOffEnd = kOffRows + kRowsCap * 4;
constexpr size_t kSmemBytes = 1024 + kOffEnd;
static_assert(kSmemBytes <= 232448, "shared memory");

struct PArgs {
    const int32_t* seg_begin;
    const int4* segs;
    const int32_t* kidx;
    __nv_bfloat16* out;
    float* opart;
    float* ml;
    int heads, nq, nk, max_parts;
    float scale_log2;
    KvPages pages;
};

struct Seg {
    int item, kbeg, len, slot;
};

__device__ __forceinline__ Seg load_seg(const PArgs& a, int s) {
    const int4 v = a.segs[s];
    Seg g;
    const int items = a.heads * a.nq;
    g.item = v.x < 0 ? 0 : (v.x >= items ? items - 1 : v.x);
    g.kbeg = v.y < 0 ? 0 : (v.y > a.nk ? a.nk : v.y);
    g.len = v.z < 0 ? 0 : (v.z > a.nk - g.kbeg ? a.nk - g.kbeg : v.z);
    g.slot = v.w < a.max_parts ? v.w : -1;
    return g;
}

// Walks the CTA's blocks in order: segment record, position in it, segment ordinal (segments with blocks only).
struct Cursor {
    int s, t, sig;
    Seg g;
    __device__ void init(int s_beg) {
        s = s_beg - 1;
        t = 0;
        sig = -1;
        g.len = 0;
    }
    // moves to the next block; true when that block opens a segment
    __device__ bool next(const PArgs& a) {
        bool opened = false;
        while (t >= g.len) {
            ++s;
            g = load_seg(a, s);
            t = 0;
            if (g.len > 0) {
                ++sig;
                opened = true;
            }
        }
        return opened;
    }
};

__global__ void __launch_bounds__(kThreadsP, 1)
    attn_bf16_persist_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV, const PArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    griddep_wait_then_release();
    const int s_beg = a.seg_begin[blockIdx.x], s_end = a.seg_begin[blockIdx.x + 1];
    int total = 0, nseg = 0;  // key blocks and non-empty segments of this CTA
    for (int s = s_beg; s < s_end; ++s) {
        const int len = load_seg(a, s).len;
        total += len;
        nseg += len > 0;
    }
    if (total == 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t ld = (int64_t)a.heads * kD;
    volatile uint32_t* abort_word = reinterpret_cast<volatile uint32_t*>(smem + kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
    auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
    auto wait = [&](int b, int phase) {
        return mbar_wait(bar(b), (uint32_t)phase & 1u, abort_word, &g_fvsr_timeout_persist, kLimitNs);
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(bQF + i), 1);
            mbar_init(bar(bQE + i), 1);
            mbar_init(bar(bKF + i), 1);
            mbar_init(bar(bVF + i), 1);
            mbar_init(bar(bPV + i), 1);
            mbar_init(bar(bM + i), 128);
        }
        for (int i = 0; i < 3; ++i) {
            mbar_init(bar(bSF + i), 1);
            mbar_init(bar(bPF + i), 128);
        }
        mbar_init(bar(bOE), 256);
        mbar_init(bar(bFin), 256);
        *abort_word = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the walk's K/V tile rows, staged once so the producer's loads do not wait on global reads
    int32_t* s_rows = reinterpret_cast<int32_t*>(smem + kOffRows);
    const bool staged = total <= kRowsCap;
    if (staged) {
        int jb = 0;
        for (int s = s_beg; s < s_end; ++s) {
            const Seg g = load_seg(a, s);
            const int32_t* lst = a.kidx + (int64_t)g.item * a.nk + g.kbeg;
            for (int t = threadIdx.x; t < g.len; t += kThreadsP) {
                int kb = lst[t];
                kb = kb < 0 ? 0 : (kb >= a.nk ? a.nk - 1 : kb);
                s_rows[jb + t] = kv_phys_block(a.pages, kb) * kBlock;
            }
            jb += g.len;
        }
        __syncthreads();
    }

    if (warp == 0) {
        // ------------- TMA producer: per segment its Q, then K_j two blocks ahead of V_j -------------
        if (lane == 0) {
            Cursor kc, vc;
            kc.init(s_beg);
            vc.init(s_beg);
            auto kv_row = [&](const Seg& g, int t, int j) {
                if (staged) return s_rows[j];
                int kb = a.kidx[(int64_t)g.item * a.nk + g.kbeg + t];
                kb = kb < 0 ? 0 : (kb >= a.nk ? a.nk - 1 : kb);
                return kv_phys_block(a.pages, kb) * kBlock;
            };
            auto load_k = [&](int j) -> bool {
                if (kc.next(a)) {  // a new segment: its Q into slot σ%2 once segment σ−2's S MMAs are done
                    const int sg = kc.sig, qs = sg & 1;
                    if (sg >= 2 && !wait(bQE + qs, sg / 2 - 1)) return false;
                    const int h = kc.g.item / a.nq, qb = kc.g.item % a.nq;
                    mbar_expect_tx(bar(bQF + qs), kTile);
                    tma_load_2d(sbase + kOffQ + qs * kTile, &tmQ, h * kD, qb * kBlock, bar(bQF + qs));
                    tma_load_2d(sbase + kOffQ + qs * kTile + kBox, &tmQ, h * kD + 64, qb * kBlock, bar(bQF + qs));
                }
                const int ks = j & 1;
                if (j >= 2 && !wait(bSF + (j - 2) % 3, (j - 2) / 3)) return false;  // S_{j−2} done: slot free
                const int row = kv_row(kc.g, kc.t, j);
                const int x0 = (kc.g.item / a.nq) * kD;
                mbar_expect_tx(bar(bKF + ks), kTile);
                tma_load_2d(sbase + kOffK + ks * kTile, &tmK, x0, row, bar(bKF + ks));
                tma_load_2d(sbase + kOffK + ks * kTile + kBox, &tmK, x0 + 64, row, bar(bKF + ks));
                ++kc.t;
                return true;
            };
            auto load_v = [&](int j) -> bool {
                vc.next(a);
                const int vs = j & 1;
                if (j >= 2 && !wait(bPV + vs, (j - 2) / 2)) return false;  // PV_{j−2} done: slot free
                const int row = kv_row(vc.g, vc.t, j);
                const int x0 = (vc.g.item / a.nq) * kD;
                mbar_expect_tx(bar(bVF + vs), kTile);
                tma_load_2d(sbase + kOffV + vs * kTile, &tmV, x0, row, bar(bVF + vs));
                tma_load_2d(sbase + kOffV + vs * kTile + kBox, &tmV, x0 + 64, row, bar(bVF + vs));
                ++vc.t;
                return true;
            };
            bool ok = load_k(0) && (total < 2 || load_k(1));
            for (int j = 0; ok && j < total; ++j) ok = load_v(j) && (j + 2 >= total || load_k(j + 2));
        }
    } else if (warp == 1) {
        // ------------- MMA issuer: S_{j+2} after O += P_j·V_j (S/P buffer j%2 is free once PV_j ran) -------------
        if (lane == 0) {
            Cursor sc, pc;
            sc.init(s_beg);
            pc.init(s_beg);
            auto issue_s = [&](int j) -> bool {
                const bool opened = sc.next(a);
                const int qs = sc.sig & 1, ks = j & 1;
                if (opened && !wait(bQF + qs, sc.sig / 2)) return false;
                if (!wait(bKF + ks, j / 2)) return false;
                tc_fence_after();
                const uint32_t d = tmem + kColS + 128u * (uint32_t)(j % 3);
                const uint64_t qd = smem_desc(sbase + kOffQ + qs * kTile, 16, 1024);
                const uint64_t kd = smem_desc(sbase + kOffK + ks * kTile, 16, 1024);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = ((uint32_t)(kk >> 2) * kBox + (uint32_t)(kk & 3) * 32u) >> 4;
                    mma_ss(d, qd + off, kd + off, kIdS, kk > 0 ? 1u : 0u);
                }
                mma_commit(bar(bSF + j % 3));
                if (sc.t == sc.g.len - 1) mma_commit(bar(bQE + qs));  // the segment's last S: Q slot free
                ++sc.t;
                return true;
            };
            auto issue_pv = [&](int j) -> bool {
                const bool opened = pc.next(a);
                const int vs = j & 1;
                if (!wait(bVF + vs, j / 2) || !wait(bPF + j % 3, j / 3)) return false;
                // a segment's first PV overwrites O: segment σ−1's epilogue must have read it
                if (opened && pc.sig >= 1 && !wait(bOE, pc.sig - 1)) return false;
                tc_fence_after();
                const uint64_t vd = smem_desc(sbase + kOffV + vs * kTile, kBox, 1024);
                const uint32_t pa = tmem + kColS + 128u * (uint32_t)(j % 3);
                const uint32_t od = tmem + kColO;
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts(od, pa + 8u * (uint32_t)kk, vd + (uint64_t)(kk * (2048 >> 4)), kIdPV,
                           (pc.t > 0 || kk > 0) ? 1u : 0u);
                mma_commit(bar(bPV + vs));
                ++pc.t;
                return true;
            };
            bool ok = issue_s(0) && (total < 2 || issue_s(1));
            // S_{j+2} lands in the buffer of P_{j−1}: PV_{j−1} was issued first, and one thread's MMAs run in order
            for (int j = 0; ok && j < total; ++j) ok = issue_pv(j) && (j + 2 >= total || issue_s(j + 2));
        }
    } else {
        // ------------- softmax sets + per-segment epilogue -------------
        const int st = (warp - 2) >> 2;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        float* m_x = reinterpret_cast<float*>(smem + kOffMx);
        float* fin = reinterpret_cast<float*>(smem + kOffFin);
        const float sl2 = a.scale_log2;
        bool ok = true;
        auto wait_warp = [&](int b, int phase) { return __all_sync(0xffffffffu, wait(b, phase)); };
        int j0 = 0, sig = 0;
        for (int s = s_beg; ok && s < s_end; ++s) {
            const Seg g = load_seg(a, s);
            if (g.len == 0) continue;
            const int os = sig & 1;
            float l = 0.0f, mref = -INFINITY;  // this set's partial row sum in the segment, relative to mref
            for (int j = j0 + ((j0 & 1) != st ? 1 : 0); j < j0 + g.len; j += 2) {
                const bool first = j == j0;
                if (!wait_warp(bSF + j % 3, j / 3)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sbuf = lane_base + kColS + 128u * (uint32_t)(j % 3);
                uint32_t sv[128];
                tmem_ld32(sbuf, sv);
                tmem_ld32(sbuf + 32, sv + 32);
                tmem_ld32(sbuf + 64, sv + 64);
                tmem_ld32(sbuf + 96, sv + 96);
                tmem_ld_wait(sv);
                tmem_ld_wait(sv + 32);
                tmem_ld_wait(sv + 64);
                tmem_ld_wait(sv + 96);
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int c = 0; c < 128; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], __uint_as_float(sv[c]));
                const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
                // the hand-off from block j−1 (other set) is awaited even across a segment boundary, which keeps
                // the two sets within one phase of each other on both hand-off barriers; its value is used only
                // inside a segment
                float m_prev = -INFINITY;
                if (j > 0) {
                    if (!wait_warp(bM + ((j - 1) & 1), (j - 1) >> 1)) {
                        ok = false;
                        break;
                    }
                    if (!first) m_prev = m_x[((j - 1) & 1) * 128 + r];
                }
                const bool need = mx > m_prev + kThreshold;
                const float m_j = need ? fmaxf(m_prev, mx) : m_prev;
                m_x[(j & 1) * 128 + r] = m_j;
                mbar_arrive(bar(bM + (j & 1)));
                const float neg = -m_j;
                float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    uint32_t pk[16];
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const float p0 = ex2_approx(fmaf(__uint_as_float(sv[32 * q4 + 2 * c]), sl2, neg));
                        const float p1 = ex2_approx(fmaf(__uint_as_float(sv[32 * q4 + 2 * c + 1]), sl2, neg));
                        rs4[c & 3] += p0 + p1;
                        pk[c] = pack_bf16x2(p0, p1);
                    }
                    tmem_st16(sbuf + 16u * (uint32_t)q4, pk);
                }
                if (m_j != mref) {
                    l *= ex2_approx(mref - m_j);
                    mref = m_j;
                }
                l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
                if (!first && __any_sync(0xffffffffu, need)) {
                    // O holds Σ_{i<j} P_i·V_i relative to m_prev once PV_{j−1} has completed
                    if (!wait_warp(bPV + ((j - 1) & 1), (j - 1) / 2)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const float alpha = need ? ex2_approx(m_prev - m_j) : 1.0f;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t ov[32];
                        tmem_ld32(lane_base + kColO + 32u * c, ov);
                        tmem_ld_wait(ov);
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                        tmem_st32(lane_base + kColO + 32u * c, ov);
                    }
                }
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(bar(bPF + j % 3));
            }
            if (!ok) break;
            // ---- segment epilogue: both sets' (l, m_ref) → the row sum at the final maximum; O after its last PV
            float* f = fin + os * 512;
            f[st * 256 + r] = l;
            f[st * 256 + 128 + r] = mref;
            mbar_arrive(bar(bFin));
            const int jl = j0 + g.len - 1;
            ok = wait_warp(bFin, sig) && wait_warp(bPV + (jl & 1), jl / 2);
            if (ok) {
                tc_fence_after();
                const float l0 = f[r], m0 = f[128 + r], l1 = f[256 + r], m1 = f[384 + r];
                const float mf = fmaxf(m0, m1);
                const float l_row = l0 * ex2_approx(m0 - mf) + l1 * ex2_approx(m1 - mf);
                const int h = g.item / a.nq, qb = g.item % a.nq;
                const uint32_t ocol = lane_base + kColO + 64u * (uint32_t)st;
                if (g.slot < 0) {
                    const float inv = 1.0f / l_row;
                    __nv_bfloat16* orow = a.out + ((int64_t)qb * kBlock + r) * ld + h * kD + 64 * st;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t ov[32];
                        tmem_ld32(ocol + 32u * c, ov);
                        tmem_ld_wait(ov);
                        uint32_t w[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i)
                            w[i] = pack_bf16x2(__uint_as_float(ov[2 * i]) * inv, __uint_as_float(ov[2 * i + 1]) * inv);
                        uint4* dst = reinterpret_cast<uint4*>(orow + 32 * c);
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                    }
                } else {  // a piece of a cut item: O relative to mf (its reference maximum), then (mf, l)
                    float* prow = a.opart + ((int64_t)g.slot * kBlock + r) * kD + 64 * st;
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t ov[32];
                        tmem_ld32(ocol + 32u * c, ov);
                        tmem_ld_wait(ov);
                        float4* dst = reinterpret_cast<float4*>(prow + 32 * c);
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            dst[i] = make_float4(__uint_as_float(ov[4 * i]), __uint_as_float(ov[4 * i + 1]),
                                                 __uint_as_float(ov[4 * i + 2]), __uint_as_float(ov[4 * i + 3]));
                    }
                    if (st == 0) {
                        a.ml[(int64_t)g.slot * 256 + r] = mf;
                        a.ml[(int64_t)g.slot * 256 + 128 + r] = l_row;
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(bar(bOE));  // O drained: the next segment's first PV may overwrite it
            j0 += g.len;
            ++sig;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
}

}  // namespace

cudaError_t read_and_clear_persist_error(int* flag) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_fvsr_timeout_persist, sizeof(int));
    if (e != cudaSuccess) return e;
    if (v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_fvsr_timeout_persist, &zero, sizeof(int));
    }
    *flag = v;
    return e;
}

cudaError_t launch_attn_bf16_persist(const void* q, const void* k, const void* v, int64_t kv_rows,
                                     const KvPages& pages, int heads, int nq, int nk, const int32_t* kidx,
                                     const SchedLayout& L, const void* sched, void* out, cudaStream_t st) {
    if (!L.persistent) return cudaErrorInvalidValue;  // the buffer holds no persistent partition
    CUtensorMap mq, mk, mv;
    const int64_t channels = (int64_t)heads * kD;
    if (!make_tile_map(&mq, q, (int64_t)nq * kBlock, channels) || !make_tile_map(&mk, k, kv_rows, channels) ||
        !make_tile_map(&mv, v, kv_rows, channels))
        return cudaErrorInvalidValue;
    cudaError_t e =
        cudaFuncSetAttribute(attn_bf16_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    const uint8_t* b = static_cast<const uint8_t*>(sched);
    PArgs a;
    a.seg_begin = reinterpret_cast<const int32_t*>(b + L.off_seg_begin);
    a.segs = reinterpret_cast<const int4*>(b + L.off_segs);
    a.kidx = kidx;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.opart = reinterpret_cast<float*>(const_cast<uint8_t*>(b) + L.off_opart);
    a.ml = reinterpret_cast<float*>(const_cast<uint8_t*>(b) + L.off_ml);
    a.heads = heads;
    a.nq = nq;
    a.nk = nk;
    a.max_parts = L.max_parts;
    a.scale_log2 = (1.0f / sqrtf((float)kD)) * 1.4426950408889634f;
    a.pages = pages;
    e = launch_pdl(attn_bf16_persist_kernel, dim3(L.G), dim3(kThreadsP), kSmemBytes, st, mq, mk, mv, a);
    if (e != cudaSuccess) return e;
    return launch_combine(L, sched, heads, nq, out, st);
}

}  // namespace fvsr
