// select.cu — LCSA block selection (draftBlockMaskAndProbs, DiT.swift:158-174) on pooled fp32 Q/K.
//
// One cooperative launch (select_fused_kernel, every CTA resident; phases separated by bounded grid barriers):
//   1. score tiles       block scores pq·pk / sqrt(d) (fixed-order fmaf dot over 128 dims) with the spatial locality
//                        mask (DiT.swift:130-145, computed from (bh, bw, R) instead of a table; −inf outside), one
//                        64 × 32 (query block × key block) tile at a time → scores (H, Nq, Nk).
//   2. softmax           one warp per (head, query block) row: softmax over key blocks, in place → probs, and pass 1
//                        of the radix select's histograms.
//   3, 4. radix passes   passes 2 and 3 of an MSB-first radix select (11 + 11 + 10 bits of the fp32 patterns —
//                        probabilities are ≥ 0, so unsigned order = float order; no sort) that finds, per
//                        (head, query slice) row of n = (Nq/q_slices)·Nk entries, the exact (min(n−1, topk)+1)-th
//                        largest probability; the entries are spread evenly over all CTAs.
//   5. compaction        p > threshold into ascending kidx lists, kcnt and the optional 0/1 mask.
//   6. item order        (optional) the longest-first order of the (head, query block) items for the attention.
// The six steps used to be six launches; in one launch they pay no launch gaps and no tail of a small grid.
//
// Bit-exactness. Every floating-point operation is an explicit round-to-nearest intrinsic (never contracted) in the
// order that the CPU restatement fixes: dot = fmaf chain over e = 0..127; score = dot / sqrtf(128); softmax
// e_j = fvsr_exp(s_j − max) with per-lane partial sums over j ≡ lane (mod 32) in increasing j, a xor-butterfly
// reduction, and p_j = e_j / sum. fvsr_exp is Cody–Waite range reduction (W. J. Cody, W. Waite, 1980) with a
// degree-7 Taylor polynomial — the same function, constant for constant, as the CPU restatement.
#include <math.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kTI = 64;   // query blocks per score tile
constexpr int kTJ = 32;   // key blocks per score tile
constexpr int kPS = 132;  // padded fp32 row stride of the staged pooled rows

__device__ __forceinline__ float pow2i(int n) { return __uint_as_float((uint32_t)(n + 127) << 23); }

// e^x: the softmax exponential of the selection (see the file comment for the method). Branch-free: the special
// cases are selected at the end, so a warp never diverges on it.
__device__ __forceinline__ float fvsr_exp(float x) {
    const float log2e = 1.44269502925872802734375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.428606765330187045e-06f;
    const float xc = fminf(fmaxf(x, -104.0f), 88.72f);  // keeps n in range; the out-of-range results are selected below
    const float n = rintf(__fmul_rn(xc, log2e));
    float r = __fmaf_rn(-n, ln2_hi, xc);
    r = __fmaf_rn(-n, ln2_lo, r);
    float p = 1.0f / 5040.0f;
    p = __fmaf_rn(p, r, 1.0f / 720.0f);
    p = __fmaf_rn(p, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n;
    // 2^n as one multiply for −126 ≤ n ≤ 127, else (p·2^(n+64))·2^−64 or (p·2^(n−1))·2 — the second factor is 1 in
    // the common case, which leaves the product unchanged
    const bool lo = ni < -126, hi = ni > 127;
    const int e1 = lo ? ni + 64 : (hi ? ni - 1 : ni);
    const float s2 = lo ? pow2i(-64) : (hi ? 2.0f : 1.0f);
    float y = __fmul_rn(__fmul_rn(p, pow2i(e1)), s2);
    y = x < -104.0f ? 0.0f : y;
    y = x > 88.72f ? INFINITY : y;
    return x != x ? x : y;
}

// Exact k-th largest by a 3-pass MSB-first radix select on the fp32 bit patterns (probabilities are ≥ 0, so the
// unsigned order of the bits is the float order): pass 1 bins bits [31:21] (2048 bins), pass 2 bits [20:10] (2048),
// pass 3 bits [9:0] (1024). Each pass only counts the entries whose higher bits equal the bins chosen so far.
constexpr int kBins1 = 2048, kBins2 = 2048, kBins3 = 1024;
// Per-row workspace words (all cleared before each selection): the three histograms, four counter words, and the
// radix state after each pass. Row 0's last counter word is the grid-barrier counter and its word kOffState + 9 the
// abort word of the selection launch.
constexpr int kOffCounter = kBins1 + kBins2 + kBins3;
constexpr int kOffState = kOffCounter + 4;             // state after pass p at kOffState + 3·(p−1): prefix, mask, rank
constexpr int kHistPerRow = kOffState + 12;

// Warp-aggregated shared-memory histogram increment (bins repeat heavily: probabilities share exponents).
__device__ __forceinline__ void hist_add(uint32_t* h, uint32_t key, bool valid) {
    const uint32_t k = valid ? key : 0xFFFFFFFFu;
    const uint32_t peers = __match_any_sync(0xffffffffu, k);
    const int lane = threadIdx.x & 31;
    if (valid && lane == __ffs(peers) - 1) atomicAdd(h + key, (uint32_t)__popc(peers));
}

// A group of kSelThreads threads (eight warps) that works as one unit: the fused selection runs kSelGroups groups per
// CTA, the stand-alone item-order kernel one group per CTA. Groups synchronise with their own named barrier.
constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelGroups = 3;       // groups per CTA of the fused selection (one CTA per SM)
constexpr int kMiscWords = 64;      // per-group shared scratch words (scan partials, broadcasts)

struct Grp {
    int id;   // group within the CTA
    int tid;  // thread within the group
    __device__ __forceinline__ void sync() const {
        asm volatile("bar.sync %0, %1;" ::"r"(1 + id), "r"(kSelThreads) : "memory");
    }
};

// Finds, among `nbins` histogram bins scanned from the highest, the bin holding the entry of descending rank `rank`
// (0 = largest). All threads of the group call it (nbins / kSelThreads ≤ 16); the result goes to every thread.
__device__ void group_find_bin(const uint32_t* __restrict__ hist, int nbins, uint32_t rank, uint32_t* out_bin,
                               uint32_t* out_rank, const Grp& g, uint32_t* misc) {
    uint32_t* warp_sums = misc;  // [kSelWarps]
    const int tid = g.tid, lane = tid & 31, warp = tid >> 5;
    const int per = nbins / kSelThreads;
    const int top = nbins - 1 - per * tid;  // this thread covers bins top, top−1, …, top−per+1
    uint32_t c[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) c[i] = i < per ? __ldcg(hist + top - i) : 0u;
    uint32_t local = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) local += c[i];
    uint32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    if (tid == 0) {
        misc[kSelWarps] = 0;
        misc[kSelWarps + 1] = 0;
    }
    g.sync();
    uint32_t before = 0;
    for (int w = 0; w < warp; ++w) before += warp_sums[w];
    const uint32_t excl = before + incl - local;
    if (rank >= excl && rank < excl + local) {
        uint32_t cum = excl;
        for (int i = 0; i < per; ++i) {
            if (rank < cum + c[i]) {
                misc[kSelWarps] = (uint32_t)(top - i);
                misc[kSelWarps + 1] = rank - cum;
                break;
            }
            cum += c[i];
        }
    }
    g.sync();
    *out_bin = misc[kSelWarps];
    *out_rank = misc[kSelWarps + 1];
    g.sync();
}

// Radix state after a pass: the bits fixed so far (prefix under mask) and the descending rank still to find among the
// entries that carry them.
struct RadixState {
    uint32_t prefix, mask, rank;
};

__device__ __forceinline__ RadixState load_state(const uint32_t* __restrict__ hrow, int pass) {
    const uint32_t* st = hrow + kOffState + 3 * (pass - 1);
    return RadixState{__ldcg(st), __ldcg(st + 1), __ldcg(st + 2)};
}

// The state of selection row `hrow` after pass `pass`, from the state after the previous pass (rank0 before pass 1)
// and this pass's complete histogram; thread 0 of the group stores it.
__device__ void compute_state(uint32_t* __restrict__ hrow, int pass, uint32_t rank0, const Grp& g, uint32_t* misc) {
    RadixState r = pass > 1 ? load_state(hrow, pass - 1) : RadixState{0u, 0u, rank0};
    const int off = pass == 1 ? 0 : (pass == 2 ? kBins1 : kBins1 + kBins2);
    const int nb = pass == 3 ? kBins3 : kBins1;
    uint32_t b;
    group_find_bin(hrow + off, nb, r.rank, &b, &r.rank, g, misc);
    if (pass == 1) {
        r.prefix = b << 21;
        r.mask = 0xFFE00000u;
    } else if (pass == 2) {
        r.prefix |= b << 10;
        r.mask |= 0x001FFC00u;
    } else {
        r.prefix |= b;
        r.mask = 0xFFFFFFFFu;
    }
    if (g.tid == 0) {
        uint32_t* st = hrow + kOffState + 3 * (pass - 1);
        st[0] = r.prefix;
        st[1] = r.mask;
        st[2] = r.rank;
    }
}

// Called by a group once its contributions to selection row sr's pass-`pass` histogram are in global memory: counts
// the group in (threadfence reduction), and the group that completes the count of the `need` groups that contribute
// to the row computes the row's state after the pass — once per row, so the next phase only reads three words.
__device__ void arrive_and_advance(uint32_t* __restrict__ hrow, int pass, uint32_t need, uint32_t rank0, const Grp& g,
                                   uint32_t* misc) {
    __threadfence();
    g.sync();
    if (g.tid == 0) misc[kSelWarps + 2] = atomicAdd(hrow + kOffCounter + pass - 1, 1u) == need - 1 ? 1u : 0u;
    g.sync();
    if (misc[kSelWarps + 2]) {
        __threadfence();
        compute_state(hrow, pass, rank0, g, misc);
    }
    g.sync();
}

__device__ __forceinline__ uint32_t row_rank0(int64_t n, int topk) {
    return (uint32_t)((int64_t)topk < n - 1 ? (int64_t)topk : n - 1);
}

// Set when a grid barrier of the selection gave up (fvsr_device_check reports it).
__device__ int g_select_timeout = 0;

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t kBarrierLimitNs = 4000000000ull;

// Grid-wide barrier of the cooperative selection launch (all CTAs are resident at once). Each CTA publishes its
// writes (fence), adds one to `counter` (zeroed with the histograms before the launch) and waits until the count
// reaches `target` = phase · gridDim.x. The wait is bounded: after kBarrierLimitNs it raises `abort_word` (so every
// other CTA stops waiting at its next poll) and the device timeout word, and returns false; the CTA then returns.
__device__ bool grid_barrier(uint32_t* counter, uint32_t* abort_word, uint32_t target) {
    __shared__ uint32_t s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(counter, 1u);
        uint32_t ok = 1;
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t it = 0; ld_acquire_u32(counter) < target; ++it) {
            if (*reinterpret_cast<volatile uint32_t*>(abort_word)) {
                ok = 0;
                break;
            }
            if ((it & 31u) == 31u && globaltimer_ns() - t0 > kBarrierLimitNs) {
                atomicExch(abort_word, 1u);
                atomicExch(&g_select_timeout, 1);
                ok = 0;
                break;
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

struct SelArgs {
    const float* pq;   // pooled queries (Nq, H·128) fp32
    const float* pk;   // pooled keys, logical block j at physical block kv_phys_block(pages, j)
    KvPages pages;
    int heads, nq, nk, bh, bw, local_range, q_slices, topk;
    float sqrt_d;
    float* probs;      // (H, Nq, Nk): scores, then probabilities in place
    uint32_t* hist;    // per selection row: histograms, arrival counters, radix states; row 0: the barrier words
    int32_t* kidx;
    int32_t* kcnt;
    uint8_t* mask;     // optional
    int32_t* order;    // optional longest-first order of the items whose query block is in [order_q0, order_q1)
    int order_q0, order_q1;
};

// Phase 1 unit — score tile `tile`: kTI query blocks × kTJ key blocks of one head. Thread (ty, tx) computes the 4 × 2
// micro-tile of rows 4·ty + a and keys tx + 16·u, each score a sequential fmaf chain over e = 0..127, then / sqrt(128)
// (IEEE division), −inf outside the locality window (DiT.swift:130-145, computed from (bh, bw, R)).
__device__ __forceinline__ void score_tile(const SelArgs& a, int tile, float* __restrict__ sq, const Grp& g) {
    static_assert(kTI == 64 && kTJ == 32, "micro-tile layout: 16 × 16 threads of 4 rows × 2 keys");
    float* sk = sq + kTI * kPS;
    const int ntj = (a.nk + kTJ - 1) / kTJ, nti = (a.nq + kTI - 1) / kTI;
    const int h = tile / (nti * ntj), rem = tile - h * nti * ntj;
    const int i0 = (rem / ntj) * kTI, j0 = (rem % ntj) * kTJ;
    const int64_t ld = (int64_t)a.heads * kD;
    const int tid = g.tid;
    {  // stage the tile's pooled rows: all 12 loads of a thread in flight before the first store
        constexpr int kPerQ = (kTI * 32) / kSelThreads, kPerK = (kTJ * 32) / kSelThreads;
        float4 vq[kPerQ], vk[kPerK];
#pragma unroll
        for (int k = 0; k < kPerQ; ++k) {
            const int idx = tid + kSelThreads * k, r = idx >> 5, e4 = idx & 31, i = i0 + r;
            vq[k] = i < a.nq ? __ldg(reinterpret_cast<const float4*>(a.pq + i * ld + h * kD) + e4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < kPerK; ++k) {
            const int idx = tid + kSelThreads * k, r = idx >> 5, e4 = idx & 31, j = j0 + r;
            vk[k] = j < a.nk ? __ldg(reinterpret_cast<const float4*>(a.pk + (int64_t)kv_phys_block(a.pages, j) * ld +
                                                                     h * kD) + e4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < kPerQ; ++k) {
            const int idx = tid + kSelThreads * k, r = idx >> 5, e4 = idx & 31;
            *reinterpret_cast<float4*>(sq + r * kPS + e4 * 4) = vq[k];
        }
#pragma unroll
        for (int k = 0; k < kPerK; ++k) {
            const int idx = tid + kSelThreads * k, r = idx >> 5, e4 = idx & 31;
            *reinterpret_cast<float4*>(sk + r * kPS + e4 * 4) = vk[k];
        }
    }
    g.sync();
    // a warp covers tile rows [8·warp, 8·warp + 8): past the last query block it has nothing to write (warp-uniform)
    if (i0 + 8 * (tid >> 5) < a.nq) {
        const int ty = tid >> 4, tx = tid & 15;
        float acc[4][2];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int u = 0; u < 2; ++u) acc[x][u] = 0.0f;
#pragma unroll 4
        for (int e4 = 0; e4 < 32; ++e4) {
            float4 x[4], y[2];
#pragma unroll
            for (int r = 0; r < 4; ++r) x[r] = reinterpret_cast<const float4*>(sq + (4 * ty + r) * kPS)[e4];
#pragma unroll
            for (int u = 0; u < 2; ++u) y[u] = reinterpret_cast<const float4*>(sk + (tx + 16 * u) * kPS)[e4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    acc[r][u] = __fmaf_rn(x[r].x, y[u].x, acc[r][u]);
                    acc[r][u] = __fmaf_rn(x[r].y, y[u].y, acc[r][u]);
                    acc[r][u] = __fmaf_rn(x[r].z, y[u].z, acc[r][u]);
                    acc[r][u] = __fmaf_rn(x[r].w, y[u].w, acc[r][u]);
                }
        }
        const int sblk = a.bh * a.bw, half = a.local_range / 2;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int i = i0 + 4 * ty + r;
            if (i >= a.nq) continue;
            const int qi = i % sblk, lo_r = qi / a.bw - half, lo_c = qi % a.bw - half;
            float* out = a.probs + ((int64_t)h * a.nq + i) * a.nk;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int j = j0 + tx + 16 * u;
                if (j >= a.nk) continue;
                const int kj = j % sblk, kr = kj / a.bw, kc = kj % a.bw;
                const bool allowed = kr >= lo_r && kr <= lo_r + a.local_range - 1 && kc >= lo_c &&
                                     kc <= lo_c + a.local_range - 1;
                out[j] = allowed ? __fdiv_rn(acc[r][u], a.sqrt_d) : -INFINITY;
            }
        }
    }
    g.sync();  // the next tile restages the shared rows
}

// Phase 2 — rows [r0, r1) of the (H·Nq, Nk) score matrix, one warp per row: softmax in place (scores → probs) and
// pass 1 of the radix select's histograms. The range's first two selection rows count in shared memory, any further
// one straight into global memory. NCH > 0: the row (at most NCH·256 key blocks) stays in registers between the
// three sweeps; NCH = 0 re-reads it. Then the group counts itself in on each selection row it touched.
template <int NCH>
__device__ __forceinline__ void softmax_rows(const SelArgs& a, int64_t r0, int64_t r1, int64_t rpc,
                                             uint32_t* __restrict__ shist, const Grp& g, uint32_t* misc) {
    const int warp = g.tid >> 5, lane = g.tid & 31;
    const int nqs = a.nq / a.q_slices, nk = a.nk;
    const int64_t sr0 = r0 / nqs;
    const int64_t nsel = (int64_t)a.heads * a.q_slices;
    for (int i = g.tid; i < 2 * kBins1; i += kSelThreads) shist[i] = 0;
    g.sync();
    for (int64_t rr = r0 + warp; rr < r1; rr += kSelWarps) {  // warp-uniform
        float* row = a.probs + rr * nk;
        constexpr int kR = NCH > 0 ? NCH * 8 : 1;
        float rv[kR];
        if (NCH > 0) {
#pragma unroll
            for (int c = 0; c < kR; ++c) {
                const int j = 256 * (c >> 3) + 32 * (c & 7) + lane;
                rv[c] = j < nk ? __ldcg(row + j) : -INFINITY;
            }
        }
        float m = -INFINITY;
        if (NCH > 0) {
#pragma unroll
            for (int c = 0; c < kR; ++c) m = fmaxf(m, rv[c]);
        } else {
            for (int jb = 0; jb < nk; jb += 256) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    v[u] = j < nk ? __ldcg(row + j) : -INFINITY;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) m = fmaxf(m, v[u]);
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float part = 0.0f;  // lane partial sum over j ≡ lane (mod 32), increasing j
        if (NCH > 0) {
#pragma unroll
            for (int c = 0; c < kR; ++c) {
                const int j = 256 * (c >> 3) + 32 * (c & 7) + lane;
                const float e = fvsr_exp(__fsub_rn(rv[c], m));
                rv[c] = j < nk ? e : 0.0f;
                if (j < nk) part = __fadd_rn(part, e);
            }
        } else {
            for (int jb = 0; jb < nk; jb += 256) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    v[u] = j < nk ? __ldcg(row + j) : -INFINITY;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    const float e = fvsr_exp(__fsub_rn(v[u], m));
                    if (j < nk) {
                        row[j] = e;
                        part = __fadd_rn(part, e);
                    }
                }
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
        const int64_t sr = rr / nqs, local = sr - sr0;
        uint32_t* gh = a.hist + sr * kHistPerRow;
        auto emit = [&](int j, float v) {
            const float p = v == 0.0f ? 0.0f : __fdiv_rn(v, part);  // 0 / sum = +0 exactly
            if (j < nk) row[j] = p;
            const uint32_t bin = __float_as_uint(p) >> 21;
            if (local < 2)
                hist_add(shist + local * kBins1, bin, j < nk);
            else if (j < nk)
                atomicAdd(gh + bin, 1u);
        };
        if (NCH > 0) {
#pragma unroll
            for (int c = 0; c < kR; ++c) emit(256 * (c >> 3) + 32 * (c & 7) + lane, rv[c]);
        } else {
            for (int jb = 0; jb < nk; jb += 256) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int j = jb + 32 * u + lane;
                    v[u] = j < nk ? __ldcg(row + j) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) emit(jb + 32 * u + lane, v[u]);
            }
        }
    }
    g.sync();
    for (int x = g.tid; x < 2 * kBins1; x += kSelThreads) {
        const uint32_t c = shist[x];
        const int64_t sr = sr0 + x / kBins1;
        if (c && sr < nsel) atomicAdd(a.hist + sr * kHistPerRow + (x % kBins1), c);
    }
    const uint32_t rank0 = row_rank0((int64_t)nqs * nk, a.topk);
    for (int64_t sr = sr0; r0 < r1 && sr * nqs < r1; ++sr) {
        // groups whose row range meets selection row sr (ranges of rpc rows each)
        const uint32_t need = (uint32_t)(((sr + 1) * nqs - 1) / rpc - (sr * nqs) / rpc + 1);
        arrive_and_advance(a.hist + sr * kHistPerRow, 1, need, rank0, g, misc);
    }
}

// Phases 3 and 4 — radix pass `pass` (2: bits [20:10], 3: bits [9:0]) over the entries [e0, e1) of the flattened
// probabilities, where selection row sr = (head, query slice) owns entries [sr·n, (sr + 1)·n), n = (Nq/q_slices)·Nk.
// Only entries whose higher bits equal the bins chosen so far are counted; the last group to count into a row
// computes the row's next state.
__device__ __forceinline__ void radix_pass(const SelArgs& a, int pass, int64_t e0, int64_t e1, int64_t epc,
                                           uint32_t* __restrict__ sh, const Grp& g, uint32_t* misc) {
    const int nqs = a.nq / a.q_slices;
    const int64_t n = (int64_t)nqs * a.nk;
    const uint32_t rank0 = row_rank0(n, a.topk);
    const uint32_t* flat = reinterpret_cast<const uint32_t*>(a.probs);
    const int nb = pass == 2 ? kBins2 : kBins3;
    for (int64_t sr = e0 / n; e0 < e1 && sr * n < e1; ++sr) {
        uint32_t* hrow = a.hist + sr * kHistPerRow;
        const RadixState st = load_state(hrow, pass - 1);
        for (int i = g.tid; i < nb; i += kSelThreads) sh[i] = 0;
        g.sync();
        const int64_t lo = e0 > sr * n ? e0 : sr * n, hi = e1 < (sr + 1) * n ? e1 : (sr + 1) * n;
        for (int64_t base = lo; base < hi; base += 4 * kSelThreads) {  // uniform trip count: whole warps in hist_add
            uint32_t u[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int64_t idx = base + g.tid + k * kSelThreads;
                u[k] = idx < hi ? __ldcg(flat + idx) : 0xFFFFFFFFu;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int64_t idx = base + g.tid + k * kSelThreads;
                const bool valid = idx < hi && (u[k] & st.mask) == st.prefix;
                hist_add(sh, pass == 2 ? (u[k] >> 10) & (kBins2 - 1) : u[k] & (kBins3 - 1), valid);
            }
        }
        g.sync();
        uint32_t* gh = hrow + (pass == 2 ? kBins1 : kBins1 + kBins2);
        for (int i = g.tid; i < nb; i += kSelThreads)
            if (sh[i]) atomicAdd(gh + i, sh[i]);
        const uint32_t need = (uint32_t)(((sr + 1) * n - 1) / epc - (sr * n) / epc + 1);
        arrive_and_advance(hrow, pass, need, rank0, g, misc);
    }
}

// Phase 5 — rows [r0, r1): threshold = the exact (min(n−1, topk)+1)-th largest entry of the row's selection row (the
// state after pass 3); p > threshold compacted into ascending kidx lists (the rest −1), kcnt and the optional 0/1
// mask, one warp per row.
__device__ __forceinline__ void finish_rows(const SelArgs& a, int64_t r0, int64_t r1, const Grp& g) {
    const int warp = g.tid >> 5, lane = g.tid & 31;
    const int nqs = a.nq / a.q_slices, nk = a.nk;
    for (int64_t rr = r0 + warp; rr < r1; rr += kSelWarps) {
        const float thr = __uint_as_float(load_state(a.hist + (rr / nqs) * kHistPerRow, 3).prefix);
        const float* p = a.probs + rr * nk;
        int32_t* lst = a.kidx + rr * nk;
        int cnt = 0;
        for (int jb = 0; jb < nk; jb += 256) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int j = jb + 32 * u + lane;
                v[u] = j < nk ? __ldcg(p + j) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int j = jb + 32 * u + lane;
                const bool keep = j < nk && v[u] > thr;
                const uint32_t bal = __ballot_sync(0xffffffffu, keep);
                if (keep) lst[cnt + __popc(bal & ((1u << lane) - 1u))] = j;
                if (a.mask && j < nk) a.mask[rr * nk + j] = keep ? 1 : 0;
                cnt += __popc(bal);
            }
        }
        for (int j = cnt + lane; j < nk; j += 32) lst[j] = -1;
        if (lane == 0) a.kcnt[rr] = cnt;
    }
}

// Longest-first order of one head segment of a range of items — the items of [item_begin, item_begin + item_count)
// whose query block lies in [q0, q1) (see launch_item_order; q0 = 0, q1 = nq for a contiguous range): the non-empty
// items of each head segment in turn (segments in head order), longest key list first within a segment (ties by id);
// then every empty item of the range, ascending. Empty items only write zeros, so they go last: placed
// between heads they would delay the next head's long items. Rank of a non-empty item inside its segment = items of
// the segment with a longer key list, or an equal one and a smaller id; empty items rank after all non-empty ones, by
// id. All threads of the group call it; sc (4096 words) and cnt (4 words) are shared scratch of the group.
__device__ void order_segment(const int32_t* __restrict__ kcnt, int nq, int item_begin, int item_count, int q0, int q1,
                              int32_t* __restrict__ order, int seg, int32_t* sc, int* cnt, const Grp& g) {
    // sc and cnt are shared memory that several threads write and read across g.sync(): not __restrict__, so the
    // compiler keeps their accesses on their side of the inline-asm barrier
    const int h = item_begin / nq + seg;
    const int s0 = max(item_begin, h * nq + q0), s1 = min(item_begin + item_count, h * nq + q1);
    const int n = s1 - s0;
    if (n <= 0) return;  // uniform over the group
    if (g.tid < 4) cnt[g.tid] = 0;
    g.sync();
    {
        int na = 0, nb = 0, nc = 0, nd = 0;
        for (int i = g.tid; i < item_count; i += kSelThreads) {
            const int it = item_begin + i, qb = it % nq;
            if (qb < q0 || qb >= q1) continue;
            const bool nz = __ldcg(kcnt + it) > 0;
            nc += nz;
            if (it < s0) {
                na += nz;
                nb += !nz;
            } else if (it < s1) {
                nd += nz;
            }
        }
        atomicAdd(&cnt[0], na);
        atomicAdd(&cnt[1], nb);
        atomicAdd(&cnt[2], nc);
        atomicAdd(&cnt[3], nd);
    }
    g.sync();
    const int ne_before = cnt[0], e_before = cnt[1], ne_total = cnt[2], ne_seg = cnt[3];
    auto place = [&](int i, int rank, bool nz) {  // rank: position inside the segment, non-empty items first
        const int pos = nz ? ne_before + rank : ne_total + e_before + (rank - ne_seg);
        order[pos] = s0 + i;
    };
    if (n > 4096) {  // no room to rank: each class in ascending id order
        if (g.tid == 0) {
            int x = 0, y = 0;
            for (int i = 0; i < n; ++i) {
                const bool nz = __ldcg(kcnt + s0 + i) > 0;
                place(i, nz ? x++ : ne_seg + y++, nz);
            }
        }
        g.sync();
        return;
    }
    for (int i = g.tid; i < n; i += kSelThreads) sc[i] = max(__ldcg(kcnt + s0 + i), 0);
    g.sync();
    for (int i = g.tid; i < n; i += kSelThreads) {
        const int ci = sc[i];
        int rank = 0;
        for (int t = 0; t < n; ++t) {
            const int ct = sc[t];
            rank += (ct > ci) || (ct == ci && t < i);
        }
        place(i, rank, ci > 0);
    }
    g.sync();
}

// Shared memory of one group: the two staged pooled tiles of a score tile (the largest phase), then its scratch words.
constexpr size_t kGroupSmemWords = (size_t)(kTI + kTJ) * kPS;

// The whole selection of one call in one cooperative launch: one CTA per SM, each of kSelGroups groups a worker
// (worker w = group·gridDim.x + CTA, so consecutive work goes to different SMs). Phases, separated by grid barriers:
// (1) score tiles, (2) softmax + radix pass 1 per row, (3) radix pass 2, (4) radix pass 3 — after each histogram
// pass the last worker to count into a selection row computes that row's radix state — (5) threshold and compaction
// per row, and with an order buffer (6) the longest-first item order. Every phase splits its work evenly over the
// workers.
template <int NCH>
__global__ void __launch_bounds__(kSelThreads * kSelGroups, 1) select_fused_kernel(const __grid_constant__ SelArgs a) {
    extern __shared__ float4 sel_smem4[];
    const Grp g{(int)threadIdx.x / kSelThreads, (int)threadIdx.x % kSelThreads};
    float* gsm = reinterpret_cast<float*>(sel_smem4) + (size_t)g.id * (kGroupSmemWords + kMiscWords);
    uint32_t* gsm_u = reinterpret_cast<uint32_t*>(gsm);
    uint32_t* misc = gsm_u + kGroupSmemWords;
    griddep_wait_then_release();
    const uint32_t G = gridDim.x;
    const int W = kSelGroups * (int)G, w = g.id * (int)G + (int)blockIdx.x;
    uint32_t* bar = a.hist + kOffCounter + 3;
    uint32_t* abort_word = a.hist + kOffState + 9;
    const int ntiles = a.heads * ((a.nq + kTI - 1) / kTI) * ((a.nk + kTJ - 1) / kTJ);
    for (int t = w; t < ntiles; t += W) score_tile(a, t, gsm, g);
    if (!grid_barrier(bar, abort_word, G)) return;

    const int64_t rows = (int64_t)a.heads * a.nq;
    const int64_t rpc = (rows + W - 1) / W;
    const int64_t r0 = min(rows, (int64_t)w * rpc), r1 = min(rows, r0 + rpc);
    softmax_rows<NCH>(a, r0, r1, rpc, gsm_u, g, misc);
    if (!grid_barrier(bar, abort_word, 2 * G)) return;

    const int64_t ents = rows * a.nk;
    const int64_t epc = (((ents + W - 1) / W) + 255) & ~int64_t(255);
    const int64_t e0 = min(ents, (int64_t)w * epc), e1 = min(ents, e0 + epc);
    radix_pass(a, 2, e0, e1, epc, gsm_u, g, misc);
    if (!grid_barrier(bar, abort_word, 3 * G)) return;
    radix_pass(a, 3, e0, e1, epc, gsm_u, g, misc);
    if (!grid_barrier(bar, abort_word, 4 * G)) return;

    finish_rows(a, r0, r1, g);
    if (!a.order) return;
    if (!grid_barrier(bar, abort_word, 5 * G)) return;
    const int items = a.heads * a.nq;
    for (int seg = w; seg < a.heads; seg += W)
        order_segment(a.kcnt, a.nq, 0, items, a.order_q0, a.order_q1, a.order, seg, reinterpret_cast<int32_t*>(gsm_u),
                      reinterpret_cast<int*>(gsm_u + 4096), g);
}

__global__ void __launch_bounds__(256) mask_to_lists_kernel(const float* __restrict__ mask, int rows, int nk,
                                                            int32_t* __restrict__ kidx, int32_t* __restrict__ kcnt) {
    griddep_wait_then_release();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* m = mask + (int64_t)warp * nk;
    int32_t* lst = kidx + (int64_t)warp * nk;
    int cnt = 0;
    for (int j0 = 0; j0 < nk; j0 += 32) {
        const int j = j0 + lane;
        const bool keep = j < nk && m[j] > 0.5f;
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (keep) lst[cnt + __popc(bal & ((1u << lane) - 1u))] = j;
        cnt += __popc(bal);
    }
    for (int j = cnt + lane; j < nk; j += 32) lst[j] = -1;
    if (lane == 0) kcnt[warp] = cnt;
}

// One 256-thread CTA (one group) per head segment of the range (order_segment).
__global__ void __launch_bounds__(kSelThreads) item_order_kernel(const int32_t* __restrict__ kcnt, int nq,
                                                                 int item_begin, int item_count,
                                                                 int32_t* __restrict__ order) {
    griddep_wait_then_release();
    __shared__ int32_t sc[4096];
    __shared__ int cnt[4];
    order_segment(kcnt, nq, item_begin, item_count, 0, nq, order, blockIdx.x, sc, cnt, Grp{0, (int)threadIdx.x});
}

}  // namespace

// Shared memory of the fused selection CTA: per group the staged score tiles and the group's scratch words.
size_t select_smem_bytes() { return sizeof(float) * (size_t)kSelGroups * (kGroupSmemWords + kMiscWords); }

size_t select_hist_bytes(int heads, int q_slices) { return sizeof(uint32_t) * (size_t)heads * q_slices * kHistPerRow; }

cudaError_t launch_select(const float* pq, const float* pk, const KvPages& pk_pages, int heads, int nq, int nk, int bh,
                          int bw, int local_range, int q_slices, int topk, float* probs, uint32_t* hist, int32_t* kidx,
                          int32_t* kcnt, uint8_t* mask, int32_t* order, cudaStream_t st, int order_q0,
                          int order_q1, int spare_sms) {
    SelArgs a;
    a.pq = pq;
    a.pk = pk;
    a.pages = pk_pages;
    a.heads = heads;
    a.nq = nq;
    a.nk = nk;
    a.bh = bh;
    a.bw = bw;
    a.local_range = local_range;
    a.q_slices = q_slices;
    a.topk = topk;
    a.sqrt_d = sqrtf((float)kD);
    a.probs = probs;
    a.hist = hist;
    a.kidx = kidx;
    a.kcnt = kcnt;
    a.mask = mask;
    a.order = order;
    a.order_q0 = order_q1 > 0 ? order_q0 : 0;
    a.order_q1 = order_q1 > 0 ? order_q1 : nq;
    const int nch = nk <= 256 ? 1 : nk <= 512 ? 2 : nk <= 768 ? 3 : nk <= 1024 ? 4 : 0;
    void (*kernels[5])(SelArgs) = {select_fused_kernel<0>, select_fused_kernel<1>, select_fused_kernel<2>,
                                   select_fused_kernel<3>, select_fused_kernel<4>};
    auto kernel = kernels[nch];
    const int smem = (int)select_smem_bytes();
    // grid = one CTA per SM (its shared memory admits no second one; the grid barriers need every CTA resident),
    // checked once per device and variant
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> grid_of;
    int grid = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = grid_of.find({dev, nch});
        if (it != grid_of.end()) {
            grid = it->second;
        } else {
            int nsm = 0, per_sm = 0;
            if ((e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess)
                return e;
            if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
            if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kSelThreads * kSelGroups, smem)) !=
                cudaSuccess)
                return e;
            if (per_sm != 1) return cudaErrorLaunchOutOfResources;
            grid = nsm;
            grid_of[{dev, nch}] = grid;
        }
    }
    cudaLaunchConfig_t cfg = {};
    // SMs left to a collective that runs beside the selection (its kernel's CTAs would otherwise keep the
    // cooperative launch waiting for a CTA slot on every SM)
    if (spare_sms > 0) grid = grid - spare_sms > grid / 2 ? grid - spare_sms : grid / 2;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kSelThreads * kSelGroups);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

cudaError_t read_and_clear_select_error(int* flag) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_select_timeout, sizeof(int));
    if (e != cudaSuccess) return e;
    if (v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_select_timeout, &zero, sizeof(int));
    }
    *flag = v;
    return e;
}

cudaError_t launch_mask_to_lists(const float* mask, int heads, int nq, int nk, int32_t* kidx, int32_t* kcnt,
                                 cudaStream_t st) {
    const int rows = heads * nq;
    return launch_pdl(mask_to_lists_kernel, dim3((rows * 32 + 255) / 256), dim3(256), 0, st, mask, rows, nk, kidx,
                      kcnt);
}

cudaError_t launch_item_order(const int32_t* kcnt, int nq, int item_begin, int item_count, int32_t* order,
                              cudaStream_t st) {
    if (item_count <= 0) return cudaSuccess;
    const int h0 = item_begin / nq, h1 = (item_begin + item_count - 1) / nq;
    return launch_pdl(item_order_kernel, dim3(h1 - h0 + 1), dim3(256), 0, st, kcnt, nq, item_begin, item_count, order);
}

}  // namespace fvsr
