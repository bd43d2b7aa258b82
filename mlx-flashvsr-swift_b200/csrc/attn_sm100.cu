// attn_sm100.cu — bf16 block-sparse flash attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the Metal kernel of SparseAttention.swift:17-153 (one threadgroup per (query block, head), walking only the
// selected key blocks by index with an fp32 online softmax; an empty query block writes zeros).
//
// One CTA per (head, query block) work item, ordered head-major so the CTAs in flight share one head's K/V in L2.
// Warp roles (320 threads):
//   warp 0      TMA producer: the Q tile, then the K and V tiles of each kept key block into a 3-slot K ring (a slot
//               frees when its S MMA completes) and a 2-slot V ring (freed when its PV MMA completes); the releases
//               reuse the S-full and PV-done barriers, so each key block costs two tcgen05.commit.
//   warp 1      TMEM owner + single-thread MMA issuer: S_j = Q·K_jᵀ (SS-MMA, 128×128×128) is issued two blocks
//               ahead of O += P_j·V_j (TS-MMA: P read from TMEM, V from shared memory as an MN-major operand), so two
//               S tiles are queued on the tensor core while the softmax of block j is in flight.
//   warps 2..9  softmax, two sets of four warps (one warp per TMEM lane quarter each): set 0 takes the even key
//               blocks, set 1 the odd ones, so two blocks are in flight on every SM sub-partition. Thread = query row
//               = TMEM lane. Per block: row maximum from S_j, the running maximum handed over from the other set
//               (raised, and O rescaled in TMEM, only when it grew by more than 2^8 — lazy rescaling), exp2 on the
//               MUFU pipe, P_j (bf16) written over the first half of S_j's TMEM columns. Each set keeps its own
//               partial row sum; at the end the two are combined and O is normalised and stored.
// TMEM (512 columns): O [0,128), S0/P0 [128,256), S1/P1 [256,384), S2/P2 [384,512).
// Shared memory: Q 32 KB + K 3 × 32 KB + V 2 × 32 KB, each tile as two 128-row × 64-column boxes in the 128-byte
// swizzled layout that TMA writes and the MMA descriptors read.
// Every wait is bounded (4 s); on expiry the kernel raises a device timeout word that fvsr_device_check reports.
#include "common.cuh"
#include "sm100.cuh"

namespace fvsr {

__device__ int g_fvsr_timeout = 0;

namespace {

using namespace sm100;

constexpr int kKSlots = 3;                        // K ring: a slot frees as soon as S_j = Q·K_jᵀ has completed
constexpr int kVSlots = 2;                        // V ring: a slot frees when O += P_j·V_j has completed
constexpr int kSBufs = 3;                         // S/P buffers in TMEM: S_{j+1} and S_{j+2} queue behind PV_j
constexpr uint32_t kTileBytes = kBlock * kD * 2;  // 32 KB bf16 tile
constexpr uint32_t kBoxBytes = kTileBytes / 2;    // one 128 × 64 box
// TMEM columns: O (fp32 128) then three S buffers (fp32 128 each); P_j (bf16 pairs) overwrites the first 64
// columns of its own S buffer once its row maximum is known.
constexpr uint32_t kColO = 0, kColS0 = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr int kThreads = 320;  // 2 role warps + 2 softmax sets of 4 warps

// Lazy rescaling: a row's running maximum (log2 units) is only raised — and O rescaled — when the block maximum
// exceeds it by more than this; otherwise P entries may reach 2^8, which bf16 P and fp32 O/l carry exactly as well.
constexpr float kRescaleThreshold = 8.0f;

constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128, 0, 0);   // A = Q, B = K (both K-major shared memory)
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, 0, 1);  // A = P (TMEM), B = V (MN-major shared memory)

// Shared-memory map (offsets from a 1024-byte aligned base).
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kTileBytes;                          // K slot i at kOffK + i·kTileBytes
constexpr uint32_t kOffV = kOffK + kKSlots * kTileBytes;        // V slot i at kOffV + i·kTileBytes
constexpr uint32_t kOffBar = kOffV + kVSlots * kTileBytes;      // barriers
// A K slot frees when its S MMA completes and a V slot when its PV MMA completes, which the S-full and PV-done
// barriers already signal, so the producer waits on those (K slot j%3 ↔ S buffer j%3, V slot j%2 ↔ PV barrier j%2):
// two tcgen05.commit per key block instead of four. Neither barrier can run a phase ahead of the producer's wait,
// because the next completion on it needs the tile the producer has not loaded yet.
static_assert(kKSlots == kSBufs && kVSlots == 2, "ring slots are released through the S and PV barriers");
constexpr int kBarQ = 0, kBarKF = 1, kBarVF = kBarKF + kKSlots, kBarSF = kBarVF + kVSlots, kBarPF = kBarSF + kSBufs,
              kBarPV = kBarPF + kSBufs, kBarM = kBarPV + 2, kBarFin = kBarM + 2, kBarDone = kBarFin + 1,
              kNumBars = kBarDone + 1;
constexpr uint32_t kOffTmemSlot = kOffBar + 8 * kNumBars;
constexpr uint32_t kOffAbort = kOffTmemSlot + 4;
constexpr uint32_t kOffM = (kOffAbort + 4 + 15) & ~15u;         // running max handoff: [2 parities][128] f32
constexpr uint32_t kOffFin = kOffM + 2 * 128 * 4;               // final (l, m_ref) of each set: [2][2][128] f32
constexpr uint32_t kOffList = kOffFin + 2 * 2 * 128 * 4;

struct AttnArgs {
    const int32_t* kidx;
    const int32_t* kcnt;
    __nv_bfloat16* out;
    int heads, nq, nk;
    int item_begin;
    const int32_t* order;  // optional item order (longest first within each head); NULL = ascending
    float scale_log2;
    KvPages pages;
    OutRows rows;
    AttnSplit split;
};

__global__ void __launch_bounds__(kThreads, 1)
    attn_bf16_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmKn,
                           const __grid_constant__ CUtensorMap tmVn, const AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    griddep_wait_then_release();
    const int item = a.order ? a.order[blockIdx.x] : a.item_begin + (int)blockIdx.x;
    const int h = item / a.nq, qb = item % a.nq;
    const int64_t ld = (int64_t)a.heads * kD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int cnt = a.kcnt ? a.kcnt[item] : a.nk;  // no lists: dense (every key block, in order)
    cnt = cnt < 0 ? 0 : (cnt > a.nk ? a.nk : cnt);
    int lo = 0;  // first list entry this launch walks
    const size_t slot = blockIdx.x;
    if (a.split.part != 0 && a.kidx) {
        // the list is ascending, so its blocks below split_nk are a prefix: count it with the whole CTA
        const int32_t* gl = a.kidx + (int64_t)item * a.nk;
        int c1 = 0;
        for (int j0 = 0; j0 < cnt; j0 += kThreads) {
            const int j = j0 + (int)threadIdx.x;
            c1 += __syncthreads_count(j < cnt && gl[j] < a.split.split_nk);
        }
        lo = a.split.part == 1 ? 0 : c1;
        cnt = a.split.part == 1 ? c1 : cnt - c1;
    }

    if (cnt == 0) {
        if (a.split.part == 1) {  // nothing below the split: an empty partial (row sum 0, row maximum −inf)
            float4* po = reinterpret_cast<float4*>(a.split.part_o + slot * kBlock * kD);
            for (int idx = threadIdx.x; idx < kBlock * kD / 4; idx += kThreads) po[idx] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = threadIdx.x; r < kBlock; r += kThreads) {
                a.split.part_ml[(slot * kBlock + r) * 2] = -INFINITY;
                a.split.part_ml[(slot * kBlock + r) * 2 + 1] = 0.0f;
            }
            return;
        }
        if (a.split.part == 2) {  // nothing from the split on: the first part's result alone (zeros if it was empty)
            for (int idx = threadIdx.x; idx < kBlock * 16; idx += kThreads) {
                const int r = idx >> 4, c = idx & 15;
                const float l = a.split.part_ml[(slot * kBlock + r) * 2 + 1];
                const float inv = l > 0.0f ? 1.0f / l : 0.0f;
                const float4* po = reinterpret_cast<const float4*>(a.split.part_o + (slot * kBlock + r) * kD + c * 8);
                const float4 x0 = po[0], x1 = po[1];
                *reinterpret_cast<uint4*>(a.out + a.rows.row(qb, r) * ld + h * kD + c * 8) =
                    make_uint4(pack_bf16x2(x0.x * inv, x0.y * inv), pack_bf16x2(x0.z * inv, x0.w * inv),
                               pack_bf16x2(x1.x * inv, x1.y * inv), pack_bf16x2(x1.z * inv, x1.w * inv));
            }
            return;
        }
        // SparseAttention.swift:47-53: a query block that selected nothing writes zeros
        for (int idx = threadIdx.x; idx < kBlock * 16; idx += kThreads) {
            const int r = idx >> 4, c = idx & 15;
            *reinterpret_cast<uint4*>(a.out + a.rows.row(qb, r) * ld + h * kD + c * 8) = make_uint4(0, 0, 0, 0);
        }
        return;
    }

    volatile uint32_t* abort_word = reinterpret_cast<volatile uint32_t*>(smem + kOffAbort);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);
    int32_t* s_list = reinterpret_cast<int32_t*>(smem + kOffList);
    auto bar = [&](int i) { return sbase + kOffBar + 8u * (uint32_t)i; };
    auto wait = [&](int b, uint32_t parity) { return mbar_wait(bar(b), parity & 1u, abort_word, &g_fvsr_timeout, kWaitLimitNs); };

    if (threadIdx.x == 0) {
        mbar_init(bar(kBarQ), 1);
        for (int i = 0; i < kKSlots; ++i) mbar_init(bar(kBarKF + i), 1);
        for (int i = 0; i < kVSlots; ++i) mbar_init(bar(kBarVF + i), 1);
        for (int b = 0; b < kSBufs; ++b) {
            mbar_init(bar(kBarSF + b), 1);
            mbar_init(bar(kBarPF + b), 128);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(kBarPV + b), 1);
            mbar_init(bar(kBarM + b), 128);
        }
        mbar_init(bar(kBarFin), 256);
        mbar_init(bar(kBarDone), 1);
        *abort_word = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        prefetch_tmap(&tmKn);
        prefetch_tmap(&tmVn);
    }
    const int32_t* glist = a.kidx ? a.kidx + (int64_t)item * a.nk + lo : nullptr;
    for (int j = threadIdx.x; j < cnt; j += kThreads) {
        int kb = glist ? glist[j] : lo + j;
        kb = kb < 0 ? 0 : (kb >= a.nk ? a.nk - 1 : kb);
        s_list[j] = kv_phys_block(a.pages, kb);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer: Q, then K and V in the order the MMA issuer consumes them ----------------
        if (lane == 0) {
            const int x0 = h * kD;
            mbar_expect_tx(bar(kBarQ), kTileBytes);
            const int qy = (int)a.rows.q_row(qb);
            tma_load_2d(sbase + kOffQ, &tmQ, x0, qy, bar(kBarQ));
            tma_load_2d(sbase + kOffQ + kBoxBytes, &tmQ, x0 + 64, qy, bar(kBarQ));
            auto load_k = [&](int j) -> bool {
                const int ks = j % kKSlots;
                if (j >= kKSlots && !wait(kBarSF + ks, (uint32_t)(j / kKSlots - 1))) return false;  // S_{j−3} done
                const uint32_t dk = sbase + kOffK + (uint32_t)ks * kTileBytes;
                mbar_expect_tx(bar(kBarKF + ks), kTileBytes);
                const bool fresh = (s_list[j] & kFreshPage) != 0;  // a block of the slice being appended
                const CUtensorMap* mk = fresh ? &tmKn : &tmK;
                const int ky = (s_list[j] & ~kFreshPage) * kBlock;
                tma_load_2d(dk, mk, x0, ky, bar(kBarKF + ks));
                tma_load_2d(dk + kBoxBytes, mk, x0 + 64, ky, bar(kBarKF + ks));
                return true;
            };
            auto load_v = [&](int j) -> bool {
                const int vs = j % kVSlots;
                if (j >= kVSlots && !wait(kBarPV + vs, (uint32_t)(j / kVSlots - 1))) return false;  // PV_{j−2} done
                const uint32_t dv = sbase + kOffV + (uint32_t)vs * kTileBytes;
                mbar_expect_tx(bar(kBarVF + vs), kTileBytes);
                const bool fresh = (s_list[j] & kFreshPage) != 0;
                const CUtensorMap* mv = fresh ? &tmVn : &tmV;
                const int vy = (s_list[j] & ~kFreshPage) * kBlock;
                tma_load_2d(dv, mv, x0, vy, bar(kBarVF + vs));
                tma_load_2d(dv + kBoxBytes, mv, x0 + 64, vy, bar(kBarVF + vs));
                return true;
            };
            bool ok = load_k(0) && (cnt < 2 || load_k(1));
            for (int j = 0; ok && j < cnt; ++j) ok = load_v(j) && (j + 2 >= cnt || load_k(j + 2));
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread): S_{j+2} and S_{j+1} queued ahead of O += P_j·V_j ----------------
        if (lane == 0) {
            bool ok = wait(kBarQ, 0);
            auto issue_s = [&](int j) -> bool {
                const int ks = j % kKSlots;
                if (!wait(kBarKF + ks, (uint32_t)(j / kKSlots))) return false;
                tc_fence_after();
                const uint32_t d = tmem + kColS0 + 128u * (uint32_t)(j % kSBufs);
                // descriptors advance by byte offset >> 4 in their start-address field (no carry: smem < 256 KB)
                const uint64_t qd = smem_desc(sbase + kOffQ, 16, 1024);
                const uint64_t kd = smem_desc(sbase + kOffK + (uint32_t)ks * kTileBytes, 16, 1024);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = ((uint32_t)(kk >> 2) * kBoxBytes + (uint32_t)(kk & 3) * 32u) >> 4;
                    mma_ss(d, qd + off, kd + off, kIdescS, kk > 0 ? 1u : 0u);
                }
                mma_commit(bar(kBarSF + j % kSBufs));
                return true;
            };
            if (ok) ok = issue_s(0) && (cnt < 2 || issue_s(1));
            for (int j = 0; ok && j < cnt; ++j) {
                // S_{j+2} lands in the buffer that held P_{j−1}; PV_{j−1} was issued before it, and tcgen05 MMAs of
                // one thread execute in issue order
                if (j + 2 < cnt && !issue_s(j + 2)) break;
                const int vs = j % kVSlots;
                if (!wait(kBarVF + vs, (uint32_t)(j / kVSlots))) break;
                if (!wait(kBarPF + j % kSBufs, (uint32_t)(j / kSBufs))) break;
                tc_fence_after();
                const uint64_t vd = smem_desc(sbase + kOffV + (uint32_t)vs * kTileBytes, kBoxBytes, 1024);
                const uint32_t pa = tmem + kColS0 + 128u * (uint32_t)(j % kSBufs);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    mma_ts(tmem + kColO, pa + 8u * (uint32_t)kk, vd + (uint64_t)(kk * (2048 >> 4)), kIdescPV,
                           (j > 0 || kk > 0) ? 1u : 0u);
                mma_commit(bar(kBarPV + (j & 1)));
                if (j == cnt - 1) mma_commit(bar(kBarDone));  // every MMA done: a single-phase barrier
            }
        }
    } else {
        // ---------------- softmax: set `st` handles blocks j ≡ st (mod 2), thread = query row ----------------
        const int st = (warp - 2) >> 2;
        const int quarter = warp & 3;  // TMEM lanes [32·quarter, 32·quarter + 32) are this warp's
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
        float* m_x = reinterpret_cast<float*>(smem + kOffM);
        float* fin = reinterpret_cast<float*>(smem + kOffFin);
        const float sl2 = a.scale_log2;
        float l = 0.0f, mref = -INFINITY;  // this set's partial row sum and the maximum it is relative to
        bool ok = true;
        auto wait_warp = [&](int b, uint32_t parity) { return __all_sync(0xffffffffu, wait(b, parity)); };
        for (int j = st; j < cnt; j += 2) {
            if (!wait_warp(kBarSF + j % kSBufs, (uint32_t)(j / kSBufs))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sbuf = lane_base + kColS0 + 128u * (uint32_t)(j % kSBufs);
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
            // running maximum after block j−1 comes from the other set (block j−1 is theirs)
            float m_prev = -INFINITY;
            if (j > 0) {
                if (!wait_warp(kBarM + ((j - 1) & 1), (uint32_t)((j - 1) >> 1))) {
                    ok = false;
                    break;
                }
                m_prev = m_x[((j - 1) & 1) * 128 + r];
            }
            const bool need = mx > m_prev + kRescaleThreshold;  // always true on block 0 (m_prev = −inf)
            const float m_j = need ? fmaxf(m_prev, mx) : m_prev;
            m_x[(j & 1) * 128 + r] = m_j;
            mbar_arrive(bar(kBarM + (j & 1)));  // published before the exponentials so block j+1 can start
            const float neg = -m_j;
            float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {  // 32 key columns → 16 packed P columns per store
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
            if (m_j != mref) {  // bring this set's partial sum to the current maximum
                l *= ex2_approx(mref - m_j);
                mref = m_j;
            }
            l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
            if (j > 0 && __any_sync(0xffffffffu, need)) {
                // after the P stores (S_j's registers are free by now): O holds Σ_{i<j} P_i·V_i relative to
                // m_prev once PV_{j−1} has completed; bring it to m_j
                if (!wait_warp(kBarPV + ((j - 1) & 1), (uint32_t)((j - 1) >> 1))) {
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
            mbar_arrive(bar(kBarPF + j % kSBufs));
        }
        // the row sum: both sets' partial sums brought to the final maximum (the larger m_ref), added in set order
        fin[(st * 2) * 128 + r] = l;
        fin[(st * 2 + 1) * 128 + r] = mref;
        mbar_arrive(bar(kBarFin));
        if (ok) ok = wait_warp(kBarFin, 0);
        // the last PV on a single-phase barrier: a parity wait for PV_{cnt−1} on the alternating PV barriers would pass
        // early if PV_{cnt−3} had not completed yet
        if (ok && wait_warp(kBarDone, 0)) {
            tc_fence_after();
            const float l0 = fin[r], m0 = fin[128 + r], l1 = fin[256 + r], m1 = fin[384 + r];
            const float mf = fmaxf(m0, m1);
            const float l_row = l0 * ex2_approx(m0 - mf) + l1 * ex2_approx(m1 - mf);
            if (a.split.part == 1) {  // unnormalised O (relative to mf), the row maximum and sum: the partial
                float* po = a.split.part_o + (slot * kBlock + r) * kD + 64 * st;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t ov[32];
                    tmem_ld32(lane_base + kColO + 64u * (uint32_t)st + 32u * c, ov);
                    tmem_ld_wait(ov);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        reinterpret_cast<float4*>(po + 32 * c)[i] =
                            make_float4(__uint_as_float(ov[4 * i]), __uint_as_float(ov[4 * i + 1]),
                                        __uint_as_float(ov[4 * i + 2]), __uint_as_float(ov[4 * i + 3]));
                }
                if (st == 0) {
                    a.split.part_ml[(slot * kBlock + r) * 2] = mf;
                    a.split.part_ml[(slot * kBlock + r) * 2 + 1] = l_row;
                }
            } else {
                // part 2 merges the first part's partial: O = (O_a·2^(m_a−M) + O_b·2^(m_b−M)) / (l_a·… + l_b·…)
                float ca = 0.0f, cb = 1.0f, lt = l_row;
                const float* pa = nullptr;
                if (a.split.part == 2) {
                    const float ma = a.split.part_ml[(slot * kBlock + r) * 2];
                    const float la = a.split.part_ml[(slot * kBlock + r) * 2 + 1];
                    const float big = fmaxf(ma, mf);
                    ca = la > 0.0f ? ex2_approx(ma - big) : 0.0f;
                    cb = ex2_approx(mf - big);
                    lt = la * ca + l_row * cb;
                    pa = a.split.part_o + (slot * kBlock + r) * kD + 64 * st;
                }
                const float inv = 1.0f / lt;
                __nv_bfloat16* orow = a.out + a.rows.row(qb, r) * ld + h * kD + 64 * st;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t ov[32];
                    tmem_ld32(lane_base + kColO + 64u * (uint32_t)st + 32u * c, ov);
                    tmem_ld_wait(ov);
                    if (pa) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 x = reinterpret_cast<const float4*>(pa + 32 * c)[i];
                            ov[4 * i] = __float_as_uint(fmaf(x.x, ca, __uint_as_float(ov[4 * i]) * cb));
                            ov[4 * i + 1] = __float_as_uint(fmaf(x.y, ca, __uint_as_float(ov[4 * i + 1]) * cb));
                            ov[4 * i + 2] = __float_as_uint(fmaf(x.z, ca, __uint_as_float(ov[4 * i + 2]) * cb));
                            ov[4 * i + 3] = __float_as_uint(fmaf(x.w, ca, __uint_as_float(ov[4 * i + 3]) * cb));
                        }
                    }
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        w[i] = pack_bf16x2(__uint_as_float(ov[2 * i]) * inv, __uint_as_float(ov[2 * i + 1]) * inv);
                    uint4* dst = reinterpret_cast<uint4*>(orow + 32 * c);
#pragma unroll
                    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

size_t attn_bf16_smem_bytes(int nk) { return 1024 + kOffList + sizeof(int32_t) * (size_t)nk; }

cudaError_t launch_attn_bf16(const void* q, const void* k, const void* v, int64_t kv_rows, const KvPages& pages,
                             int heads, int nq, int nk, const int32_t* kidx, const int32_t* kcnt, void* out,
                             int item_begin, int item_count, const int32_t* order, cudaStream_t st, OutRows rows,
                             AttnSplit split, FreshKv fresh) {
    if (item_count <= 0) return cudaSuccess;
    CUtensorMap mq, mk, mv, mkn, mvn;
    const int64_t channels = (int64_t)heads * kD;
    const int64_t q_rows = (int64_t)(rows.q_blocks > 0 ? rows.q_blocks : nq) * kBlock;
    if (!make_tile_map(&mq, q, q_rows, channels) || !make_tile_map(&mk, k, kv_rows, channels) ||
        !make_tile_map(&mv, v, kv_rows, channels))
        return cudaErrorInvalidValue;
    if (fresh.k) {
        if (!make_tile_map(&mkn, fresh.k, fresh.rows, channels) || !make_tile_map(&mvn, fresh.v, fresh.rows, channels))
            return cudaErrorInvalidValue;
    } else {  // no page is marked fresh: the maps are never read
        mkn = mk;
        mvn = mv;
    }
    const size_t smem = attn_bf16_smem_bytes(nk);
    cudaError_t e = cudaFuncSetAttribute(attn_bf16_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    AttnArgs a;
    a.kidx = kidx;
    a.kcnt = kcnt;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.heads = heads;
    a.nq = nq;
    a.nk = nk;
    a.item_begin = item_begin;
    a.order = order;
    a.scale_log2 = (1.0f / sqrtf((float)kD)) * 1.4426950408889634f;
    a.pages = pages;
    a.rows = rows;
    a.split = split;
    return launch_pdl(attn_bf16_sm100_kernel, dim3(item_count), dim3(kThreads), smem, st, mq, mk, mv, mkn, mvn, a);
}

namespace {

// The failure path of the bounded waits, without a fault: one thread waits, with mbar_wait and the attention kernel's
// timeout word, on an mbarrier whose single expected arrival never comes. The wait gives up after limit_ns, raises
// the CTA abort word and the device timeout word, and the kernel returns normally.
__global__ void wait_probe_kernel(uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t abort_word;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_word = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        mbar_wait(smem_u32(&bar), 0, reinterpret_cast<volatile uint32_t*>(&abort_word), &g_fvsr_timeout, limit_ns);
    __syncthreads();
}

}  // namespace

cudaError_t launch_wait_probe(uint64_t limit_ns, cudaStream_t st) {
    wait_probe_kernel<<<1, 32, 0, st>>>(limit_ns);
    return cudaGetLastError();
}

cudaError_t read_and_clear_device_error(int* flag, cudaStream_t st) {
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return e;
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, g_fvsr_timeout, sizeof(int));
    if (e != cudaSuccess) return e;
    if (v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_fvsr_timeout, &zero, sizeof(int));
        if (e != cudaSuccess) return e;
    }
    int vp = 0, vs = 0, vg = 0;
    e = read_and_clear_persist_error(&vp);
    if (e == cudaSuccess) e = read_and_clear_select_error(&vs);
    if (e == cudaSuccess) e = read_and_clear_gemm_error(&vg);
    *flag = v | vp | vs | vg;
    return e;
}

}  // namespace fvsr
