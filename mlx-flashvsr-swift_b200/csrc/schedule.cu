// schedule.cu — equal-work partition of an item range for the persistent attention kernel, and the merge of the
// items it splits.
//
// With few CTA waves (one GPU's share of a sharded problem) the per-item CTAs of the plain attention kernel are
// bounded by the longest key lists: in config 5, 62 % of the items are empty and the rest keep up to 198 key blocks,
// while an 8-GPU rank averages 147 blocks per SM. The schedule therefore concatenates the key lists of the range's
// non-empty items in item order (S blocks) and gives persistent CTA c the positions [c·Q, (c+1)·Q), Q = ceil(S / G):
// every CTA walks the same number of key blocks, as segments (item, first list position, length) of one to a few
// items. An item cut by a CTA boundary is computed in pieces whose partial results — fp32 O relative to the row
// maximum m (log2 units) and the row sum l — the combine kernel merges: O = Σ 2^(m_c − M) O_c / Σ 2^(m_c − M) l_c,
// M = max_c m_c. The combine kernel also writes the zeros of the empty items.
//
// Bounds (for the buffer size): segments ≤ non-empty items + G − 1; pieces of cut items ≤ 2·(G − 1); cut items ≤
// G − 1; empty items ≤ item_count.
#include <algorithm>

#include "common.cuh"

namespace fvsr {

namespace {

constexpr int kSchedThreads = 1024;

__device__ __forceinline__ int clamp_cnt(int c, int nk) { return c < 0 ? 0 : (c > nk ? nk : c); }

// Block-wide exclusive scan of three counters (kSchedThreads threads): on return a/b/c hold the exclusive prefixes
// and ta/tb/tc the totals. Uses sh[0, 192).
__device__ void block_scan3(long long& a, int& b, int& c, long long& ta, int& tb, int& tc, long long* shl, int* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    long long x = a;
    int y = b, z = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long xs = __shfl_up_sync(0xffffffffu, x, o);
        const int ys = __shfl_up_sync(0xffffffffu, y, o), zs = __shfl_up_sync(0xffffffffu, z, o);
        if (lane >= o) {
            x += xs;
            y += ys;
            z += zs;
        }
    }
    if (lane == 31) {
        shl[warp] = x;
        sh[warp] = y;
        sh[32 + warp] = z;
    }
    __syncthreads();
    if (warp == 0) {
        long long p = shl[lane];
        int q = sh[lane], r = sh[32 + lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long ps = __shfl_up_sync(0xffffffffu, p, o);
            const int qs = __shfl_up_sync(0xffffffffu, q, o), rs = __shfl_up_sync(0xffffffffu, r, o);
            if (lane >= o) {
                p += ps;
                q += qs;
                r += rs;
            }
        }
        shl[32 + lane] = p;
        sh[64 + lane] = q;
        sh[96 + lane] = r;
    }
    __syncthreads();
    const long long wa = warp ? shl[32 + warp - 1] : 0;
    const int wb = warp ? sh[64 + warp - 1] : 0, wc = warp ? sh[96 + warp - 1] : 0;
    ta = shl[32 + 31];
    tb = sh[64 + 31];
    tc = sh[96 + 31];
    a = wa + x - a;
    b = wb + y - b;
    c = wc + z - c;
    __syncthreads();
}

// Binary search over the items [lo, hi) of the range: the first i with P[i + 1] > x (P = exclusive block prefix).
__device__ __forceinline__ int first_ending_after(const int32_t* P, int lo, int hi, int x) {
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (P[mid + 1] > x) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

// One CTA. Per head of the range, the head's kept key blocks (its items' lists concatenated in item order) are cut
// into G equal shares; CTA c walks its share of the first head, then of the next, ... (segments in CTA-major, then
// head, then item order), so all CTAs work through the heads together and the K/V being read stays one head's.
__global__ void __launch_bounds__(kSchedThreads) schedule_kernel(const int32_t* __restrict__ kcnt, int nk, int nq,
                                                                 int item_begin, int item_count, int G, int Hr,
                                                                 int32_t* __restrict__ hdr,
                                                                 int32_t* __restrict__ seg_begin,
                                                                 int4* __restrict__ segs, int4* __restrict__ comb,
                                                                 int32_t* __restrict__ empties) {
    griddep_wait_then_release();
    extern __shared__ int32_t dsm[];
    int32_t* P = dsm;                       // [item_count + 1] exclusive kept-block prefix over the range
    int32_t* NE = P + item_count + 1;       // [item_count + 1] exclusive non-empty-item prefix
    int32_t* SB = NE + item_count + 1;      // [item_count] first piece slot of a cut item, else −1
    int32_t* PC = SB + item_count;          // [G·Hr] segments of (CTA c, head hh), then their first index
    __shared__ int32_t ha[64], qh[64];      // per head of the range: first item (range-relative), blocks per CTA
    __shared__ long long shl[64];
    __shared__ int sh[128];
    const int tid = threadIdx.x;
    const int per = (item_count + kSchedThreads - 1) / kSchedThreads;
    const int i0 = min(tid * per, item_count), i1 = min(i0 + per, item_count);
    // pass 1: block and non-empty prefixes; empty items
    long long pos = 0;
    int nne = 0, ne = 0;
    for (int i = i0; i < i1; ++i) {
        const int c = clamp_cnt(kcnt[item_begin + i], nk);
        pos += c;
        nne += c > 0;
        ne += c == 0;
    }
    long long S = 0;
    int NNE = 0, NEM = 0;
    block_scan3(pos, nne, ne, S, NNE, NEM, shl, sh);
    {
        long long p = pos;
        int q = nne;
        for (int i = i0; i < i1; ++i) {
            const int c = clamp_cnt(kcnt[item_begin + i], nk);
            P[i] = (int32_t)p;
            NE[i] = q;
            if (c == 0) empties[ne++] = item_begin + i;
            p += c;
            q += c > 0;
        }
        if (tid == kSchedThreads - 1) {
            P[item_count] = (int32_t)S;
            NE[item_count] = NNE;
        }
    }
    const int h0 = item_begin / nq;
    for (int hh = tid; hh < Hr; hh += kSchedThreads) ha[hh] = max(item_begin, (h0 + hh) * nq) - item_begin;
    if (tid == 0) ha[Hr] = item_count;
    __syncthreads();
    for (int hh = tid; hh < Hr; hh += kSchedThreads) {
        const int Sh = P[ha[hh + 1]] - P[ha[hh]];
        qh[hh] = Sh > 0 ? (Sh + G - 1) / G : 1;
    }
    __syncthreads();
    // pass 2: cut items (an item whose blocks reach two CTAs' shares of its head) and their piece slots
    int np = 0, nc = 0;
    for (int i = i0; i < i1; ++i) {
        const int c = clamp_cnt(kcnt[item_begin + i], nk);
        if (c == 0) continue;
        const int hh = (item_begin + i) / nq - h0;
        const int p = P[i] - P[ha[hh]];
        const int pieces = (p + c - 1) / qh[hh] - p / qh[hh] + 1;
        if (pieces > 1) {
            np += pieces;
            nc += 1;
        }
    }
    int n_parts = 0, n_comb = 0;
    {
        long long z = 0, zt = 0;
        block_scan3(z, np, nc, zt, n_parts, n_comb, shl, sh);
    }
    for (int i = i0; i < i1; ++i) {
        const int c = clamp_cnt(kcnt[item_begin + i], nk);
        SB[i] = -1;
        if (c == 0) continue;
        const int hh = (item_begin + i) / nq - h0;
        const int p = P[i] - P[ha[hh]];
        const int pieces = (p + c - 1) / qh[hh] - p / qh[hh] + 1;
        if (pieces > 1) {
            SB[i] = np;
            comb[nc++] = make_int4(item_begin + i, np, pieces, 0);
            np += pieces;
        }
    }
    // pass 3: segments per (CTA, head) pair, CTA-major
    const int npairs = G * Hr;
    const int pper = (npairs + kSchedThreads - 1) / kSchedThreads;
    const int t0 = min(tid * pper, npairs), t1 = min(t0 + pper, npairs);
    __syncthreads();
    auto pair_items = [&](int t, int& first, int& last, int& lo, int& hi, int& base_blocks, int& hh) -> bool {
        const int c = t / Hr;
        hh = t % Hr;
        base_blocks = P[ha[hh]];
        const int Sh = P[ha[hh + 1]] - base_blocks;
        lo = c * qh[hh];
        hi = min((c + 1) * qh[hh], Sh);
        if (lo >= hi) return false;
        first = first_ending_after(P, ha[hh], ha[hh + 1], base_blocks + lo);
        last = first_ending_after(P, ha[hh], ha[hh + 1], base_blocks + hi - 1);
        return true;
    };
    long long nsl = 0;
    for (int t = t0; t < t1; ++t) {
        int first, last, lo, hi, bb, hh;
        const int n = pair_items(t, first, last, lo, hi, bb, hh) ? NE[last + 1] - NE[first] : 0;
        PC[t] = n;
        nsl += n;
    }
    long long n_segs_l = 0;
    {
        int z0 = 0, z1 = 0, zt0 = 0, zt1 = 0;
        block_scan3(nsl, z0, z1, n_segs_l, zt0, zt1, shl, sh);
    }
    const int n_segs = (int)n_segs_l;
    {
        int base = (int)nsl;
        for (int t = t0; t < t1; ++t) {
            const int n = PC[t];
            if (t % Hr == 0) seg_begin[t / Hr] = base;
            int first, last, lo, hi, bb, hh;
            if (n > 0 && pair_items(t, first, last, lo, hi, bb, hh)) {
                const int c = t / Hr;
                for (int i = first; i <= last; ++i) {
                    const int cnt = P[i + 1] - P[i];
                    if (cnt == 0) continue;
                    const int pi = P[i] - bb;
                    const int a = max(lo, pi), b = min(hi, pi + cnt);
                    const int slot = SB[i] >= 0 ? SB[i] + (c - pi / qh[hh]) : -1;
                    segs[base++] = make_int4(item_begin + i, a - pi, b - a, slot);
                }
            }
        }
    }
    if (tid == 0) {
        seg_begin[G] = n_segs;
        hdr[0] = n_segs;
        hdr[1] = n_comb;
        hdr[2] = n_parts;
        hdr[3] = Hr;
        hdr[4] = NEM;
    }
}

// CTA b < n_comb merges cut item b; CTA n_comb + e writes the zeros of empty item e (SparseAttention.swift:47-53);
// the rest exit. Thread t: row t/2, output columns [64·(t%2), 64·(t%2) + 64).
__global__ void __launch_bounds__(256) combine_kernel(const int32_t* __restrict__ hdr, const int4* __restrict__ comb,
                                                      const int32_t* __restrict__ empties,
                                                      const float* __restrict__ opart, const float* __restrict__ ml,
                                                      int heads, int nq, __nv_bfloat16* __restrict__ out) {
    griddep_wait_then_release();
    const int n_comb = hdr[1], n_empty = hdr[4];
    const int b = blockIdx.x;
    if (b >= n_comb + n_empty) return;
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    const int64_t ld = (int64_t)heads * kD;
    if (b >= n_comb) {
        const int item = empties[b - n_comb];
        const int h = item / nq, qb = item % nq;
        uint4* orow = reinterpret_cast<uint4*>(out + ((int64_t)qb * kBlock + r) * ld + h * kD + 64 * half);
#pragma unroll
        for (int i = 0; i < 8; ++i) orow[i] = make_uint4(0, 0, 0, 0);
        return;
    }
    const int4 cr = comb[b];
    const int item = cr.x, p0 = cr.y, ch = cr.z;
    const int h = item / nq, qb = item % nq;
    float M = -INFINITY;
    for (int c = 0; c < ch; ++c) M = fmaxf(M, ml[(int64_t)(p0 + c) * 256 + r]);
    float den = 0.f;
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    for (int c = 0; c < ch; ++c) {
        const int64_t s = p0 + c;
        const float w = exp2f(ml[s * 256 + r] - M);
        den = fmaf(w, ml[s * 256 + 128 + r], den);
        const float4* src = reinterpret_cast<const float4*>(opart + (s * kBlock + r) * kD + 64 * half);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float4 o = src[i];
            acc[4 * i] = fmaf(w, o.x, acc[4 * i]);
            acc[4 * i + 1] = fmaf(w, o.y, acc[4 * i + 1]);
            acc[4 * i + 2] = fmaf(w, o.z, acc[4 * i + 2]);
            acc[4 * i + 3] = fmaf(w, o.w, acc[4 * i + 3]);
        }
    }
    const float inv = 1.0f / den;
    uint4* orow = reinterpret_cast<uint4*>(out + ((int64_t)qb * kBlock + r) * ld + h * kD + 64 * half);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 v2 = __floats2bfloat162_rn(acc[8 * i + 2 * k] * inv, acc[8 * i + 2 * k + 1] * inv);
            w[k] = *reinterpret_cast<const uint32_t*>(&v2);
        }
        orow[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace

SchedLayout sched_layout(int item_count, int nq, int heads, int G) {
    auto a = [](size_t x) { return (x + 255) & ~size_t(255); };
    SchedLayout L = {};
    L.G = G;
    L.item_count = item_count;
    // heads a range of item_count items can touch, wherever it starts
    L.Hr = item_count > 0 ? std::min(heads, (item_count - 1) / nq + 2) : 1;
    L.persistent = item_count > 0 && item_count <= kPersistItemsPerSm * G && item_count <= kSchedItemCap &&
                   L.Hr <= kSchedHeadCap && G * L.Hr <= kSchedPairCap;  // room for the persistent partition
    L.max_segs = item_count + G * L.Hr;
    L.max_parts = 2 * G * L.Hr;
    L.max_comb = G * L.Hr;
    size_t off = 0;
    L.off_hdr = off;
    off += a(8 * sizeof(int32_t));
    L.off_order = off;  // longest-first item order (non-persistent mode)
    off += a((size_t)(item_count > 0 ? item_count : 1) * sizeof(int32_t));
    if (L.persistent) {
        L.off_seg_begin = off;
        off += a((size_t)(G + 1) * sizeof(int32_t));
        L.off_segs = off;
        off += a((size_t)L.max_segs * sizeof(int4));
        L.off_comb = off;
        off += a((size_t)L.max_comb * sizeof(int4));
        L.off_empties = off;
        off += a((size_t)item_count * sizeof(int32_t));
        L.off_ml = off;
        off += a((size_t)L.max_parts * 256 * sizeof(float));
        L.off_opart = off;
        off += a((size_t)L.max_parts * kBlock * kD * sizeof(float));
    }
    L.bytes = off;
    return L;
}

bool sched_persistent(const SchedLayout& L, int item_begin, int nq) {
    return L.persistent && item_begin / nq == (item_begin + L.item_count - 1) / nq;
}

cudaError_t launch_schedule(const int32_t* kcnt, int nk, int nq, int item_begin, int item_count,
                            const SchedLayout& L, void* buf, cudaStream_t st) {
    uint8_t* b = static_cast<uint8_t*>(buf);
    if (!sched_persistent(L, item_begin, nq))
        return launch_item_order(kcnt, nq, item_begin, item_count, reinterpret_cast<int32_t*>(b + L.off_order), st);
    const int Hr = (item_begin + item_count - 1) / nq - item_begin / nq + 1;  // <= L.Hr
    const size_t smem = sizeof(int32_t) * (3 * (size_t)item_count + 2 + (size_t)L.G * Hr);
    cudaError_t e = cudaFuncSetAttribute(schedule_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(schedule_kernel, dim3(1), dim3(kSchedThreads), smem, st, kcnt, nk, nq, item_begin, item_count,
                      L.G, Hr, reinterpret_cast<int32_t*>(b + L.off_hdr),
                      reinterpret_cast<int32_t*>(b + L.off_seg_begin), reinterpret_cast<int4*>(b + L.off_segs),
                      reinterpret_cast<int4*>(b + L.off_comb), reinterpret_cast<int32_t*>(b + L.off_empties));
}

cudaError_t launch_combine(const SchedLayout& L, const void* buf, int heads, int nq, void* out, cudaStream_t st) {
    const uint8_t* b = static_cast<const uint8_t*>(buf);
    return launch_pdl(combine_kernel, dim3(L.max_comb + L.item_count), dim3(256), 0, st,
                      reinterpret_cast<const int32_t*>(b + L.off_hdr), reinterpret_cast<const int4*>(b + L.off_comb),
                      reinterpret_cast<const int32_t*>(b + L.off_empties),
                      reinterpret_cast<const float*>(b + L.off_opart), reinterpret_cast<const float*>(b + L.off_ml),
                      heads, nq, static_cast<__nv_bfloat16*>(out));
}

}  // namespace fvsr
