// common.cuh — shared definitions of the sm_100a LCSA kernels (internal; the public surface is include/fvsr_lcsa.h).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fvsr {

constexpr int kBlock = 128;  // tokens per window / block (DiT.swift:113-118)
constexpr int kD = 128;      // head dim (SparseAttention.swift:173)
constexpr int kMaxPages = 32;

// Logical key block j lives at physical block page_block[j / s] + j % s of the K/V arena (a contiguous K/V buffer is
// the identity table). Used by the attention and selection kernels to read the paged streaming cache in place.
struct KvPages {
    int32_t page_block[kMaxPages];
    int32_t s;  // blocks per page (spatial blocks per temporal slice)
};

__host__ __device__ inline int32_t kv_phys_block(const KvPages& pg, int32_t j) {
    return pg.page_block[j / pg.s] + j % pg.s;
}
// A page entry with this bit set names a slice being appended by the same call: the bf16 attention reads its key and
// value blocks (the entry without the bit, plus the block's index in the slice) from the caller's k_new / v_new
// (FreshKv) instead of the arena, so the copy into the arena can run beside it.
constexpr int32_t kFreshPage = 1 << 30;
struct FreshKv {
    const void* k = nullptr;  // (rows, channels) window order, or NULL: no fresh pages
    const void* v = nullptr;
    int64_t rows = 0;
};

// Token r of window (query block) w on the (F, 8·bh, 8·bw) patch grid (windowPartition, DiT.swift:113-118): windows
// ordered (nf, nh, nw), tokens inside a window (wf, wh, ww). token_row gives the token-order row (the layout
// windowReverse, DiT.swift:121-126, restores).
__host__ __device__ __forceinline__ int64_t token_row(int bh, int bw, int w, int r) {
    const int s = bh * bw, nf = w / s, rem = w - nf * s, nh = rem / bw, nw = rem - nh * bw;
    const int wf = r >> 6, wh = (r >> 3) & 7, ww = r & 7;
    return ((int64_t)(2 * nf + wf) * (8 * bh) + 8 * nh + wh) * (8 * bw) + 8 * nw + ww;
}

// Where the attention reads query block qb and writes its output row r: window order (bw == 0), with q and out
// holding the query blocks [qbase, qbase + q_blocks) (a rank's shard; q_blocks = 0 means all of them, qbase 0), or
// token order (windowReverse fused into the epilogue; whole chunk only).
struct OutRows {
    int bh = 0, bw = 0;
    int qbase = 0, q_blocks = 0;
    __device__ __forceinline__ int64_t row(int qb, int r) const {
        return bw == 0 ? (int64_t)(qb - qbase) * kBlock + r : token_row(bh, bw, qb, r);
    }
    __device__ __forceinline__ int64_t q_row(int qb) const { return (int64_t)(qb - qbase) * kBlock; }
};

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// Programmatic dependent launch: every kernel of the path first waits for the kernel before it in the stream to have
// completed (griddepcontrol.wait — a hardware wait, and a no-op when launched without the attribute), then lets the
// next kernel start launching, so launch latency and CTA ramp-up overlap the previous kernel's tail.
__device__ __forceinline__ void griddep_wait_then_release() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---- launchers (each returns the launch's cudaError_t) ----
cudaError_t launch_pool(const void* x, int dtype, int64_t nblocks, int channels, float* out, void* copy_dst,
                        cudaStream_t st);
// The cache append in one launch: nblocks new key/value blocks (k_new, v_new, window order) are copied to arena blocks
// dst.page_block[b / dst.s] + b % dst.s of k_arena / v_arena and the keys pooled into pk_arena (same arena blocks).
cudaError_t launch_append(const void* k_new, const void* v_new, int dtype, int64_t nblocks, int channels,
                          const KvPages& dst, void* k_arena, void* v_arena, float* pk_arena, cudaStream_t st);
// Pools two tensors (n1 and n2 blocks) in one launch; also clears zero_words 32-bit words at `zero` (the selection's
// histograms, which the next kernels accumulate into).
cudaError_t launch_pool2(const void* x1, int64_t n1, float* out1, void* copy_dst, const void* x2, int64_t n2,
                         float* out2, int dtype, int channels, cudaStream_t st, uint32_t* zero = nullptr,
                         size_t zero_words = 0);
// The whole selection on pooled inputs in one cooperative launch (select.cu): scores, softmax (probs, in place),
// the exact per-(head, query slice) threshold, kidx / kcnt / optional mask, and with `order` non-NULL the
// longest-first order of all H·nq items. `hist` (select_hist_bytes) must have been cleared by an earlier launch on
// the stream (the pooling or prepare launch clears it).
// The order covers the items whose query block lies in [order_q0, order_q1) (all heads); order_q1 <= 0 means all.
// spare_sms > 0 runs the launch on that many SMs fewer (at most half of them), for a collective running beside it.
cudaError_t launch_select(const float* pq, const float* pk, const KvPages& pk_pages, int heads, int nq, int nk, int bh,
                          int bw, int local_range, int q_slices, int topk, float* probs, uint32_t* hist, int32_t* kidx,
                          int32_t* kcnt, uint8_t* mask, int32_t* order, cudaStream_t st, int order_q0 = 0,
                          int order_q1 = 0, int spare_sms = 0);
size_t select_smem_bytes();
size_t select_hist_bytes(int heads, int q_slices);
// Reads and clears the selection's grid-barrier timeout word of the current device.
cudaError_t read_and_clear_select_error(int* flag);
size_t attn_bf16_smem_bytes(int nk);
cudaError_t launch_mask_to_lists(const float* mask, int heads, int nq, int nk, int32_t* kidx, int32_t* kcnt,
                                 cudaStream_t st);
// Attention over work items [item_begin, item_begin + item_count), item = h·nq + qb (head-major); CTA b takes
// item order[b] when an order is given (a permutation of the range), else item_begin + b.
cudaError_t launch_attn_f32(const float* q, const float* k, const float* v, const KvPages& pages, int heads, int nq,
                            int nk, const int32_t* kidx, const int32_t* kcnt, float* out, int item_begin,
                            int item_count, const int32_t* order, cudaStream_t st, OutRows rows = {});
// A key list split at key block split_nk (the lists are ascending): part 0 = the whole list (no split); part 1 = the
// blocks below split_nk, written unnormalised to fp32 partials — O (slot, 128, 128) and (row maximum in log2 units,
// row sum) (slot, 128, 2), slot = the CTA's position in the launch; part 2 = the blocks from split_nk on, merged with
// part 1's partials (same order, same slots) into the output. Lets the cached slices' blocks run while the current
// slice's keys are still arriving.
struct AttnSplit {
    int part = 0, split_nk = 0;
    float* part_o = nullptr;
    float* part_ml = nullptr;
};
cudaError_t launch_attn_bf16(const void* q, const void* k, const void* v, int64_t kv_rows, const KvPages& pages,
                             int heads, int nq, int nk, const int32_t* kidx, const int32_t* kcnt, void* out,
                             int item_begin, int item_count, const int32_t* order, cudaStream_t st,
                             OutRows rows = {}, AttnSplit split = {}, FreshKv fresh = {});
// The q/k/v side of one layer from the linear outputs (prepare.cu). Token grid (2·q_slices, 8·bh, 8·bw); nq windows.
struct PrepArgs {
    const void* x[3];        // q, k, v linear outputs, token order (L, C)
    const void* norm_w[2];   // RMSNorm weights of q and k (C, dtype) or NULL (no norm)
    const float* cosv;       // (L, 64) fp32 rotation tables or NULL (no rotation)
    const float* sinv;
    void* q_out;             // (L, C) window order
    void* kv_out[2];         // K and V arenas; window w goes to arena block kv_pages.page_block[w / s] + w % s
    float* pooled[2];        // pooled q (nq, C) and pooled k (arena blocks, like K) or NULL
    KvPages kv_pages;
    uint32_t* zero;          // words cleared before the pass (the selection histograms) or NULL
    size_t zero_words;
    float eps;
    int heads, bh, bw, nq;
};
cudaError_t launch_prepare(const PrepArgs& a, int dtype, cudaStream_t st);
constexpr int kPrepMaxHeads = 16;
// Work schedule of an item range (schedule.cu). A short range inside one head (at most kPersistItemsPerSm items per
// SM) gets the persistent kernel's partition: the head's kept key blocks cut into G equal shares, CTA c walking its
// share as segments (item, first list position, length, partial slot or −1); items cut by a share boundary are
// merged, and empty items zero-filled, by launch_combine. Other ranges get the longest-first item order for the
// per-item kernel. One buffer (sized for either) holds the one chosen.
constexpr int kPersistItemsPerSm = 8;
constexpr int kSchedItemCap = 4096;   // items of a persistent range (shared-memory prefix arrays)
constexpr int kSchedHeadCap = 63;     // heads of a persistent range
constexpr int kSchedPairCap = 16384;  // (CTA, head) pairs of a persistent range
struct SchedLayout {
    int G, item_count, Hr, max_segs, max_parts, max_comb;
    bool persistent;
    size_t off_hdr, off_order, off_seg_begin, off_segs, off_comb, off_empties, off_ml, off_opart, bytes;
};
SchedLayout sched_layout(int item_count, int nq, int heads, int G);
bool sched_persistent(const SchedLayout& L, int item_begin, int nq);  // the mode a range gets
cudaError_t launch_schedule(const int32_t* kcnt, int nk, int nq, int item_begin, int item_count,
                            const SchedLayout& L, void* buf, cudaStream_t st);
cudaError_t launch_combine(const SchedLayout& L, const void* buf, int heads, int nq, void* out, cudaStream_t st);
// Persistent bf16 attention over a schedule (grid G), then the combine.
cudaError_t launch_attn_bf16_persist(const void* q, const void* k, const void* v, int64_t kv_rows,
                                     const KvPages& pages, int heads, int nq, int nk, const int32_t* kidx,
                                     const SchedLayout& L, const void* sched, void* out, cudaStream_t st);
// Longest-first order of the items [item_begin, item_begin + item_count): the non-empty items of each head in turn
// by decreasing kcnt (stable by item id), then all empty items of the range by id.
cudaError_t launch_item_order(const int32_t* kcnt, int nq, int item_begin, int item_count, int32_t* order,
                              cudaStream_t st);
// The linear layers of the DiT block on tcgen05 (gemm.cu): out = epilogue(A · Bᵀ + bias), A (M, K), B (N, K) bf16,
// M % 128 = N % 256 = K % 64 = 0. Epilogues (the reference's bf16 rounding points): the Linear (round(acc + bias)),
// GELU(tanh) of it, or the gated residual round(resid + round(gate · linear)). Outputs: out[j] receives the columns
// [j·split, (j+1)·split) when split > 0 (the q/k/v projection into three tensors), else out[0] all N; row stride ldo.
enum GemmMode { kGemmPlain = 0, kGemmGelu = 1, kGemmGatedResidual = 2 };
struct GemmArgs {
    int M, N, K;
    const __nv_bfloat16* bias;   // (N) or NULL
    const __nv_bfloat16* gate;   // (N), gated residual only
    const __nv_bfloat16* resid;  // (M, ldo), gated residual only
    void* out[3];
    int split, ldo, mode;
};
cudaError_t launch_gemm_bf16(const GemmArgs& args, const void* A, const void* B, cudaStream_t st);
size_t gemm_smem_bytes();
cudaError_t read_and_clear_gemm_error(int* flag);
// Row normalisations of the DiT block (norm.cu); x / out (m, ch) bf16, ch a multiple of 256 up to 2048.
cudaError_t launch_layernorm(int m, int ch, const void* x, const void* weight, const void* bias, const void* shift,
                             const void* scale, float eps, void* out, cudaStream_t st);
cudaError_t launch_rmsnorm(int m, int ch, const void* x, const void* weight, float eps, void* out, cudaStream_t st);
// Reads and clears the persistent kernel's timeout word of the current device.
cudaError_t read_and_clear_persist_error(int* flag);
// One bounded wait that runs out (fvsr_wait_probe): sets the device timeout word after limit_ns, faults nothing.
cudaError_t launch_wait_probe(uint64_t limit_ns, cudaStream_t st);
// Reads and clears the device-side timeout words of the current device (1 if a wait gave up since the last read).
cudaError_t read_and_clear_device_error(int* flag, cudaStream_t st);

}  // namespace fvsr
