/*
 * fvsr_lcsa.h — C ABI of the B200 (sm_100a) LCSA hot path: FlashVSR's locality-constrained block-sparse
 * self-attention (block selection + block-sparse flash attention over a streaming window KV cache).
 *
 * Drop-in boundary. The Swift DiT of xocialize/mlx-flashvsr-swift calls two functions per layer per chunk:
 *   draftBlockMaskAndProbs(qW:kW:heads:qSlices:spatialBlocks:local:topk:)   Sources/FlashVSRMLX/DiT.swift:158-174
 *   kernelBlockAttention(q:k:v:blockMask:heads:simdgroups:)                 Sources/FlashVSRMLX/SparseAttention.swift:169-187
 * and keeps the window K/V cache in blockForward (DiT.swift:507-511, 532-538). The entry points below replace those
 * with device-resident calls on plain pointers; a thin Swift shim over this header binds them.
 *
 * Tensor layout (identical to the Swift side): window-ordered tokens, row-major (L, H·128). Token t of window w is
 * row w·128 + t; head h owns columns [h·128, h·128 + 128). Query block i = window i of the chunk; key block j =
 * window j of (cache ⊕ current), oldest slice first. bf16 or fp32 storage (params.dtype).
 *
 * Conventions:
 *   - All pointers are device pointers unless stated; the caller owns every buffer.
 *   - Alignment (checked on the host, FVSR_EINVAL otherwise): 16 bytes for token rows (q, k, v, out and their
 *     token-order forms), pooled keys passed in, RoPE tables, the workspace and the schedule; 4 bytes for index lists,
 *     counts, orders, probabilities, fp32 block masks, pooled rows written out and the RMSNorm weights.
 *   - Every call is asynchronous on `stream` (a cudaStream_t; NULL = the legacy default stream) and never
 *     synchronises, except where noted.
 *   - No call allocates device memory except fvsr_kv_cache_create and fvsr_stream_create. Scratch comes from a
 *     caller-provided workspace whose size fvsr_lcsa_workspace_size (fvsr_stream_workspace_size) reports.
 *   - Errors are returned, never trapped: FVSR_EINVAL for bad shapes / NULL pointers (checked on the host before any
 *     launch), FVSR_ECUDA for a failed launch, FVSR_ETIMEOUT when a device-side wait gave up (reported by
 *     fvsr_device_check). fvsr_last_error() returns a message for the calling thread's last failure.
 *   - Thread-safe across distinct streams and distinct cache handles; one cache handle is used by one stream.
 */
#ifndef FVSR_LCSA_H
#define FVSR_LCSA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* fvsr_stream_t; /* a cudaStream_t */
typedef struct CUevent_st* fvsr_event_t;   /* a cudaEvent_t */

typedef enum fvsr_status {
    FVSR_OK = 0,
    FVSR_EINVAL = 1,      /* bad argument (shape, NULL pointer, misaligned pointer) */
    FVSR_ECUDA = 2,       /* a CUDA runtime call or kernel launch failed */
    FVSR_ETIMEOUT = 3,    /* a device-side wait hit its iteration limit and the kernel returned early */
    FVSR_ENOMEM = 4,      /* workspace too small, or cache allocation failed */
    FVSR_EUNSUPPORTED = 5 /* a size beyond the kernels' limits, or no sm_100 device */
} fvsr_status;

typedef enum fvsr_dtype { FVSR_F32 = 0, FVSR_BF16 = 1 } fvsr_dtype;

/* One LCSA call's geometry. Mirrors the Swift StepGeometry fields the path reads (DiT.swift:473-485). */
typedef struct fvsr_lcsa_params {
    int32_t heads;       /* H — FlashVSR: 12 */
    int32_t head_dim;    /* must be 128 (SparseAttention.swift:173) */
    int32_t bh, bw;      /* spatial block grid of one temporal slice (latent h/8, w/8 on the patch grid); s = bh·bw */
    int32_t q_slices;    /* temporal slices in the query chunk (StepGeometry.seqlen = f/2); Nq = q_slices·s */
    int32_t kv_slices;   /* temporal slices of keys, cache ⊕ current; Nk = kv_slices·s */
    int32_t local_range; /* R of localBlockMask (DiT.swift:130-145), ≥ 1 */
    int32_t topk;        /* integer top-k (DiT.swift:482), ≥ 0; keeps p > the (min(n−1, topk)+1)-th largest */
    int32_t dtype;       /* fvsr_dtype of q, k, v and out */
} fvsr_lcsa_params;

/* Library / error reporting. */
int32_t fvsr_version(void);
const char* fvsr_status_string(fvsr_status s);
const char* fvsr_last_error(void);

/* Synchronises `stream`, then reports (and clears) a device-side wait timeout recorded by any kernel of this library
 * on the current device: FVSR_ETIMEOUT if one was recorded, else FVSR_OK. No reference counterpart (the reference's
 * Metal kernel has no waits); this is the host side of the library's bounded device waits. */
fvsr_status fvsr_device_check(fvsr_stream_t stream);

/* Diagnostic of the failure path, no reference counterpart: launches one kernel whose single thread runs the
 * library's bounded device wait (the one every attention wait uses) on a barrier that nothing completes, with a limit
 * of limit_us microseconds (1 .. 4,000,000). The wait gives up, records the device timeout and the kernel returns;
 * the next fvsr_device_check reports FVSR_ETIMEOUT and the context stays usable. Nothing faults or hangs. */
fvsr_status fvsr_wait_probe(uint32_t limit_us, fvsr_stream_t stream);

/* Bytes of workspace that fvsr_lcsa_select, fvsr_lcsa_attention_mask and fvsr_lcsa_forward need for `p`
 * (the maximum of the three). */
fvsr_status fvsr_lcsa_workspace_size(const fvsr_lcsa_params* p, size_t* bytes);

/* fp32 mean over each 128-token block: x (nblocks·128, H·128) in p->dtype → pooled (nblocks, H·128) fp32.
 * Replaces qW.asType(.float32).mean(axis: 1) (DiT.swift:161-162). Summation order: four sequential partial sums over
 * tokens [0,32) [32,64) [64,96) [96,128), combined (s0+s1)+(s2+s3), times 1/128. */
fvsr_status fvsr_lcsa_pool(const fvsr_lcsa_params* p, const void* x, int64_t nblocks, float* pooled,
                           fvsr_stream_t stream);

/* Block selection — replaces draftBlockMaskAndProbs (DiT.swift:158-174).
 *   q (Nq·128, H·128), k (Nk·128, H·128) in p->dtype, window order. If pooled_k is non-NULL it holds the pooled keys
 *   (Nk, H·128) fp32 and k is not read (may be NULL) — the streaming cache keeps pooled keys per slice.
 *   Outputs: kidx (H, Nq, Nk) int32 — the kept key blocks of each (head, query block) first, ascending, the rest −1;
 *            kcnt (H, Nq) int32; mask (H, Nq, Nk) uint8 0/1 (optional, NULL to skip);
 *            probs (H, Nq, Nk) fp32 softmaxed block probabilities (optional).
 *   The top-k threshold is joint over each (head, query temporal slice) row, strict '>' (DiT.swift:169-173). */
fvsr_status fvsr_lcsa_select(const fvsr_lcsa_params* p, const void* q, const void* k, const float* pooled_k,
                             int32_t* kidx, int32_t* kcnt, uint8_t* mask, float* probs, void* workspace,
                             size_t workspace_bytes, fvsr_stream_t stream);

/* Size of the fixed scratch array behind fvsr_lcsa_select_noalloc (device memory held by every GPU that loads the
 * library, for the life of the process). */
#define FVSR_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)

/* fvsr_lcsa_select without a workspace: for callers that cannot allocate device memory — an engine that owns every
 * buffer under a fixed budget, or a real-time thread that must not take an allocation's device-wide synchronisation.
 * Same arguments and results as fvsr_lcsa_select, except that probs is required (an output, as in the reference) and
 * the scratch (pooled queries/keys, selection histograms) comes from one fixed FVSR_NOALLOC_SCRATCH_BYTES array
 * inside the library. Calls needing more scratch than that fail with FVSR_EUNSUPPORTED; nothing is allocated.
 * Outside a stream capture every call looks the array's address up in the calling thread's current CUDA context
 * (cudaGetSymbolAddress); inside a capture the address found by that context's last uncaptured call is used, so make
 * one call in each context before capturing (a captured call in a context without one fails with FVSR_EINVAL).
 * All calls on a device share the array and it keeps the last call's contents (what must start at zero is cleared
 * by each call); calls that overlap on the GPU race, so order them on one stream. No counterpart in the reference: it is an addition for hosts without an allocator. */
fvsr_status fvsr_lcsa_select_noalloc(const fvsr_lcsa_params* p, const void* q, const void* k, const float* pooled_k,
                                     int32_t* kidx, int32_t* kcnt, uint8_t* mask, float* probs, fvsr_stream_t stream);

/* Block-sparse attention over the kept pairs — replaces kernelBlockAttention (SparseAttention.swift:169-187) fed with
 * index lists. q (Nq·128, H·128), k / v (Nk·128, H·128), out (Nq·128, H·128), all p->dtype; kidx / kcnt as produced by
 * fvsr_lcsa_select. Scale 1/sqrt(128). A query block with kcnt = 0 writes zeros (SparseAttention.swift:47-53).
 * bf16 runs the tcgen05/TMEM tensor-core kernel; fp32 runs an fp32 CUDA-core kernel. */
fvsr_status fvsr_lcsa_attention(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                const int32_t* kidx, const int32_t* kcnt, void* out, fvsr_stream_t stream);

/* One LCSA layer on window-ordered q (Nq·128, H·128) and k, v (Nk·128, H·128) without a cache: the selection of
 * fvsr_lcsa_select, then the attention of fvsr_lcsa_attention over every (head, query block) item, longest key list
 * first — the two calls FlashVSRAttention makes per layer (DiT.swift:512-527: draftBlockMaskAndProbs, then
 * kernelBlockAttention). kidx / kcnt are optional outputs (NULL → kept in the workspace). Same workspace as
 * fvsr_lcsa_select. Three kernel launches: pooling, selection (which also orders the items), attention. */
fvsr_status fvsr_lcsa_layer(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v, void* out,
                            int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                            fvsr_stream_t stream);

/* Work items are the (head, query block) pairs, item = h·Nq + qb (head-major). */

/* Longest-first schedule of the items [item_begin, item_begin + item_count): order receives the non-empty item ids
 * (kcnt > 0) sorted by decreasing kcnt within each head (ties by id), heads kept in order, then the empty items of the
 * range by id — so long items start first, short ones fill the tail of the launch, and the items that only write
 * zeros come last. order has item_count entries. No reference counterpart (scheduling only). */
fvsr_status fvsr_lcsa_item_order(const fvsr_lcsa_params* p, const int32_t* kcnt, int32_t item_begin,
                                 int32_t item_count, int32_t* order, fvsr_stream_t stream);

/* fvsr_lcsa_attention restricted to the items [item_begin, item_begin + item_count), in the order given by `order`
 * (a permutation of the range from fvsr_lcsa_item_order, or NULL for ascending): the query-block sharding unit when
 * one (head, query block) space is split across GPUs. Rows of `out` outside the range are not written. The
 * reference has no multi-device path; its per-item semantics are SparseAttention.swift:17-153 (one threadgroup per
 * (query block, head)). */
fvsr_status fvsr_lcsa_attention_range(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                      const int32_t* kidx, const int32_t* kcnt, void* out, int32_t item_begin,
                                      int32_t item_count, const int32_t* order, fvsr_stream_t stream);

/* Balanced schedule of the items [item_begin, item_begin + item_count) — no counterpart in the reference (it is the
 * B200 kernel's work distribution). With S kept key blocks in the range and M multiprocessors on the current device,
 * the bf16 lane cuts every key list longer than T = max(ceil(S / 2M), 16) blocks into ceil(len / T) near-equal
 * chunks, so a short range (few CTA waves, as on each GPU of a sharded problem) is not bounded by its longest items;
 * units (item, chunk) run longest first and split items are merged afterwards. The fp32 lane orders without
 * splitting. fvsr_lcsa_schedule_size gives the bytes of the device buffer (header, units, order, fp32 partial
 * results: about 66 KB × 4M + 20 B × item_count); the buffer is reused by fvsr_lcsa_attention_scheduled. */
fvsr_status fvsr_lcsa_schedule_size(const fvsr_lcsa_params* p, int32_t item_count, size_t* bytes);
fvsr_status fvsr_lcsa_schedule(const fvsr_lcsa_params* p, const int32_t* kcnt, int32_t item_begin,
                               int32_t item_count, void* schedule, size_t schedule_bytes, fvsr_stream_t stream);

/* fvsr_lcsa_attention_range over a schedule from fvsr_lcsa_schedule (same p, kcnt and range, same device): the
 * attention over its units, then the merge of split items. Same output as fvsr_lcsa_attention_range up to the
 * summation order of split key lists. */
fvsr_status fvsr_lcsa_attention_scheduled(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                          const int32_t* kidx, const int32_t* kcnt, void* out, int32_t item_begin,
                                          int32_t item_count, const void* schedule, size_t schedule_bytes,
                                          fvsr_stream_t stream);

/* kernelBlockAttention with the reference's own argument form (SparseAttention.swift:169-177): block_mask
 * (H, Nq, Nk) fp32, kept where > 0.5. Builds the index lists in `workspace`, then runs fvsr_lcsa_attention. */
fvsr_status fvsr_lcsa_attention_mask(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                     const float* block_mask, void* out, void* workspace, size_t workspace_bytes,
                                     fvsr_stream_t stream);

/* ------------------------------------------------------------------------------------------------------------ */
/* Streaming window KV cache — replaces the cacheK / cacheV arrays of blockForward (DiT.swift:507-511, 532-538).   */
/* Keys/values live in slice pages of one device arena (one page = s·128 tokens × H·128), appended in place; the   */
/* logical order (oldest first) is a page table, so eviction moves no data. Pooled keys are kept per page.         */
/* ------------------------------------------------------------------------------------------------------------ */

typedef struct fvsr_kv_cache fvsr_kv_cache;

/* Allocates a cache for geometry p (heads, bh, bw, dtype are used) holding up to kv_len + max_new_slices pages.
 * kv_len = the reference's kvLen = Int(kvRatio) (Pipeline.swift:129). Not a hot call: it is the one allocating entry. */
fvsr_status fvsr_kv_cache_create(const fvsr_lcsa_params* p, int32_t kv_len, int32_t max_new_slices,
                                 fvsr_kv_cache** cache);
fvsr_status fvsr_kv_cache_destroy(fvsr_kv_cache* cache);
/* Forget every slice (a new clip). Host-side only. */
fvsr_status fvsr_kv_cache_reset(fvsr_kv_cache* cache);
/* Number of slices currently held. */
fvsr_status fvsr_kv_cache_slices(const fvsr_kv_cache* cache, int32_t* slices);
/* Append new_slices slices of keys/values (new_slices·s·128, H·128) in p->dtype: one kernel launch on `stream` copies
 * them into free pages and pools the keys (the concat of DiT.swift:508-511). */
fvsr_status fvsr_kv_cache_append(fvsr_kv_cache* cache, const void* k_new, const void* v_new, int32_t new_slices,
                                 fvsr_stream_t stream);
/* DiT.swift:532-538: if more than kv_len slices are held, drop the oldest one. Host-side only. */
fvsr_status fvsr_kv_cache_trim(fvsr_kv_cache* cache);
/* Copy the logical (cache order) keys and values into k_out / v_out (slices·s·128, H·128). For checks and export. */
fvsr_status fvsr_kv_cache_gather(const fvsr_kv_cache* cache, void* k_out, void* v_out, fvsr_stream_t stream);
/* Slot table for save/restore: pages[i] = arena page of logical slice i, for i < *slices (pages has room for
 * kv_len + max_new_slices entries). */
fvsr_status fvsr_kv_cache_state(const fvsr_kv_cache* cache, int32_t* pages, int32_t* slices);

/* One layer of LCSA in streaming mode — the self-attention core of blockForward (DiT.swift:504-538):
 * append (k_new, v_new) to the cache, select over cache ⊕ current with q, attend, then trim.
 * p->q_slices gives the chunk's slices (k_new / v_new hold q_slices·s·128 rows); p->kv_slices is ignored (taken from
 * the cache after the append). kidx / kcnt are optional outputs (NULL → kept in the workspace). */
fvsr_status fvsr_lcsa_forward(const fvsr_lcsa_params* p, const void* q, const void* k_new, const void* v_new,
                              fvsr_kv_cache* cache, void* out, int32_t* kidx, int32_t* kcnt, void* workspace,
                              size_t workspace_bytes, fvsr_stream_t stream);

/* ---- Query-block sharding of one chunk across GPUs ----
 * The reference runs on one device; this is the B200 partition of one chunk over N GPUs of a node. Rank r holds the
 * chunk's query blocks (windows) [qb_begin, qb_end) of q, k_new and v_new — what a sequence-split QKV projection
 * leaves on it. Per layer it pools its shard (fvsr_lcsa_pool), all-gathers the pooled queries and keys of every rank,
 * all-gathers the current slice's K and V straight into a reserved cache page (the caller's collective, e.g. NCCL),
 * commits the page, and calls fvsr_lcsa_forward_shard: the full selection (every rank computes the same one) and the
 * attention of its own query blocks over all heads. */

/* fvsr_kv_cache_create with a page stride of page_blocks ≥ s blocks (at most 2s + 64): a page can then receive N equal
 * shards of ceil(s / N) blocks each in one all-gather, the blocks past s being padding that is never read. */
fvsr_status fvsr_kv_cache_create_padded(const fvsr_lcsa_params* p, int32_t kv_len, int32_t max_new_slices,
                                        int32_t page_blocks, fvsr_kv_cache** cache);
/* Device pointers to the next free page (one slice): keys and values (page_blocks·128, H·128) in the cache dtype and
 * pooled keys (page_blocks, H·128) fp32, to be filled by the caller (window w of the slice at row w·128 / pooled
 * row w). Calling it again before fvsr_kv_cache_commit returns the same page. Host only. */
fvsr_status fvsr_kv_cache_reserve(fvsr_kv_cache* cache, void** k_page, void** v_page, float** pooled_k_page);
/* Appends the reserved page as the newest slice (the concat of DiT.swift:508-511 without a copy). Host only. */
fvsr_status fvsr_kv_cache_commit(fvsr_kv_cache* cache);

/* The layer call of one rank: selection over pooled_q (Nq, H·128) fp32 — every query block of the chunk — and the
 * cache's pooled keys (the current slice committed), then, after kv_ready (an event recorded once the K/V gather
 * into the page is complete; NULL = none), the attention of the items (h, qb) with qb in [qb_begin, qb_end), every
 * head, longest key list first, then the trim (DiT.swift:532-538). q and out hold only those query blocks:
 * ((qb_end − qb_begin)·128, H·128) window order. kidx / kcnt (H, Nq, Nk) / (H, Nq): optional outputs for all items.
 * p->q_slices = the chunk's slices; p->kv_slices is taken from the cache. Same workspace as fvsr_lcsa_forward.
 * The selection is identical on every rank, so the ranks' outputs together equal fvsr_lcsa_forward's. */
fvsr_status fvsr_lcsa_forward_shard(const fvsr_lcsa_params* p, const void* q, int32_t qb_begin, int32_t qb_end,
                                    const float* pooled_q, fvsr_kv_cache* cache, fvsr_event_t kv_ready, void* out,
                                    int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                                    fvsr_stream_t stream);

/* fvsr_lcsa_forward_shard in two calls, so that the current slice's K/V gather can run beside the attention of the
 * cached slices (cached pairs first, current pairs after the gather):
 *   fvsr_lcsa_select_shard — the selection (same as in fvsr_lcsa_forward_shard) and the order of the rank's items;
 *     needs only the pooled keys of the current slice in the committed page. Its one launch takes a CTA slot on
 *     every SM unless spare_sms > 0 leaves that many SMs (at most half) to a collective running beside it, so the
 *     K/V gather can start before the selection.
 *   fvsr_lcsa_attend_shard — with `partial` (fvsr_lcsa_partial_size bytes, bf16 only): the attention of every item
 *     over its kept blocks in the cached slices, written as fp32 partial results; then a wait for kv_ready; then
 *     the blocks of the chunk's own slices, merged with the partials into out (softmax of the union, so the result
 *     equals the one-launch attention up to fp32 summation order). Without `partial`: the wait, then the one-launch
 *     attention. Then the trim. kidx / kcnt: as given to fvsr_lcsa_select_shard (NULL: the workspace's). */
fvsr_status fvsr_lcsa_partial_size(const fvsr_lcsa_params* p, int32_t qb_begin, int32_t qb_end, size_t* bytes);
fvsr_status fvsr_lcsa_select_shard(const fvsr_lcsa_params* p, const float* pooled_q, int32_t qb_begin, int32_t qb_end,
                                   fvsr_kv_cache* cache, int32_t* kidx, int32_t* kcnt, void* workspace,
                                   size_t workspace_bytes, int32_t spare_sms, fvsr_stream_t stream);
fvsr_status fvsr_lcsa_attend_shard(const fvsr_lcsa_params* p, const void* q, int32_t qb_begin, int32_t qb_end,
                                   fvsr_kv_cache* cache, fvsr_event_t kv_ready, void* partial, size_t partial_size,
                                   void* out, const int32_t* kidx, const int32_t* kcnt, void* workspace,
                                   size_t workspace_bytes, fvsr_stream_t stream);

/* ---- Token-order entry points: the q/k/v side and the output side of blockForward's self-attention ----
 * Token grid of a chunk: (F, Hp, Wp) = (2·q_slices, 8·bh, 8·bw) patches, L = F·Hp·Wp = Nq·128 tokens in token order
 * (row (f·Hp + y)·Wp + x), the layout the Swift DiT holds before windowPartition and after windowReverse. At most 16
 * heads (FVSR_EUNSUPPORTED beyond).
 *
 * Rounding points (the reference's, with its order of operations): WanRMSNorm (DiT.swift:34-47)
 *   ss = Σ_c x_c² in fp32, inv = 1/√(ss / C + eps) correctly rounded, n = T(x·inv), y = T(n·w)
 * where Σ runs as 32 lane partials combined by a butterfly v_l += v_{l^o}, o = 16, 8, 4, 2, 1; lane l's partial is
 * (s0 + s1) + (s2 + s3) with s_e = the sum of x² over channels 128·i + 4l + e for i = 0..H−1 in order (MLX's reduction
 * order is unspecified; this is the library's);
 * ropeApply (DiT.swift:100-107) on each head's pairs (2j, 2j+1) with the token's (cos_j, sin_j):
 *   re' = T(re·cos − im·sin), im' = T(re·sin + im·cos), every product and sum rounded to fp32;
 * T = the storage type (bf16 round-to-nearest-even, or fp32).
 *
 * fvsr_lcsa_prepare: q_lin, k_lin, v_lin (L, H·128) token order, the three linear outputs of DiT.swift:497-499 →
 * q_win, k_win, v_win (L, H·128) window order (DiT.swift:504-506) after norm (q, k; weight NULL = skipped) and
 * rotation (q, k; tables NULL = skipped), plus optional pooled_q / pooled_k (Nq, H·128) fp32 block means of q_win /
 * k_win, bit-identical to fvsr_lcsa_pool of those outputs. norm_q / norm_k: (H·128) in p->dtype. rope_cos / rope_sin:
 * (L, 64) fp32, row = token, the tables RopeTables.grid builds (DiT.swift:80-97). One kernel launch. */
fvsr_status fvsr_lcsa_prepare(const fvsr_lcsa_params* p, const void* q_lin, const void* k_lin, const void* v_lin,
                              const void* norm_q, const void* norm_k, float eps, const float* rope_cos,
                              const float* rope_sin, void* q_win, void* k_win, void* v_win, float* pooled_q,
                              float* pooled_k, fvsr_stream_t stream);

/* One streaming layer from the linear outputs to the input of the output projection — DiT.swift:499-539 between
 * sa.q/k/v and sa.o: fvsr_lcsa_prepare with k and v written straight into the cache's new pages (the append) and the
 * pooled keys into its pooled arena, selection over cache ⊕ current, attention, trim, and the output written in token
 * order (windowReverse, DiT.swift:539, fused into the attention's epilogue). q_win: caller-owned (L, H·128) buffer
 * that receives the window-ordered q. out: (L, H·128) token order. Same workspace as fvsr_lcsa_forward. */
fvsr_status fvsr_lcsa_forward_tokens(const fvsr_lcsa_params* p, const void* q_lin, const void* k_lin,
                                     const void* v_lin, const void* norm_q, const void* norm_k, float eps,
                                     const float* rope_cos, const float* rope_sin, fvsr_kv_cache* cache, void* q_win,
                                     void* out, int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                                     fvsr_stream_t stream);

/* ---- Linear layers of the DiT block on the tensor cores ----
 * MLX's Linear (x·Wᵀ + b, DiT.swift:318-381) for the layers around the path: the q/k/v and output projections of
 * the self-attention (DiT.swift:496-499, 539), the feed-forward pair Linear → GELU(tanh) → Linear (DiT.swift:378,
 * 546-547) and the gated residual adds tok + gate · f(x) (DiT.swift:540, 547). x (M, K), w (N, K) (the Linear's weight
 * layout), bias (N) or NULL, all bf16; out (M, N) bf16; M a multiple of 128, N of 256, K of 64 (FVSR_EINVAL else).
 * fp32 accumulation; the output is rounded to bf16 once (the Linear), and the epilogues keep the reference's
 * rounding points: GELU → round(gelu(linear)); gated residual → round(resid + round(gate · linear)) with gate (N)
 * and resid (M, N) bf16 (resid may be out). One persistent tcgen05 kernel over CTA pairs (clusters of two CTAs,
 * 256 × 256 output tiles). */
typedef enum fvsr_linear_epilogue {
    FVSR_LINEAR = 0,
    FVSR_LINEAR_GELU = 1,
    FVSR_LINEAR_GATED_RESIDUAL = 2
} fvsr_linear_epilogue;
fvsr_status fvsr_linear(int32_t m, int32_t n, int32_t k, const void* x, const void* w, const void* bias,
                        int32_t epilogue, const void* gate, const void* resid, void* out, fvsr_stream_t stream);
/* The q, k and v projections in one launch: w = [Wq; Wk; Wv] (3·n, k), bias = [bq; bk; bv] (3·n) or NULL; the three
 * (m, n) outputs go to q_out, k_out, v_out (n a multiple of 256). Same arithmetic as three fvsr_linear calls. */
fvsr_status fvsr_linear_qkv(int32_t m, int32_t n, int32_t k, const void* x, const void* w, const void* bias,
                            void* q_out, void* k_out, void* v_out, fvsr_stream_t stream);

/* ---- The rest of the DiT block: norms and the cross-attention ----
 * fvsr_layernorm — LayerNorm over c channels of each of m rows (x, out (m, c) bf16, c a multiple of 256, at most
 * 2048; eps as the model's): without weight the reference's norm1 / norm2 (affine: false), followed, when shift and
 * scale (c) are given, by the block's modulation y·(1 + scale) + shift (DiT.swift:489-494, 546); with weight and bias
 * (c) the affine norm3 (DiT.swift:543). Rounding points: round(n), then round(round(n·round(1 + scale)) + shift);
 * affine round(n·w + b). fp32 statistics (mean, then the variance about it).
 * fvsr_rmsnorm — WanRMSNorm (DiT.swift:34-47): round(round(x / √(mean(x²) + eps))·w), the cross-attention's normQ.
 * fvsr_cross_attention — the cross-attention core (DiT.swift:351-360): softmax(q·kᵀ/√128)·v for every query over all
 * lk keys of the cached context, per head; q (lq, H·128), k / v (lk, H·128), out (lq, H·128) bf16, lq and lk
 * multiples of 128 (lk ≤ 327,680). The tcgen05 attention kernel with every key block kept. */
fvsr_status fvsr_layernorm(int32_t m, int32_t c, const void* x, const void* weight, const void* bias,
                           const void* shift, const void* scale, float eps, void* out, fvsr_stream_t stream);
fvsr_status fvsr_rmsnorm(int32_t m, int32_t c, const void* x, const void* weight, float eps, void* out,
                         fvsr_stream_t stream);
fvsr_status fvsr_cross_attention(int32_t heads, int32_t lq, int32_t lk, const void* q, const void* k, const void* v,
                                 void* out, fvsr_stream_t stream);

/* ---- Streaming driver: the LCSA side of FlashVSR's chunk loop ----
 * Mirrors FlashVSRPipeline.chunk / FlashVSRDiT.step (Pipeline.swift:95-102, 112-131; DiT.swift:472-485, 554-578) for
 * the self-attention of `layers` DiT blocks at an output size out_h × out_w (multiples of 128; spatial blocks
 * bh = out_h/128, bw = out_w/128):
 *   - chunk k covers latents [0, 6) for k = 0 (3 temporal slices), [4 + 2k, 6 + 2k) after (1 slice);
 *   - RoPE temporal start t0 = the chunk's first latent; tables as RopeTables (DiT.swift:52-97), built on the device;
 *   - topk = Int(Double(s²)·topk_ratio) − 1 (DiT.swift:482), topk_ratio <= 0 → 2·768·1280 / (out_h·out_w)
 *     (Pipeline.swift:68); kvLen = Int(kv_ratio) (Pipeline.swift:129); local range as given (default 11);
 *   - one window K/V cache per block (DiT.swift:507-511, 532-538). */
typedef struct fvsr_stream fvsr_stream;

/* Geometry of chunk k without a device: the layer params (kv_slices = q_slices; the caches set it per call) and the
 * chunk's latent range [latent_begin, latent_end) (latent_begin is the RoPE t0). Host only. */
fvsr_status fvsr_stream_chunk_geometry(int32_t heads, int32_t out_h, int32_t out_w, int32_t dtype, double topk_ratio,
                                       int32_t local_range, int32_t k, fvsr_lcsa_params* p, int32_t* latent_begin,
                                       int32_t* latent_end);
/* Allocates the caches (kvLen + 3 slice pages each) and the rotation tables. */
fvsr_status fvsr_stream_create(int32_t heads, int32_t out_h, int32_t out_w, int32_t layers, int32_t dtype,
                               double topk_ratio, double kv_ratio, int32_t local_range, fvsr_stream** s);
fvsr_status fvsr_stream_destroy(fvsr_stream* s);
/* A new clip (FlashVSRPipeline.begin, Pipeline.swift:105-108): empties every cache; the next chunk is 0. Host only. */
fvsr_status fvsr_stream_begin(fvsr_stream* s);
/* Workspace bytes fvsr_stream_layer needs for every chunk of this stream. */
fvsr_status fvsr_stream_workspace_size(const fvsr_stream* s, size_t* bytes);
/* Starts chunk k (k = 0, 1, 2, … in order after fvsr_stream_begin): builds its RoPE tables on `stream`. */
fvsr_status fvsr_stream_start_chunk(fvsr_stream* s, int32_t k, fvsr_stream_t stream);
/* Device pointers to the current chunk's (tokens, 64) fp32 RoPE tables. */
fvsr_status fvsr_stream_rope(const fvsr_stream* s, const float** rope_cos, const float** rope_sin, int64_t* tokens);
/* Self-attention of block `layer` in the current chunk: fvsr_lcsa_forward_tokens with the chunk's geometry and
 * tables and that block's cache. q_lin/k_lin/v_lin: (tokens, H·128) token order; out: (tokens, H·128) token order;
 * kidx / kcnt: optional selection outputs as in fvsr_lcsa_forward_tokens (NULL → kept in the workspace). */
fvsr_status fvsr_stream_layer(fvsr_stream* s, int32_t layer, const void* q_lin, const void* k_lin, const void* v_lin,
                              const void* norm_q, const void* norm_k, float eps, void* q_win, void* out,
                              int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                              fvsr_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FVSR_LCSA_H */
