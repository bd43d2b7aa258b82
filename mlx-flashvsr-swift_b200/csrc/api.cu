// api.cu — the C ABI of include/fvsr_lcsa.h: host-side validation, workspace layout, the paged streaming KV cache
// and the per-layer forward that chains append → select → attention → trim.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/fvsr_lcsa.h"
#include "common.cuh"

namespace fvsr {
void set_last_error(const char* msg);
}

using namespace fvsr;

namespace {

thread_local std::string g_last_error;

}  // namespace

void fvsr::set_last_error(const char* msg) { g_last_error = msg; }

namespace {

fvsr_status fail(fvsr_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

fvsr_status cuda_fail(cudaError_t e, const char* what) {
    return fail(FVSR_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define FVSR_CU(call, what)                          \
    do {                                             \
        cudaError_t _e = (call);                     \
        if (_e != cudaSuccess) return cuda_fail(_e, what); \
    } while (0)

constexpr int kMaxNk = 2560;       // selection keeps one score row per query block in shared memory
constexpr int kMaxHeads = 64;

struct Dims {
    int heads, s, nq, nk, q_slices;
    int64_t channels, elt;
};

fvsr_status check_params(const fvsr_lcsa_params* p, Dims* d, bool need_kv = true) {
    if (!p) return fail(FVSR_EINVAL, "params is NULL");
    if (p->heads < 1 || p->heads > kMaxHeads) return fail(FVSR_EINVAL, "heads must be in [1, %d], got %d", kMaxHeads, p->heads);
    if (p->head_dim != 128) return fail(FVSR_EINVAL, "head_dim must be 128, got %d", p->head_dim);
    if (p->bh < 1 || p->bw < 1) return fail(FVSR_EINVAL, "block grid must be positive, got %dx%d", p->bh, p->bw);
    if (p->q_slices < 1) return fail(FVSR_EINVAL, "q_slices must be >= 1, got %d", p->q_slices);
    if (need_kv && p->kv_slices < 1) return fail(FVSR_EINVAL, "kv_slices must be >= 1, got %d", p->kv_slices);
    if (p->local_range < 1) return fail(FVSR_EINVAL, "local_range must be >= 1, got %d", p->local_range);
    if (p->topk < 0) return fail(FVSR_EINVAL, "topk must be >= 0, got %d", p->topk);
    if (p->dtype != FVSR_F32 && p->dtype != FVSR_BF16) return fail(FVSR_EINVAL, "dtype must be FVSR_F32 or FVSR_BF16");
    // block counts in 64 bits: a 32-bit product of large grid sizes could wrap around and pass the bounds below
    const int64_t s64 = (int64_t)p->bh * p->bw;
    const int64_t nq64 = s64 <= 65535 ? (int64_t)p->q_slices * s64 : INT64_MAX;
    const int64_t nk64 = !need_kv ? 0 : s64 <= 65535 ? (int64_t)p->kv_slices * s64 : INT64_MAX;
    if (nk64 > kMaxNk) return fail(FVSR_EUNSUPPORTED, "Nk = %lld key blocks exceeds the supported %d", (long long)nk64, kMaxNk);
    if (nq64 > 65535 || (int64_t)p->heads * nq64 > (1ll << 30))
        return fail(FVSR_EUNSUPPORTED, "Nq = %lld query blocks is too large", (long long)nq64);
    // the selection pools the query and key blocks in one launch whose grid rows are blocks, and runs its radix
    // passes with one grid row per (head, query slice): both at most 65535
    if (nq64 + nk64 > 65535)
        return fail(FVSR_EUNSUPPORTED, "Nq + Nk = %lld blocks is too large for one selection", (long long)(nq64 + nk64));
    if (need_kv && (int64_t)p->heads * p->q_slices > 65535)
        return fail(FVSR_EUNSUPPORTED, "heads x q_slices = %lld selection rows is too large",
                    (long long)p->heads * p->q_slices);
    d->heads = p->heads;
    d->s = (int)s64;
    d->nq = (int)nq64;
    d->q_slices = p->q_slices;
    d->nk = (int)nk64;
    d->channels = (int64_t)p->heads * 128;
    d->elt = p->dtype == FVSR_BF16 ? 2 : 4;
    return FVSR_OK;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Buffers of 4-byte elements (index lists, counts, orders, probabilities, fp32 masks, pooled rows, norm weights read
// as 32-bit words) need that alignment; NULL passes (presence is checked separately).
bool aligned4(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3u) == 0; }

size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

struct Workspace {
    float* pooled_q;
    float* pooled_k;
    float* probs;
    int32_t* kidx;
    int32_t* kcnt;
    uint32_t* hist;
    int32_t* order;
    size_t bytes;
};

Workspace layout(const Dims& d, void* base) {
    Workspace w{};
    uint8_t* p = static_cast<uint8_t*>(base);
    size_t off = 0;
    auto take = [&](size_t n) {
        uint8_t* r = p ? p + off : nullptr;
        off += align_up(n);
        return r;
    };
    w.pooled_q = reinterpret_cast<float*>(take((size_t)d.nq * d.channels * 4));
    w.pooled_k = reinterpret_cast<float*>(take((size_t)d.nk * d.channels * 4));
    w.probs = reinterpret_cast<float*>(take((size_t)d.heads * d.nq * d.nk * 4));
    w.kidx = reinterpret_cast<int32_t*>(take((size_t)d.heads * d.nq * d.nk * 4));
    w.kcnt = reinterpret_cast<int32_t*>(take((size_t)d.heads * d.nq * 4));
    w.hist = reinterpret_cast<uint32_t*>(take(select_hist_bytes(d.heads, d.q_slices)));
    w.order = reinterpret_cast<int32_t*>(take((size_t)d.heads * d.nq * 4));
    w.bytes = off;
    return w;
}

// The caller's workspace: large enough for the layout, and 16-byte aligned (pooled rows are read as float4).
fvsr_status check_workspace(const Workspace& w, const void* workspace, size_t workspace_bytes) {
    if (!workspace || workspace_bytes < w.bytes)
        return fail(FVSR_ENOMEM, "workspace of %zu bytes is smaller than the %zu required", workspace_bytes, w.bytes);
    if (!aligned16(workspace)) return fail(FVSR_EINVAL, "workspace must be 16-byte aligned");
    return FVSR_OK;
}

fvsr_status check_lists(const int32_t* kidx, const int32_t* kcnt) {
    if (!aligned4(kidx) || !aligned4(kcnt)) return fail(FVSR_EINVAL, "kidx and kcnt must be 4-byte aligned");
    return FVSR_OK;
}

// A contiguous K/V buffer: one page holding all nk blocks, so logical block j is physical block j.
KvPages identity_pages(int nk) {
    KvPages pg{};
    pg.s = nk;
    return pg;
}

// Checks once per device that it is an sm_100 part (the tcgen05 kernel's target).
fvsr_status check_device_sm100() {
    int dev = 0;
    FVSR_CU(cudaGetDevice(&dev), "cudaGetDevice");
    static std::mutex mu;
    static std::vector<int> ok_cache(64, -1);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && ok_cache[dev] >= 0)
        return ok_cache[dev] ? FVSR_OK : fail(FVSR_EUNSUPPORTED, "device %d is not sm_100", dev);
    int major = 0, minor = 0;
    FVSR_CU(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "cudaDeviceGetAttribute");
    FVSR_CU(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev), "cudaDeviceGetAttribute");
    const bool ok = major == 10 && minor == 0;
    if (dev < 64) ok_cache[dev] = ok ? 1 : 0;
    return ok ? FVSR_OK : fail(FVSR_EUNSUPPORTED, "device %d is sm_%d%d, the kernels need sm_100a", dev, major, minor);
}

// The selection on pooled inputs (one cooperative launch); with `order` non-NULL it also writes the longest-first
// item order the attention takes. The histograms in `hist` were cleared by the pooling or prepare launch before it.
fvsr_status run_select(const fvsr_lcsa_params* p, const Dims& d, const float* pooled_q, const float* pooled_k,
                       const KvPages& pk_pages, int32_t* kidx, int32_t* kcnt, uint8_t* mask, float* probs,
                       uint32_t* hist, int32_t* order, cudaStream_t st) {
    FVSR_CU(launch_select(pooled_q, pooled_k, pk_pages, d.heads, d.nq, d.nk, p->bh, p->bw, p->local_range, p->q_slices,
                          p->topk, probs, hist, kidx, kcnt, mask, order, st),
            "selection launch");
    return FVSR_OK;
}

fvsr_status run_attention(const fvsr_lcsa_params* p, const Dims& d, const void* q, const void* k, const void* v,
                          int64_t kv_rows, const KvPages& pages, const int32_t* kidx, const int32_t* kcnt, void* out,
                          cudaStream_t st, int item_begin = 0, int item_count = -1, const int32_t* order = nullptr,
                          OutRows rows = {}, AttnSplit split = {}, FreshKv fresh = {}) {
    fvsr_status s = check_device_sm100();
    if (s != FVSR_OK) return s;
    if (item_count < 0) item_count = d.heads * d.nq;
    if (p->dtype == FVSR_BF16) {
        FVSR_CU(launch_attn_bf16(q, k, v, kv_rows, pages, d.heads, d.nq, d.nk, kidx, kcnt, out, item_begin, item_count,
                                 order, st, rows, split, fresh),
                "bf16 attention launch");
    } else {
        FVSR_CU(launch_attn_f32(static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v),
                                pages, d.heads, d.nq, d.nk, kidx, kcnt, static_cast<float*>(out), item_begin, item_count,
                                order, st, rows),
                "fp32 attention launch");
    }
    return FVSR_OK;
}

}  // namespace

struct fvsr_kv_cache {
    fvsr_lcsa_params p;
    Dims d;
    int kv_len, capacity;
    int page_blocks;             // arena blocks per page: s, or more when a page receives N equal gathered shards
    std::vector<int32_t> pages;  // logical slice order, oldest first → arena page
    int reserved = -1;           // page handed out by fvsr_kv_cache_reserve and not yet committed
    void* k_arena = nullptr;
    void* v_arena = nullptr;
    float* pk_arena = nullptr;   // pooled keys, (capacity·page_blocks, H·128) fp32
    int device = 0;
    // fvsr_lcsa_forward's copy of the appended slices into the arena runs on this stream beside the selection and the
    // attention (which read the new slices from the caller's buffers); fork / join events order it (bf16 caches)
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    int64_t page_rows() const { return (int64_t)page_blocks * 128; }
    int64_t page_bytes() const { return page_rows() * d.channels * d.elt; }
    int64_t slice_bytes() const { return (int64_t)d.s * 128 * d.channels * d.elt; }
    KvPages kv_pages() const {  // the logical slices as the kernels read them
        KvPages pg{};
        pg.s = d.s;
        for (int i = 0; i < kMaxPages; ++i) pg.page_block[i] = (i < (int)pages.size() ? pages[i] : 0) * page_blocks;
        return pg;
    }
};

namespace {

// The arena pages new_slices appended slices take (the lowest free ones, in slice order): *dst maps new window w to
// arena block dst->page_block[w / s] + w % s, *pages is the cache's page list after the append.
void choose_pages(const fvsr_kv_cache* c, int new_slices, KvPages* dst, std::vector<int32_t>* pages) {
    *dst = KvPages{};
    dst->s = c->d.s;
    *pages = c->pages;
    for (int t = 0; t < new_slices; ++t) {
        int page = -1;
        for (int cand = 0; cand < c->capacity && page < 0; ++cand) {
            bool used = false;
            for (int32_t u : *pages) used |= (u == cand);
            used |= (cand == c->reserved);  // a page handed out for a gather and not yet committed
            if (!used) page = cand;
        }
        dst->page_block[t] = page * c->page_blocks;
        pages->push_back(page);
    }
}

// Host checks shared by the two token-order entry points; fills the parts of *a that do not depend on destinations.
fvsr_status check_prepare_inputs(const fvsr_lcsa_params* p, const Dims& d, const void* q_lin, const void* k_lin,
                                 const void* v_lin, const void* norm_q, const void* norm_k, float eps,
                                 const float* rope_cos, const float* rope_sin, PrepArgs* a) {
    if (d.heads > kPrepMaxHeads)
        return fail(FVSR_EUNSUPPORTED, "the token-order path supports at most %d heads, got %d", kPrepMaxHeads, d.heads);
    if (!q_lin || !k_lin || !v_lin) return fail(FVSR_EINVAL, "q_lin, k_lin and v_lin are required");
    if (!aligned16(q_lin) || !aligned16(k_lin) || !aligned16(v_lin))
        return fail(FVSR_EINVAL, "q_lin, k_lin and v_lin must be 16-byte aligned");
    if ((rope_cos == nullptr) != (rope_sin == nullptr))
        return fail(FVSR_EINVAL, "rope_cos and rope_sin are given together or not at all");
    if (rope_cos && (!aligned16(rope_cos) || !aligned16(rope_sin)))
        return fail(FVSR_EINVAL, "rope_cos and rope_sin must be 16-byte aligned");
    if ((norm_q || norm_k) && !(eps >= 0.0f && eps < 1e30f)) return fail(FVSR_EINVAL, "eps must be finite and >= 0");
    if (!aligned4(norm_q) || !aligned4(norm_k)) return fail(FVSR_EINVAL, "norm_q and norm_k must be 4-byte aligned");
    *a = PrepArgs{};
    a->x[0] = q_lin;
    a->x[1] = k_lin;
    a->x[2] = v_lin;
    a->norm_w[0] = norm_q;
    a->norm_w[1] = norm_k;
    a->cosv = rope_cos;
    a->sinv = rope_sin;
    a->eps = eps;
    a->heads = d.heads;
    a->bh = p->bh;
    a->bw = p->bw;
    a->nq = d.nq;
    return FVSR_OK;
}

}  // namespace

extern "C" {

int32_t fvsr_version(void) { return 100; }

const char* fvsr_status_string(fvsr_status s) {
    switch (s) {
        case FVSR_OK: return "ok";
        case FVSR_EINVAL: return "invalid argument";
        case FVSR_ECUDA: return "CUDA error";
        case FVSR_ETIMEOUT: return "device wait timed out";
        case FVSR_ENOMEM: return "out of memory / workspace too small";
        case FVSR_EUNSUPPORTED: return "unsupported size or device";
    }
    return "unknown status";
}

const char* fvsr_last_error(void) { return g_last_error.c_str(); }

fvsr_status fvsr_device_check(fvsr_stream_t stream) {
    int flag = 0;
    FVSR_CU(read_and_clear_device_error(&flag, reinterpret_cast<cudaStream_t>(stream)), "device check");
    return flag ? fail(FVSR_ETIMEOUT, "a device-side wait hit its limit; the kernel returned early") : FVSR_OK;
}

fvsr_status fvsr_wait_probe(uint32_t limit_us, fvsr_stream_t stream) {
    if (limit_us < 1 || limit_us > 4000000) return fail(FVSR_EINVAL, "limit_us must be in [1, 4000000]");
    fvsr_status s = check_device_sm100();
    if (s != FVSR_OK) return s;
    FVSR_CU(launch_wait_probe((uint64_t)limit_us * 1000u, reinterpret_cast<cudaStream_t>(stream)), "wait probe launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_workspace_size(const fvsr_lcsa_params* p, size_t* bytes) {
    Dims d;
    fvsr_status s = check_params(p, &d);
    if (s != FVSR_OK) return s;
    if (!bytes) return fail(FVSR_EINVAL, "bytes is NULL");
    *bytes = layout(d, nullptr).bytes;
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_pool(const fvsr_lcsa_params* p, const void* x, int64_t nblocks, float* pooled,
                           fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d, false);
    if (s != FVSR_OK) return s;
    if (nblocks < 0 || nblocks > 65535) return fail(FVSR_EINVAL, "nblocks must be in [0, 65535], got %lld", (long long)nblocks);
    if (nblocks > 0 && (!x || !pooled)) return fail(FVSR_EINVAL, "x and pooled must be non-NULL");
    if (!aligned16(x) || !aligned16(pooled)) return fail(FVSR_EINVAL, "x and pooled must be 16-byte aligned");
    FVSR_CU(launch_pool(x, p->dtype, nblocks, (int)d.channels, pooled, nullptr, reinterpret_cast<cudaStream_t>(stream)),
            "pool launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_select(const fvsr_lcsa_params* p, const void* q, const void* k, const float* pooled_k,
                             int32_t* kidx, int32_t* kcnt, uint8_t* mask, float* probs, void* workspace,
                             size_t workspace_bytes, fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d);
    if (s != FVSR_OK) return s;
    if (!q || (!k && !pooled_k) || !kidx || !kcnt) return fail(FVSR_EINVAL, "q, k (or pooled_k), kidx and kcnt are required");
    if (!aligned16(q) || (k && !aligned16(k)) || (pooled_k && !aligned16(pooled_k)))
        return fail(FVSR_EINVAL, "q, k and pooled_k must be 16-byte aligned");
    s = check_lists(kidx, kcnt);
    if (s != FVSR_OK) return s;
    if (!aligned4(probs)) return fail(FVSR_EINVAL, "probs must be 4-byte aligned");
    Workspace w = layout(d, workspace);
    s = check_workspace(w, workspace, workspace_bytes);
    if (s != FVSR_OK) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const float* pk = pooled_k ? pooled_k : w.pooled_k;
    FVSR_CU(launch_pool2(q, d.nq, w.pooled_q, nullptr, pooled_k ? nullptr : k, pooled_k ? 0 : d.nk, w.pooled_k, p->dtype,
                         (int)d.channels, st, w.hist, select_hist_bytes(d.heads, d.q_slices) / 4),
            "pool launch");
    return run_select(p, d, w.pooled_q, pk, identity_pages(d.nk), kidx, kcnt, mask, probs ? probs : w.probs, w.hist,
                      nullptr, st);
}

fvsr_status fvsr_lcsa_attention(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                const int32_t* kidx, const int32_t* kcnt, void* out, fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d);
    if (s != FVSR_OK) return s;
    if (!q || !k || !v || !kidx || !kcnt || !out) return fail(FVSR_EINVAL, "q, k, v, kidx, kcnt and out are required");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(FVSR_EINVAL, "q, k, v and out must be 16-byte aligned");
    s = check_lists(kidx, kcnt);
    if (s != FVSR_OK) return s;
    return run_attention(p, d, q, k, v, (int64_t)d.nk * 128, identity_pages(d.nk), kidx, kcnt, out,
                         reinterpret_cast<cudaStream_t>(stream));
}

fvsr_status fvsr_lcsa_layer(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v, void* out,
                            int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                            fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d);
    if (s != FVSR_OK) return s;
    if (!q || !k || !v || !out) return fail(FVSR_EINVAL, "q, k, v and out are required");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(FVSR_EINVAL, "q, k, v and out must be 16-byte aligned");
    if (!aligned4(kidx) || !aligned4(kcnt)) return fail(FVSR_EINVAL, "kidx and kcnt must be 4-byte aligned");
    Workspace w = layout(d, workspace);
    s = check_workspace(w, workspace, workspace_bytes);
    if (s != FVSR_OK) return s;
    s = check_device_sm100();
    if (s != FVSR_OK) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int32_t* li = kidx ? kidx : w.kidx;
    int32_t* lc = kcnt ? kcnt : w.kcnt;
    FVSR_CU(launch_pool2(q, d.nq, w.pooled_q, nullptr, k, d.nk, w.pooled_k, p->dtype, (int)d.channels, st, w.hist,
                         select_hist_bytes(d.heads, d.q_slices) / 4),
            "pool launch");
    s = run_select(p, d, w.pooled_q, w.pooled_k, identity_pages(d.nk), li, lc, nullptr, w.probs, w.hist, w.order, st);
    if (s != FVSR_OK) return s;
    return run_attention(p, d, q, k, v, (int64_t)d.nk * 128, identity_pages(d.nk), li, lc, out, st, 0, d.heads * d.nq,
                         w.order);
}

fvsr_status fvsr_lcsa_item_order(const fvsr_lcsa_params* p, const int32_t* kcnt, int32_t item_begin, int32_t item_count,
                                 int32_t* order, fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d);
    if (s != FVSR_OK) return s;
    if (!kcnt || !order) return fail(FVSR_EINVAL, "kcnt and order are required");
    if (!aligned4(kcnt) || !aligned4(order)) return fail(FVSR_EINVAL, "kcnt and order must be 4-byte aligned");
    const int64_t items = (int64_t)d.heads * d.nq;
    if (item_begin < 0 || item_count < 0 || (int64_t)item_begin + item_count > items)
        return fail(FVSR_EINVAL, "item range [%d, %d) is outside [0, %lld)", item_begin, item_begin + item_count,
                    (long long)items);
    FVSR_CU(launch_item_order(kcnt, d.nq, item_begin, item_count, order, reinterpret_cast<cudaStream_t>(stream)),
            "item order launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_attention_range(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                      const int32_t* kidx, const int32_t* kcnt, void* out, int32_t item_begin,
                                      int32_t item_count, const int32_t* order, fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d);
    if (s != FVSR_OK) return s;
    if (!q || !k || !v || !kidx || !kcnt || !out) return fail(FVSR_EINVAL, "q, k, v, kidx, kcnt and out are required");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(FVSR_EINVAL, "q, k, v and out must be 16-byte aligned");
    s = check_lists(kidx, kcnt);
    if (s != FVSR_OK) return s;
    if (!aligned4(order)) return fail(FVSR_EINVAL, "order must be 4-byte aligned");
    const int64_t items = (int64_t)d.heads * d.nq;
    if (item_begin < 0 || item_count < 0 || (int64_t)item_begin + item_count > items)
        return fail(FVSR_EINVAL, "item range [%d, %d) is outside [0, %lld)", item_begin, item_begin + item_count,
                    (long long)items);
    return run_attention(p, d, q, k, v, (int64_t)d.nk * 128, identity_pages(d.nk), kidx, kcnt, out,
                         reinterpret_cast<cudaStream_t>(stream), item_begin, item_count, order);
}

namespace {

fvsr_status sched_geometry(const fvsr_lcsa_params* p, Dims* d, int32_t item_begin, int32_t item_count,
                           fvsr::SchedLayout* L) {
    fvsr_status s = check_params(p, d);
    if (s != FVSR_OK) return s;
    const int64_t items = (int64_t)d->heads * d->nq;
    if (item_begin < 0 || item_count < 0 || (int64_t)item_begin + item_count > items)
        return fail(FVSR_EINVAL, "item range [%d, %d) is outside [0, %lld)", item_begin, item_begin + item_count,
                    (long long)items);
    int dev = 0, nsm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) !=
                                                  cudaSuccess || nsm <= 0) {
        cudaGetLastError();
        return fail(FVSR_ECUDA, "cannot read the device's multiprocessor count");
    }
    *L = fvsr::sched_layout(item_count, d->nq, d->heads, nsm);
    return FVSR_OK;
}

}  // namespace

fvsr_status fvsr_lcsa_schedule_size(const fvsr_lcsa_params* p, int32_t item_count, size_t* bytes) {
    Dims d;
    fvsr::SchedLayout L;
    if (!bytes) return fail(FVSR_EINVAL, "bytes is NULL");
    fvsr_status s = sched_geometry(p, &d, 0, item_count, &L);
    if (s != FVSR_OK) return s;
    *bytes = L.bytes;
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_schedule(const fvsr_lcsa_params* p, const int32_t* kcnt, int32_t item_begin, int32_t item_count,
                               void* schedule, size_t schedule_bytes, fvsr_stream_t stream) {
    // pointer checks first: the geometry query below reads the device
    if (!kcnt || !schedule) return fail(FVSR_EINVAL, "kcnt and schedule are required");
    if (!aligned16(schedule)) return fail(FVSR_EINVAL, "schedule must be 16-byte aligned");
    if (!aligned4(kcnt)) return fail(FVSR_EINVAL, "kcnt must be 4-byte aligned");
    Dims d;
    fvsr::SchedLayout L;
    fvsr_status s = sched_geometry(p, &d, item_begin, item_count, &L);
    if (s != FVSR_OK) return s;
    if (schedule_bytes < L.bytes)
        return fail(FVSR_ENOMEM, "schedule of %zu bytes is smaller than the %zu required", schedule_bytes, L.bytes);
    if (item_count == 0) return FVSR_OK;
    s = check_device_sm100();
    if (s != FVSR_OK) return s;
    FVSR_CU(fvsr::launch_schedule(kcnt, d.nk, d.nq, item_begin, item_count, L, schedule,
                                  reinterpret_cast<cudaStream_t>(stream)),
            "schedule launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_attention_scheduled(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                          const int32_t* kidx, const int32_t* kcnt, void* out, int32_t item_begin,
                                          int32_t item_count, const void* schedule, size_t schedule_bytes,
                                          fvsr_stream_t stream) {
    // pointer checks first: the geometry query below reads the device
    if (!q || !k || !v || !kidx || !kcnt || !out || !schedule)
        return fail(FVSR_EINVAL, "q, k, v, kidx, kcnt, out and schedule are required");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(schedule))
        return fail(FVSR_EINVAL, "q, k, v, out and schedule must be 16-byte aligned");
    fvsr_status s = check_lists(kidx, kcnt);
    if (s != FVSR_OK) return s;
    Dims d;
    fvsr::SchedLayout L;
    s = sched_geometry(p, &d, item_begin, item_count, &L);
    if (s != FVSR_OK) return s;
    if (schedule_bytes < L.bytes)
        return fail(FVSR_ENOMEM, "schedule of %zu bytes is smaller than the %zu required", schedule_bytes, L.bytes);
    if (item_count == 0) return FVSR_OK;
    s = check_device_sm100();
    if (s != FVSR_OK) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // long ranges, and the fp32 lane: the per-item kernel (in the schedule's longest-first order when it has one)
    const bool persistent = fvsr::sched_persistent(L, item_begin, d.nq);
    if (!persistent || p->dtype != FVSR_BF16)
        return run_attention(p, d, q, k, v, (int64_t)d.nk * 128, identity_pages(d.nk), kidx, kcnt, out, st,
                             item_begin, item_count,
                             persistent ? nullptr
                                        : reinterpret_cast<const int32_t*>(static_cast<const uint8_t*>(schedule) +
                                                                           L.off_order));
    FVSR_CU(fvsr::launch_attn_bf16_persist(q, k, v, (int64_t)d.nk * 128, identity_pages(d.nk), d.heads, d.nq, d.nk,
                                           kidx, L, schedule, out, st),
            "persistent bf16 attention launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_attention_mask(const fvsr_lcsa_params* p, const void* q, const void* k, const void* v,
                                     const float* block_mask, void* out, void* workspace, size_t workspace_bytes,
                                     fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d);
    if (s != FVSR_OK) return s;
    if (!block_mask) return fail(FVSR_EINVAL, "block_mask is required");
    if (!aligned4(block_mask)) return fail(FVSR_EINVAL, "block_mask must be 4-byte aligned");
    Workspace w = layout(d, workspace);
    s = check_workspace(w, workspace, workspace_bytes);
    if (s != FVSR_OK) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    FVSR_CU(launch_mask_to_lists(block_mask, d.heads, d.nq, d.nk, w.kidx, w.kcnt, st), "mask to lists launch");
    FVSR_CU(launch_item_order(w.kcnt, d.nq, 0, d.heads * d.nq, w.order, st), "item order launch");
    return fvsr_lcsa_attention_range(p, q, k, v, w.kidx, w.kcnt, out, 0, d.heads * d.nq, w.order, stream);
}

// ---------------------------------------------------------------------------------------------------------------
// KV cache
// ---------------------------------------------------------------------------------------------------------------

fvsr_status fvsr_kv_cache_create(const fvsr_lcsa_params* p, int32_t kv_len, int32_t max_new_slices,
                                 fvsr_kv_cache** cache) {
    if (!p) return fail(FVSR_EINVAL, "params is NULL");
    return fvsr_kv_cache_create_padded(p, kv_len, max_new_slices, p->bh * p->bw, cache);
}

fvsr_status fvsr_kv_cache_create_padded(const fvsr_lcsa_params* p, int32_t kv_len, int32_t max_new_slices,
                                        int32_t page_blocks, fvsr_kv_cache** cache) {
    Dims d;
    fvsr_status s = check_params(p, &d, false);
    if (s != FVSR_OK) return s;
    if (!cache) return fail(FVSR_EINVAL, "cache is NULL");
    *cache = nullptr;
    if (kv_len < 1 || max_new_slices < 1 || kv_len + max_new_slices > kMaxPages)
        return fail(FVSR_EINVAL, "need kv_len >= 1, max_new_slices >= 1 and kv_len + max_new_slices <= %d", kMaxPages);
    if (page_blocks < d.s || page_blocks > 2 * d.s + 64)
        return fail(FVSR_EINVAL, "page_blocks must be in [s, 2s + 64] = [%d, %d], got %d", d.s, 2 * d.s + 64, page_blocks);
    if ((int64_t)(kv_len + max_new_slices) * d.s > kMaxNk)
        return fail(FVSR_EUNSUPPORTED, "cache of %d key blocks exceeds the supported %d", (kv_len + max_new_slices) * d.s, kMaxNk);
    if ((int64_t)(kv_len + max_new_slices) * page_blocks * 128 > (1ll << 31) - 1)
        return fail(FVSR_EUNSUPPORTED, "cache arena of %lld rows is too large",
                    (long long)(kv_len + max_new_slices) * page_blocks * 128);
    fvsr_kv_cache* c = new (std::nothrow) fvsr_kv_cache();
    if (!c) return fail(FVSR_ENOMEM, "host allocation failed");
    c->p = *p;
    c->d = d;
    c->kv_len = kv_len;
    c->capacity = kv_len + max_new_slices;
    c->page_blocks = page_blocks;
    cudaGetDevice(&c->device);
    const size_t bytes = (size_t)c->capacity * c->page_bytes();
    const size_t pbytes = (size_t)c->capacity * page_blocks * d.channels * 4;
    if (cudaMalloc(&c->k_arena, bytes) != cudaSuccess || cudaMalloc(&c->v_arena, bytes) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void**>(&c->pk_arena), pbytes) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(c->k_arena);
        cudaFree(c->v_arena);
        cudaFree(c->pk_arena);
        delete c;
        return fail(FVSR_ENOMEM, "cache arena allocation of %zu bytes failed", 2 * bytes + pbytes);
    }
    if (c->p.dtype == FVSR_BF16 &&
        (cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess ||
         cudaEventCreateWithFlags(&c->fork, cudaEventDisableTiming) != cudaSuccess ||
         cudaEventCreateWithFlags(&c->join, cudaEventDisableTiming) != cudaSuccess)) {
        cudaGetLastError();
        fvsr_kv_cache_destroy(c);
        return fail(FVSR_ECUDA, "cache side stream creation failed");
    }
    *cache = c;
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_destroy(fvsr_kv_cache* c) {
    if (!c) return FVSR_OK;
    if (c->side) cudaStreamDestroy(c->side);
    if (c->fork) cudaEventDestroy(c->fork);
    if (c->join) cudaEventDestroy(c->join);
    cudaFree(c->k_arena);
    cudaFree(c->v_arena);
    cudaFree(c->pk_arena);
    delete c;
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_reset(fvsr_kv_cache* c) {
    if (!c) return fail(FVSR_EINVAL, "cache is NULL");
    c->pages.clear();
    c->reserved = -1;
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_reserve(fvsr_kv_cache* c, void** k_page, void** v_page, float** pooled_k_page) {
    if (!c || !k_page || !v_page || !pooled_k_page) return fail(FVSR_EINVAL, "cache and the three outputs are required");
    if (c->reserved < 0) {
        if ((int)c->pages.size() + 1 > c->capacity)
            return fail(FVSR_EINVAL, "no free page: %zu slices held, capacity %d", c->pages.size(), c->capacity);
        KvPages dst{};
        std::vector<int32_t> pages;
        choose_pages(c, 1, &dst, &pages);
        c->reserved = pages.back();
    }
    const int64_t off = (int64_t)c->reserved * c->page_bytes();
    *k_page = static_cast<uint8_t*>(c->k_arena) + off;
    *v_page = static_cast<uint8_t*>(c->v_arena) + off;
    *pooled_k_page = c->pk_arena + (int64_t)c->reserved * c->page_blocks * c->d.channels;
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_commit(fvsr_kv_cache* c) {
    if (!c) return fail(FVSR_EINVAL, "cache is NULL");
    if (c->reserved < 0) return fail(FVSR_EINVAL, "no page is reserved");
    c->pages.push_back(c->reserved);
    c->reserved = -1;
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_slices(const fvsr_kv_cache* c, int32_t* slices) {
    if (!c || !slices) return fail(FVSR_EINVAL, "cache and slices must be non-NULL");
    *slices = (int32_t)c->pages.size();
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_append(fvsr_kv_cache* c, const void* k_new, const void* v_new, int32_t new_slices,
                                 fvsr_stream_t stream) {
    if (!c) return fail(FVSR_EINVAL, "cache is NULL");
    if (!k_new || !v_new) return fail(FVSR_EINVAL, "k_new and v_new are required");
    if (!aligned16(k_new) || !aligned16(v_new)) return fail(FVSR_EINVAL, "k_new and v_new must be 16-byte aligned");
    if (new_slices < 1 || (int)c->pages.size() + new_slices > c->capacity)
        return fail(FVSR_EINVAL, "appending %d slices to %zu exceeds the capacity %d", new_slices, c->pages.size(), c->capacity);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // lowest free arena page for each new slice, then one launch copies keys and values and pools the keys
    KvPages dst{};
    std::vector<int32_t> pages;
    choose_pages(c, new_slices, &dst, &pages);
    FVSR_CU(launch_append(k_new, v_new, c->p.dtype, (int64_t)new_slices * c->d.s, (int)c->d.channels, dst, c->k_arena,
                          c->v_arena, c->pk_arena, st),
            "cache append launch");
    c->pages = pages;
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_trim(fvsr_kv_cache* c) {
    if (!c) return fail(FVSR_EINVAL, "cache is NULL");
    if ((int)c->pages.size() > c->kv_len) c->pages.erase(c->pages.begin());
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_gather(const fvsr_kv_cache* c, void* k_out, void* v_out, fvsr_stream_t stream) {
    if (!c) return fail(FVSR_EINVAL, "cache is NULL");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    for (size_t i = 0; i < c->pages.size(); ++i) {
        const int64_t off = (int64_t)c->pages[i] * c->page_bytes();
        if (k_out)
            FVSR_CU(cudaMemcpyAsync(static_cast<uint8_t*>(k_out) + i * c->slice_bytes(), static_cast<uint8_t*>(c->k_arena) + off,
                                    c->slice_bytes(), cudaMemcpyDeviceToDevice, st),
                    "cache gather (keys)");
        if (v_out)
            FVSR_CU(cudaMemcpyAsync(static_cast<uint8_t*>(v_out) + i * c->slice_bytes(), static_cast<uint8_t*>(c->v_arena) + off,
                                    c->slice_bytes(), cudaMemcpyDeviceToDevice, st),
                    "cache gather (values)");
    }
    return FVSR_OK;
}

fvsr_status fvsr_kv_cache_state(const fvsr_kv_cache* c, int32_t* pages, int32_t* slices) {
    if (!c || !slices) return fail(FVSR_EINVAL, "cache and slices must be non-NULL");
    *slices = (int32_t)c->pages.size();
    if (pages)
        for (size_t i = 0; i < c->pages.size(); ++i) pages[i] = c->pages[i];
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_forward(const fvsr_lcsa_params* p, const void* q, const void* k_new, const void* v_new,
                              fvsr_kv_cache* cache, void* out, int32_t* kidx, int32_t* kcnt, void* workspace,
                              size_t workspace_bytes, fvsr_stream_t stream) {
    if (!cache) return fail(FVSR_EINVAL, "cache is NULL");
    if (!p) return fail(FVSR_EINVAL, "params is NULL");
    if (p->heads != cache->p.heads || p->bh != cache->p.bh || p->bw != cache->p.bw || p->dtype != cache->p.dtype)
        return fail(FVSR_EINVAL, "params do not match the cache geometry");
    if (!q || !out) return fail(FVSR_EINVAL, "q and out are required");
    if (!aligned16(q) || !aligned16(out)) return fail(FVSR_EINVAL, "q and out must be 16-byte aligned");
    if (!aligned4(kidx) || !aligned4(kcnt)) return fail(FVSR_EINVAL, "kidx and kcnt must be 4-byte aligned");
    fvsr_lcsa_params pp = *p;
    pp.kv_slices = (int32_t)cache->pages.size() + p->q_slices;
    Dims d;
    fvsr_status s = check_params(&pp, &d);
    if (s != FVSR_OK) return s;
    Workspace w = layout(d, workspace);
    s = check_workspace(w, workspace, workspace_bytes);
    if (s != FVSR_OK) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int32_t* li = kidx ? kidx : w.kidx;
    int32_t* lc = kcnt ? kcnt : w.kcnt;
    if (pp.dtype != FVSR_BF16) {  // the fp32 lane reads the arena: append first
        s = fvsr_kv_cache_append(cache, k_new, v_new, p->q_slices, stream);
        if (s != FVSR_OK) return s;
        const KvPages pages = cache->kv_pages();
        FVSR_CU(launch_pool2(q, d.nq, w.pooled_q, nullptr, nullptr, 0, nullptr, pp.dtype, (int)d.channels, st, w.hist,
                             select_hist_bytes(d.heads, d.q_slices) / 4),
                "pool q launch");
        s = run_select(&pp, d, w.pooled_q, cache->pk_arena, pages, li, lc, nullptr, w.probs, w.hist, w.order, st);
        if (s != FVSR_OK) return s;
        s = run_attention(&pp, d, q, cache->k_arena, cache->v_arena, (int64_t)cache->capacity * cache->page_rows(),
                          pages, li, lc, out, st, 0, d.heads * d.nq, w.order);
        if (s != FVSR_OK) return s;
        return fvsr_kv_cache_trim(cache);
    }
    // bf16: the new slices' keys are pooled into their arena pages (the selection reads every slice's pooled keys
    // there); their K/V rows are copied into the pages on the cache's side stream while the selection and the
    // attention run, the attention reading those blocks from k_new / v_new themselves; the call's stream waits for
    // the copy at the end, so the cache is whole when the call's work is.
    if (!k_new || !v_new) return fail(FVSR_EINVAL, "k_new and v_new are required");
    if (!aligned16(k_new) || !aligned16(v_new)) return fail(FVSR_EINVAL, "k_new and v_new must be 16-byte aligned");
    if (p->q_slices < 1 || (int)cache->pages.size() + p->q_slices > cache->capacity)
        return fail(FVSR_EINVAL, "appending %d slices to %zu exceeds the capacity %d", p->q_slices, cache->pages.size(),
                    cache->capacity);
    if (!cache->side) return fail(FVSR_ECUDA, "the cache has no side stream");
    KvPages dst{};
    std::vector<int32_t> after;
    choose_pages(cache, p->q_slices, &dst, &after);
    const int64_t slice = cache->slice_bytes();
    for (int t = 0; t < p->q_slices; ++t)
        FVSR_CU(launch_pool(static_cast<const uint8_t*>(k_new) + t * slice, pp.dtype, d.s, (int)d.channels,
                            cache->pk_arena + (int64_t)dst.page_block[t] * d.channels, nullptr, st),
                "pool k_new launch");
    FVSR_CU(cudaEventRecord(cache->fork, st), "fork record");
    FVSR_CU(cudaStreamWaitEvent(cache->side, cache->fork, 0), "fork wait");
    for (int t = 0; t < p->q_slices; ++t) {
        const int64_t off = (int64_t)dst.page_block[t] * 128 * d.channels * d.elt;
        FVSR_CU(cudaMemcpyAsync(static_cast<uint8_t*>(cache->k_arena) + off,
                                static_cast<const uint8_t*>(k_new) + t * slice, slice, cudaMemcpyDeviceToDevice,
                                cache->side),
                "append copy (keys)");
        FVSR_CU(cudaMemcpyAsync(static_cast<uint8_t*>(cache->v_arena) + off,
                                static_cast<const uint8_t*>(v_new) + t * slice, slice, cudaMemcpyDeviceToDevice,
                                cache->side),
                "append copy (values)");
    }
    FVSR_CU(cudaEventRecord(cache->join, cache->side), "join record");
    const size_t old_slices = cache->pages.size();
    cache->pages = after;
    const KvPages pages = cache->kv_pages();
    KvPages attn_pages = pages;  // the appended slices marked fresh: block t·s + b of k_new / v_new
    for (int t = 0; t < p->q_slices; ++t) attn_pages.page_block[old_slices + t] = kFreshPage | (t * d.s);
    FreshKv fresh;
    fresh.k = k_new;
    fresh.v = v_new;
    fresh.rows = (int64_t)p->q_slices * d.s * 128;
    FVSR_CU(launch_pool2(q, d.nq, w.pooled_q, nullptr, nullptr, 0, nullptr, pp.dtype, (int)d.channels, st, w.hist,
                         select_hist_bytes(d.heads, d.q_slices) / 4),
            "pool q launch");
    s = run_select(&pp, d, w.pooled_q, cache->pk_arena, pages, li, lc, nullptr, w.probs, w.hist, w.order, st);
    if (s == FVSR_OK)
        s = run_attention(&pp, d, q, cache->k_arena, cache->v_arena, (int64_t)cache->capacity * cache->page_rows(),
                          attn_pages, li, lc, out, st, 0, d.heads * d.nq, w.order, OutRows{}, AttnSplit{}, fresh);
    FVSR_CU(cudaStreamWaitEvent(st, cache->join, 0), "join wait");  // also on failure: the side work stays ordered
    if (s != FVSR_OK) return s;
    return fvsr_kv_cache_trim(cache);
}

}  // extern "C"

namespace {

// Shared checks of the sharded layer entries: geometry against the cache, the committed current slice, the rank's
// query block range, the workspace. Fills pp (kv_slices from the cache), d and w.
fvsr_status shard_setup(const fvsr_lcsa_params* p, int32_t qb_begin, int32_t qb_end, const fvsr_kv_cache* cache,
                        void* workspace, size_t workspace_bytes, fvsr_lcsa_params* pp, Dims* d, Workspace* w) {
    if (!cache) return fail(FVSR_EINVAL, "cache is NULL");
    if (!p) return fail(FVSR_EINVAL, "params is NULL");
    if (p->heads != cache->p.heads || p->bh != cache->p.bh || p->bw != cache->p.bw || p->dtype != cache->p.dtype)
        return fail(FVSR_EINVAL, "params do not match the cache geometry");
    if (cache->reserved >= 0) return fail(FVSR_EINVAL, "a reserved page is not committed");
    if ((int)cache->pages.size() < p->q_slices)
        return fail(FVSR_EINVAL, "the cache holds %zu slices, fewer than the chunk's %d", cache->pages.size(), p->q_slices);
    *pp = *p;
    pp->kv_slices = (int32_t)cache->pages.size();
    fvsr_status s = check_params(pp, d);
    if (s != FVSR_OK) return s;
    if (qb_begin < 0 || qb_end < qb_begin || qb_end > d->nq)
        return fail(FVSR_EINVAL, "query block range [%d, %d) is outside [0, %d)", qb_begin, qb_end, d->nq);
    *w = layout(*d, workspace);
    s = check_workspace(*w, workspace, workspace_bytes);
    if (s != FVSR_OK) return s;
    return check_device_sm100();
}

size_t partial_bytes(const Dims& d, int32_t qb_begin, int32_t qb_end) {
    return (size_t)d.heads * (size_t)(qb_end - qb_begin) * kBlock * (kD + 2) * sizeof(float);
}

}  // namespace

extern "C" {

fvsr_status fvsr_lcsa_partial_size(const fvsr_lcsa_params* p, int32_t qb_begin, int32_t qb_end, size_t* bytes) {
    Dims d;
    fvsr_status s = check_params(p, &d, false);
    if (s != FVSR_OK) return s;
    if (!bytes) return fail(FVSR_EINVAL, "bytes is NULL");
    if (qb_begin < 0 || qb_end < qb_begin) return fail(FVSR_EINVAL, "bad query block range [%d, %d)", qb_begin, qb_end);
    *bytes = partial_bytes(d, qb_begin, qb_end);
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_select_shard(const fvsr_lcsa_params* p, const float* pooled_q, int32_t qb_begin, int32_t qb_end,
                                   fvsr_kv_cache* cache, int32_t* kidx, int32_t* kcnt, void* workspace,
                                   size_t workspace_bytes, int32_t spare_sms, fvsr_stream_t stream) {
    fvsr_lcsa_params pp;
    Dims d;
    Workspace w;
    fvsr_status s = shard_setup(p, qb_begin, qb_end, cache, workspace, workspace_bytes, &pp, &d, &w);
    if (s != FVSR_OK) return s;
    if (!pooled_q) return fail(FVSR_EINVAL, "pooled_q is required");
    if (!aligned16(pooled_q)) return fail(FVSR_EINVAL, "pooled_q must be 16-byte aligned");
    if (!aligned4(kidx) || !aligned4(kcnt)) return fail(FVSR_EINVAL, "kidx and kcnt must be 4-byte aligned");
    if (spare_sms < 0) return fail(FVSR_EINVAL, "spare_sms must be >= 0, got %d", spare_sms);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    FVSR_CU(cudaMemsetAsync(w.hist, 0, select_hist_bytes(d.heads, d.q_slices), st), "histogram clear");
    FVSR_CU(launch_select(pooled_q, cache->pk_arena, cache->kv_pages(), d.heads, d.nq, d.nk, pp.bh, pp.bw,
                          pp.local_range, pp.q_slices, pp.topk, w.probs, w.hist, kidx ? kidx : w.kidx,
                          kcnt ? kcnt : w.kcnt, nullptr, w.order, st, qb_begin, qb_end, spare_sms),
            "selection launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_attend_shard(const fvsr_lcsa_params* p, const void* q, int32_t qb_begin, int32_t qb_end,
                                   fvsr_kv_cache* cache, fvsr_event_t kv_ready, void* partial, size_t partial_size,
                                   void* out, const int32_t* kidx, const int32_t* kcnt, void* workspace,
                                   size_t workspace_bytes, fvsr_stream_t stream) {
    fvsr_lcsa_params pp;
    Dims d;
    Workspace w;
    fvsr_status s = shard_setup(p, qb_begin, qb_end, cache, workspace, workspace_bytes, &pp, &d, &w);
    if (s != FVSR_OK) return s;
    if (!q || !out) return fail(FVSR_EINVAL, "q and out are required");
    if (!aligned16(q) || !aligned16(out) || !aligned16(partial))
        return fail(FVSR_EINVAL, "q, out and partial must be 16-byte aligned");
    if (!aligned4(kidx) || !aligned4(kcnt)) return fail(FVSR_EINVAL, "kidx and kcnt must be 4-byte aligned");
    if (partial && partial_size < partial_bytes(d, qb_begin, qb_end))
        return fail(FVSR_ENOMEM, "partial buffer of %zu bytes is smaller than the %zu required", partial_size,
                    partial_bytes(d, qb_begin, qb_end));
    if (qb_end == qb_begin) return fvsr_kv_cache_trim(cache);  // a rank past the end of the chunk: nothing to attend
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaEvent_t ev = reinterpret_cast<cudaEvent_t>(kv_ready);
    const KvPages pages = cache->kv_pages();
    const int32_t* li = kidx ? kidx : w.kidx;
    const int32_t* lc = kcnt ? kcnt : w.kcnt;
    OutRows rows;
    rows.qbase = qb_begin;
    rows.q_blocks = qb_end - qb_begin;
    const int items = d.heads * (qb_end - qb_begin);
    const int64_t kv_rows = (int64_t)cache->capacity * cache->page_rows();
    if (partial && pp.dtype == FVSR_BF16) {
        // the cached slices' blocks first (they are in the cache already), the chunk's own slices' blocks once the
        // gather has landed, merged in the second launch's epilogue
        AttnSplit sp;
        sp.split_nk = (pp.kv_slices - pp.q_slices) * d.s;
        sp.part_o = static_cast<float*>(partial);
        sp.part_ml = sp.part_o + (size_t)items * kBlock * kD;
        sp.part = 1;
        s = run_attention(&pp, d, q, cache->k_arena, cache->v_arena, kv_rows, pages, li, lc, out, st, 0, items, w.order,
                          rows, sp);
        if (s != FVSR_OK) return s;
        if (ev) FVSR_CU(cudaStreamWaitEvent(st, ev, 0), "wait for the K/V gather");
        sp.part = 2;
        s = run_attention(&pp, d, q, cache->k_arena, cache->v_arena, kv_rows, pages, li, lc, out, st, 0, items, w.order,
                          rows, sp);
    } else {
        if (ev) FVSR_CU(cudaStreamWaitEvent(st, ev, 0), "wait for the K/V gather");
        s = run_attention(&pp, d, q, cache->k_arena, cache->v_arena, kv_rows, pages, li, lc, out, st, 0, items, w.order,
                          rows);
    }
    if (s != FVSR_OK) return s;
    return fvsr_kv_cache_trim(cache);
}

fvsr_status fvsr_lcsa_forward_shard(const fvsr_lcsa_params* p, const void* q, int32_t qb_begin, int32_t qb_end,
                                    const float* pooled_q, fvsr_kv_cache* cache, fvsr_event_t kv_ready, void* out,
                                    int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                                    fvsr_stream_t stream) {
    fvsr_lcsa_params pp;
    Dims d;
    Workspace w;
    fvsr_status s = shard_setup(p, qb_begin, qb_end, cache, workspace, workspace_bytes, &pp, &d, &w);
    if (s != FVSR_OK) return s;
    if (qb_end == qb_begin) return fvsr_kv_cache_trim(cache);
    s = fvsr_lcsa_select_shard(p, pooled_q, qb_begin, qb_end, cache, kidx, kcnt, workspace, workspace_bytes, 0, stream);
    if (s != FVSR_OK) return s;
    return fvsr_lcsa_attend_shard(p, q, qb_begin, qb_end, cache, kv_ready, nullptr, 0, out, kidx, kcnt, workspace,
                                  workspace_bytes, stream);
}

fvsr_status fvsr_linear(int32_t m, int32_t n, int32_t k, const void* x, const void* w, const void* bias,
                        int32_t epilogue, const void* gate, const void* resid, void* out, fvsr_stream_t stream) {
    if (m <= 0 || n <= 0 || k <= 0 || m % 128 || n % 256 || k % 64)
        return fail(FVSR_EINVAL, "linear shape (%d, %d, %d): m must be a multiple of 128, n of 256, k of 64", m, n, k);
    if ((int64_t)m * k > (1ll << 31) || (int64_t)n * k > (1ll << 31) || (int64_t)m * n > (1ll << 31))
        return fail(FVSR_EUNSUPPORTED, "linear shape (%d, %d, %d) is too large", m, n, k);
    if (epilogue < FVSR_LINEAR || epilogue > FVSR_LINEAR_GATED_RESIDUAL)
        return fail(FVSR_EINVAL, "unknown epilogue %d", epilogue);
    if (!x || !w || !out) return fail(FVSR_EINVAL, "x, w and out are required");
    if (epilogue == FVSR_LINEAR_GATED_RESIDUAL && (!gate || !resid))
        return fail(FVSR_EINVAL, "the gated residual needs gate and resid");
    if (!aligned16(x) || !aligned16(w) || !aligned16(out) || !aligned16(resid) || !aligned4(bias) || !aligned4(gate))
        return fail(FVSR_EINVAL, "x, w, out and resid must be 16-byte aligned, bias and gate 4-byte aligned");
    fvsr_status s = check_device_sm100();
    if (s != FVSR_OK) return s;
    GemmArgs a{};
    a.M = m;
    a.N = n;
    a.K = k;
    a.bias = static_cast<const __nv_bfloat16*>(bias);
    a.gate = static_cast<const __nv_bfloat16*>(gate);
    a.resid = epilogue == FVSR_LINEAR_GATED_RESIDUAL ? static_cast<const __nv_bfloat16*>(resid) : nullptr;
    a.out[0] = out;
    a.split = 0;
    a.ldo = n;
    a.mode = epilogue;
    FVSR_CU(launch_gemm_bf16(a, x, w, reinterpret_cast<cudaStream_t>(stream)), "linear launch");
    return FVSR_OK;
}

fvsr_status fvsr_linear_qkv(int32_t m, int32_t n, int32_t k, const void* x, const void* w, const void* bias,
                            void* q_out, void* k_out, void* v_out, fvsr_stream_t stream) {
    if (m <= 0 || n <= 0 || k <= 0 || m % 128 || n % 256 || k % 64)
        return fail(FVSR_EINVAL, "linear shape (%d, %d, %d): m must be a multiple of 128, n of 256, k of 64", m, n, k);
    if ((int64_t)m * k > (1ll << 31) || 3ll * n * k > (1ll << 31) || (int64_t)m * n > (1ll << 31))
        return fail(FVSR_EUNSUPPORTED, "linear shape (%d, %d, %d) is too large", m, n, k);
    if (!x || !w || !q_out || !k_out || !v_out) return fail(FVSR_EINVAL, "x, w and the three outputs are required");
    if (!aligned16(x) || !aligned16(w) || !aligned16(q_out) || !aligned16(k_out) || !aligned16(v_out) ||
        !aligned4(bias))
        return fail(FVSR_EINVAL, "x, w and the outputs must be 16-byte aligned, bias 4-byte aligned");
    fvsr_status s = check_device_sm100();
    if (s != FVSR_OK) return s;
    GemmArgs a{};
    a.M = m;
    a.N = 3 * n;
    a.K = k;
    a.bias = static_cast<const __nv_bfloat16*>(bias);
    a.out[0] = q_out;
    a.out[1] = k_out;
    a.out[2] = v_out;
    a.split = n;
    a.ldo = n;
    a.mode = kGemmPlain;
    FVSR_CU(launch_gemm_bf16(a, x, w, reinterpret_cast<cudaStream_t>(stream)), "q/k/v projection launch");
    return FVSR_OK;
}

fvsr_status fvsr_layernorm(int32_t m, int32_t c, const void* x, const void* weight, const void* bias,
                           const void* shift, const void* scale, float eps, void* out, fvsr_stream_t stream) {
    if (m < 0 || c <= 0 || c % 256 || c > 2048)
        return fail(FVSR_EINVAL, "layernorm: c must be a positive multiple of 256 up to 2048, got %d (m %d)", c, m);
    if (!x || !out) return fail(FVSR_EINVAL, "x and out are required");
    if ((shift == nullptr) != (scale == nullptr)) return fail(FVSR_EINVAL, "shift and scale go together");
    if (bias && !weight) return fail(FVSR_EINVAL, "bias needs weight");
    if (!(eps >= 0.0f && eps < 1e30f)) return fail(FVSR_EINVAL, "eps must be finite and >= 0");
    if (!aligned16(x) || !aligned16(out) || !aligned4(weight) || !aligned4(bias) || !aligned4(shift) ||
        !aligned4(scale))
        return fail(FVSR_EINVAL, "x and out must be 16-byte aligned, the vectors 4-byte aligned");
    FVSR_CU(launch_layernorm(m, c, x, weight, bias, shift, scale, eps, out, reinterpret_cast<cudaStream_t>(stream)),
            "layernorm launch");
    return FVSR_OK;
}

fvsr_status fvsr_rmsnorm(int32_t m, int32_t c, const void* x, const void* weight, float eps, void* out,
                         fvsr_stream_t stream) {
    if (m < 0 || c <= 0 || c % 256 || c > 2048)
        return fail(FVSR_EINVAL, "rmsnorm: c must be a positive multiple of 256 up to 2048, got %d (m %d)", c, m);
    if (!x || !out || !weight) return fail(FVSR_EINVAL, "x, weight and out are required");
    if (!(eps >= 0.0f && eps < 1e30f)) return fail(FVSR_EINVAL, "eps must be finite and >= 0");
    if (!aligned16(x) || !aligned16(out) || !aligned4(weight))
        return fail(FVSR_EINVAL, "x and out must be 16-byte aligned, weight 4-byte aligned");
    FVSR_CU(launch_rmsnorm(m, c, x, weight, eps, out, reinterpret_cast<cudaStream_t>(stream)), "rmsnorm launch");
    return FVSR_OK;
}

fvsr_status fvsr_cross_attention(int32_t heads, int32_t lq, int32_t lk, const void* q, const void* k, const void* v,
                                 void* out, fvsr_stream_t stream) {
    if (heads < 1 || heads > kMaxHeads) return fail(FVSR_EINVAL, "heads must be in [1, %d], got %d", kMaxHeads, heads);
    if (lq <= 0 || lk <= 0 || lq % 128 || lk % 128)
        return fail(FVSR_EINVAL, "lq and lk must be positive multiples of 128, got %d and %d", lq, lk);
    if (lk / 128 > kMaxNk) return fail(FVSR_EUNSUPPORTED, "lk = %d keys exceeds %d blocks", lk, kMaxNk);
    if ((int64_t)heads * (lq / 128) > (1ll << 30)) return fail(FVSR_EUNSUPPORTED, "lq = %d is too large", lq);
    if (!q || !k || !v || !out) return fail(FVSR_EINVAL, "q, k, v and out are required");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
        return fail(FVSR_EINVAL, "q, k, v and out must be 16-byte aligned");
    fvsr_status s = check_device_sm100();
    if (s != FVSR_OK) return s;
    const int nq = lq / 128, nk = lk / 128;
    FVSR_CU(launch_attn_bf16(q, k, v, (int64_t)lk, identity_pages(nk), heads, nq, nk, nullptr, nullptr, out, 0,
                             heads * nq, nullptr, reinterpret_cast<cudaStream_t>(stream)),
            "cross-attention launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_prepare(const fvsr_lcsa_params* p, const void* q_lin, const void* k_lin, const void* v_lin,
                              const void* norm_q, const void* norm_k, float eps, const float* rope_cos,
                              const float* rope_sin, void* q_win, void* k_win, void* v_win, float* pooled_q,
                              float* pooled_k, fvsr_stream_t stream) {
    Dims d;
    fvsr_status s = check_params(p, &d, /*need_kv=*/false);
    if (s != FVSR_OK) return s;
    PrepArgs a;
    s = check_prepare_inputs(p, d, q_lin, k_lin, v_lin, norm_q, norm_k, eps, rope_cos, rope_sin, &a);
    if (s != FVSR_OK) return s;
    if (!q_win || !k_win || !v_win) return fail(FVSR_EINVAL, "q_win, k_win and v_win are required");
    if (!aligned16(q_win) || !aligned16(k_win) || !aligned16(v_win))
        return fail(FVSR_EINVAL, "q_win, k_win and v_win must be 16-byte aligned");
    if (!aligned4(pooled_q) || !aligned4(pooled_k)) return fail(FVSR_EINVAL, "pooled_q and pooled_k must be 4-byte aligned");
    s = check_device_sm100();
    if (s != FVSR_OK) return s;
    a.q_out = q_win;
    a.kv_out[0] = k_win;
    a.kv_out[1] = v_win;
    a.pooled[0] = pooled_q;
    a.pooled[1] = pooled_k;
    a.kv_pages.s = d.nq;  // one page: window w → block w
    FVSR_CU(launch_prepare(a, p->dtype, reinterpret_cast<cudaStream_t>(stream)), "prepare launch");
    return FVSR_OK;
}

fvsr_status fvsr_lcsa_forward_tokens(const fvsr_lcsa_params* p, const void* q_lin, const void* k_lin,
                                     const void* v_lin, const void* norm_q, const void* norm_k, float eps,
                                     const float* rope_cos, const float* rope_sin, fvsr_kv_cache* cache, void* q_win,
                                     void* out, int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                                     fvsr_stream_t stream) {
    if (!cache) return fail(FVSR_EINVAL, "cache is NULL");
    if (!p) return fail(FVSR_EINVAL, "params is NULL");
    if (p->heads != cache->p.heads || p->bh != cache->p.bh || p->bw != cache->p.bw || p->dtype != cache->p.dtype)
        return fail(FVSR_EINVAL, "params do not match the cache geometry");
    if (!q_win || !out) return fail(FVSR_EINVAL, "q_win and out are required");
    if (!aligned16(q_win) || !aligned16(out)) return fail(FVSR_EINVAL, "q_win and out must be 16-byte aligned");
    if (!aligned4(kidx) || !aligned4(kcnt)) return fail(FVSR_EINVAL, "kidx and kcnt must be 4-byte aligned");
    if (p->q_slices < 1 || (int)cache->pages.size() + p->q_slices > cache->capacity)
        return fail(FVSR_EINVAL, "appending %d slices to %zu exceeds the capacity %d", p->q_slices, cache->pages.size(),
                    cache->capacity);
    fvsr_lcsa_params pp = *p;
    pp.kv_slices = (int32_t)cache->pages.size() + p->q_slices;
    Dims d;
    fvsr_status s = check_params(&pp, &d);
    if (s != FVSR_OK) return s;
    PrepArgs a;
    s = check_prepare_inputs(&pp, d, q_lin, k_lin, v_lin, norm_q, norm_k, eps, rope_cos, rope_sin, &a);
    if (s != FVSR_OK) return s;
    Workspace w = layout(d, workspace);
    s = check_workspace(w, workspace, workspace_bytes);
    if (s != FVSR_OK) return s;
    s = check_device_sm100();
    if (s != FVSR_OK) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // norm + rotation + partition of q, k, v; k and v straight into the cache's new pages (the append), pooled k into
    // the pooled arena, pooled q into the workspace; the selection histograms cleared on the way
    std::vector<int32_t> new_pages;
    choose_pages(cache, p->q_slices, &a.kv_pages, &new_pages);
    a.q_out = q_win;
    a.kv_out[0] = cache->k_arena;
    a.kv_out[1] = cache->v_arena;
    a.pooled[0] = w.pooled_q;
    a.pooled[1] = cache->pk_arena;
    a.zero = w.hist;
    a.zero_words = select_hist_bytes(d.heads, d.q_slices) / 4;
    FVSR_CU(launch_prepare(a, pp.dtype, st), "prepare launch");
    cache->pages = new_pages;
    const KvPages pages = cache->kv_pages();
    int32_t* li = kidx ? kidx : w.kidx;
    int32_t* lc = kcnt ? kcnt : w.kcnt;
    s = run_select(&pp, d, w.pooled_q, cache->pk_arena, pages, li, lc, nullptr, w.probs, w.hist, w.order, st);
    if (s != FVSR_OK) return s;
    OutRows rows;
    rows.bh = pp.bh;
    rows.bw = pp.bw;
    s = run_attention(&pp, d, q_win, cache->k_arena, cache->v_arena, (int64_t)cache->capacity * cache->page_rows(), pages,
                      li, lc, out, st, 0, d.heads * d.nq, w.order, rows);
    if (s != FVSR_OK) return s;
    return fvsr_kv_cache_trim(cache);
}

}  // extern "C"
