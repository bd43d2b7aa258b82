// stream.cu — the LCSA side of FlashVSR's streaming pipeline over the C ABI: the chunk schedule (Pipeline.swift:95-102),
// the per-chunk step geometry (DiT.swift:472-485, 554-578: RoPE tables from the chunk's first latent, topk, kvLen,
// local range) and one window K/V cache per DiT block, driving fvsr_lcsa_forward_tokens layer by layer.
//
// Host logic plus one small kernel that expands the three factor tables of the 3-D rotation (temporal 44 | height 42 |
// width 42 of a 128-wide head, RopeTables, DiT.swift:52-97) into the chunk's per-token (L, 64) tables.
#include <math.h>

#include <new>
#include <vector>

#include "../../include/fvsr_lcsa.h"
#include "common.cuh"

namespace fvsr {
void set_last_error(const char* msg);
}

using namespace fvsr;

namespace {

constexpr int kRopeEnd = 1024;                   // positions per factor table (RopeTables.end)
constexpr int kRopeT = 22, kRopeH = 21, kRopeW = 21;  // complex pairs per axis for a 128-wide head

fvsr_status sfail(fvsr_status s, const char* msg) {
    set_last_error(msg);
    return s;
}

// cos / sin of the chunk's tokens (token order (t, y, x) over an (f, h, w) patch grid), entry j of token:
// j < 22 temporal (position t0 + t), j < 43 height (y), else width (x).
__global__ void rope_expand_kernel(const float* __restrict__ fac_cos, const float* __restrict__ fac_sin, int t0, int f,
                                   int h, int w, float* __restrict__ cos_out, float* __restrict__ sin_out) {
    const int64_t n = (int64_t)f * h * w * 64;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(i & 63);
        const int64_t tok = i >> 6;
        const int x = (int)(tok % w), y = (int)(tok / w % h), t = (int)(tok / ((int64_t)w * h));
        int64_t src;
        if (j < kRopeT)
            src = (int64_t)(t0 + t) * kRopeT + j;
        else if (j < kRopeT + kRopeH)
            src = (int64_t)kRopeEnd * kRopeT + (int64_t)y * kRopeH + (j - kRopeT);
        else
            src = (int64_t)kRopeEnd * (kRopeT + kRopeH) + (int64_t)x * kRopeW + (j - kRopeT - kRopeH);
        cos_out[i] = fac_cos[src];
        sin_out[i] = fac_sin[src];
    }
}

// One axis table of RopeTables.init (DiT.swift:59-74): n = dim/2 pairs, freq_j = 1 / theta^(2j/dim) in double,
// angle = p·freq_j, stored as fp32 cos / sin for positions p < kRopeEnd.
void rope_axis(int dim, std::vector<float>& c, std::vector<float>& s, size_t off) {
    const int n = dim / 2;
    for (int p = 0; p < kRopeEnd; ++p)
        for (int j = 0; j < n; ++j) {
            const double freq = 1.0 / pow(10000.0, (double)(2 * j) / (double)dim);
            const double a = (double)p * freq;
            c[off + (size_t)p * n + j] = (float)cos(a);
            s[off + (size_t)p * n + j] = (float)sin(a);
        }
}

// Chunk k of the schedule (Pipeline.swift:95-102): latents [0, 6) for chunk 0, [4 + 2k, 6 + 2k) after.
void chunk_latents(int k, int* begin, int* end) {
    *begin = k == 0 ? 0 : 4 + 2 * k;
    *end = k == 0 ? 6 : 6 + 2 * k;
}

fvsr_status stream_geometry(int heads, int out_h, int out_w, int dtype, double topk_ratio, int local_range, int k,
                            fvsr_lcsa_params* p, int* lb, int* le) {
    if (heads < 1 || heads > kPrepMaxHeads) return sfail(FVSR_EINVAL, "heads must be in [1, 16]");
    if (out_h < 128 || out_w < 128 || out_h % 128 || out_w % 128)
        return sfail(FVSR_EINVAL, "the output size must be a positive multiple of 128 in both dimensions");
    if (dtype != FVSR_F32 && dtype != FVSR_BF16) return sfail(FVSR_EINVAL, "dtype must be FVSR_F32 or FVSR_BF16");
    if (out_h / 16 > kRopeEnd || out_w / 16 > kRopeEnd)
        return sfail(FVSR_EUNSUPPORTED, "the patch grid passes the rotation table end (1024 positions per axis)");
    if (local_range < 1) return sfail(FVSR_EINVAL, "local_range must be >= 1");
    if (k < 0) return sfail(FVSR_EINVAL, "chunk index must be >= 0");
    int b = 0, e = 0;
    chunk_latents(k, &b, &e);
    if (e > kRopeEnd) return sfail(FVSR_EUNSUPPORTED, "the chunk's temporal positions pass the rotation table end (1024)");
    const int bh = out_h / 128, bw = out_w / 128, s = bh * bw;
    // upstream's example default at the output size (Pipeline.swift:68), topk = Int(Double(s·s)·ratio) − 1 (DiT.swift:482)
    const double ratio = topk_ratio > 0.0 ? topk_ratio : 2.0 * 768.0 * 1280.0 / ((double)out_h * (double)out_w);
    const double t = (double)s * (double)s * ratio;
    if (!(t >= 1.0) || t > 2.0e9) return sfail(FVSR_EINVAL, "topk ratio gives a top-k below 0 or beyond int range");
    *p = fvsr_lcsa_params{};
    p->heads = heads;
    p->head_dim = 128;
    p->bh = bh;
    p->bw = bw;
    p->q_slices = (e - b) / 2;
    p->kv_slices = p->q_slices;
    p->local_range = local_range;
    p->topk = (int32_t)t - 1;
    p->dtype = dtype;
    if (lb) *lb = b;
    if (le) *le = e;
    return FVSR_OK;
}

}  // namespace

struct fvsr_stream {
    int heads, out_h, out_w, layers, dtype, local_range, kv_len;
    double topk_ratio;
    std::vector<fvsr_kv_cache*> caches;
    float* fac = nullptr;        // factor tables: cos (kRopeEnd·64 floats), then sin
    float* rope = nullptr;       // chunk tables: cos (max_tokens·64), then sin
    int64_t max_tokens = 0;
    int chunk = -1;              // chunk whose tables are built; -1 before the first
    int next_chunk = 0;
};

extern "C" {

fvsr_status fvsr_stream_chunk_geometry(int32_t heads, int32_t out_h, int32_t out_w, int32_t dtype, double topk_ratio,
                                       int32_t local_range, int32_t k, fvsr_lcsa_params* p, int32_t* latent_begin,
                                       int32_t* latent_end) {
    if (!p) return sfail(FVSR_EINVAL, "params is NULL");
    int b = 0, e = 0;
    fvsr_status st = stream_geometry(heads, out_h, out_w, dtype, topk_ratio, local_range, k, p, &b, &e);
    if (st != FVSR_OK) return st;
    if (latent_begin) *latent_begin = b;
    if (latent_end) *latent_end = e;
    return FVSR_OK;
}

fvsr_status fvsr_stream_create(int32_t heads, int32_t out_h, int32_t out_w, int32_t layers, int32_t dtype,
                               double topk_ratio, double kv_ratio, int32_t local_range, fvsr_stream** out) {
    if (!out) return sfail(FVSR_EINVAL, "out is NULL");
    *out = nullptr;
    fvsr_lcsa_params p0;
    fvsr_status st = stream_geometry(heads, out_h, out_w, dtype, topk_ratio, local_range, 0, &p0, nullptr, nullptr);
    if (st != FVSR_OK) return st;
    if (layers < 1 || layers > 1024) return sfail(FVSR_EINVAL, "layers must be in [1, 1024]");
    if (!(kv_ratio >= 1.0 && kv_ratio < 64.0)) return sfail(FVSR_EINVAL, "kv_ratio must give 1 <= kvLen <= 29");
    const int kv_len = (int)kv_ratio;  // Int(options.kvRatio) (Pipeline.swift:129)
    if (kv_len < 1 || kv_len + p0.q_slices > kMaxPages) return sfail(FVSR_EINVAL, "kv_ratio must give 1 <= kvLen <= 29");
    fvsr_stream* s = new (std::nothrow) fvsr_stream();
    if (!s) return sfail(FVSR_ENOMEM, "out of host memory");
    s->heads = heads;
    s->out_h = out_h;
    s->out_w = out_w;
    s->layers = layers;
    s->dtype = dtype;
    s->local_range = local_range;
    s->kv_len = kv_len;
    s->topk_ratio = topk_ratio;
    s->max_tokens = (int64_t)p0.q_slices * p0.bh * p0.bw * 128;
    auto cleanup = [&](fvsr_status code, const char* msg) {
        fvsr_stream_destroy(s);
        return sfail(code, msg);
    };
    for (int i = 0; i < layers; ++i) {
        fvsr_kv_cache* c = nullptr;
        st = fvsr_kv_cache_create(&p0, kv_len, p0.q_slices, &c);
        if (st != FVSR_OK) {
            fvsr_stream_destroy(s);
            return st;
        }
        s->caches.push_back(c);
    }
    const size_t fac_floats = (size_t)kRopeEnd * 64;
    std::vector<float> fc(fac_floats, 0.0f), fs(fac_floats, 0.0f);
    rope_axis(2 * kRopeT, fc, fs, 0);
    rope_axis(2 * kRopeH, fc, fs, (size_t)kRopeEnd * kRopeT);
    rope_axis(2 * kRopeW, fc, fs, (size_t)kRopeEnd * (kRopeT + kRopeH));
    if (cudaMalloc(&s->fac, 2 * fac_floats * sizeof(float)) != cudaSuccess) return cleanup(FVSR_ENOMEM, "rotation tables");
    if (cudaMemcpy(s->fac, fc.data(), fac_floats * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->fac + fac_floats, fs.data(), fac_floats * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
        return cleanup(FVSR_ECUDA, "uploading the rotation tables failed");
    if (cudaMalloc(&s->rope, 2 * (size_t)s->max_tokens * 64 * sizeof(float)) != cudaSuccess)
        return cleanup(FVSR_ENOMEM, "chunk rotation tables");
    *out = s;
    return FVSR_OK;
}

fvsr_status fvsr_stream_destroy(fvsr_stream* s) {
    if (!s) return FVSR_OK;
    for (fvsr_kv_cache* c : s->caches) fvsr_kv_cache_destroy(c);
    if (s->fac) cudaFree(s->fac);
    if (s->rope) cudaFree(s->rope);
    delete s;
    return FVSR_OK;
}

fvsr_status fvsr_stream_begin(fvsr_stream* s) {
    if (!s) return sfail(FVSR_EINVAL, "stream is NULL");
    for (fvsr_kv_cache* c : s->caches) fvsr_kv_cache_reset(c);
    s->chunk = -1;
    s->next_chunk = 0;
    return FVSR_OK;
}

fvsr_status fvsr_stream_workspace_size(const fvsr_stream* s, size_t* bytes) {
    if (!s || !bytes) return sfail(FVSR_EINVAL, "stream and bytes must be non-NULL");
    // the largest selection: chunk 0 (3 slices against 3) or a later chunk (1 slice against kvLen + 1)
    size_t best = 0;
    for (int k = 0; k < 2; ++k) {
        fvsr_lcsa_params p;
        fvsr_status st = stream_geometry(s->heads, s->out_h, s->out_w, s->dtype, s->topk_ratio, s->local_range, k, &p,
                                         nullptr, nullptr);
        if (st != FVSR_OK) return st;
        // after chunk 0 a cache holds 3 slices, less one if 3 > kvLen; each later chunk appends one and drops at most
        // one (DiT.swift:532-538), so a later chunk attends to max(kvLen + 1, 3) slices
        p.kv_slices = k == 0 ? p.q_slices : (s->kv_len + 1 > 3 ? s->kv_len + 1 : 3);
        size_t n = 0;
        st = fvsr_lcsa_workspace_size(&p, &n);
        if (st != FVSR_OK) return st;
        if (n > best) best = n;
    }
    *bytes = best;
    return FVSR_OK;
}

fvsr_status fvsr_stream_start_chunk(fvsr_stream* s, int32_t k, fvsr_stream_t stream) {
    if (!s) return sfail(FVSR_EINVAL, "stream is NULL");
    if (k != s->next_chunk) return sfail(FVSR_EINVAL, "chunks run in order from 0 after fvsr_stream_begin");
    fvsr_lcsa_params p;
    int b = 0, e = 0;
    fvsr_status st = stream_geometry(s->heads, s->out_h, s->out_w, s->dtype, s->topk_ratio, s->local_range, k, &p, &b, &e);
    if (st != FVSR_OK) return st;
    const int f = e - b, h = p.bh * 8, w = p.bw * 8;
    const int64_t n = (int64_t)f * h * w * 64;
    const int blocks = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
    rope_expand_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        s->fac, s->fac + (size_t)kRopeEnd * 64, b, f, h, w, s->rope, s->rope + (size_t)s->max_tokens * 64);
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) return sfail(FVSR_ECUDA, "rotation table launch failed");
    s->chunk = k;
    s->next_chunk = k + 1;
    return FVSR_OK;
}

fvsr_status fvsr_stream_rope(const fvsr_stream* s, const float** rope_cos, const float** rope_sin, int64_t* tokens) {
    if (!s || !rope_cos || !rope_sin) return sfail(FVSR_EINVAL, "stream and outputs must be non-NULL");
    if (s->chunk < 0) return sfail(FVSR_EINVAL, "no chunk started");
    fvsr_lcsa_params p;
    fvsr_status st = stream_geometry(s->heads, s->out_h, s->out_w, s->dtype, s->topk_ratio, s->local_range, s->chunk,
                                     &p, nullptr, nullptr);
    if (st != FVSR_OK) return st;
    *rope_cos = s->rope;
    *rope_sin = s->rope + (size_t)s->max_tokens * 64;
    if (tokens) *tokens = (int64_t)p.q_slices * p.bh * p.bw * 128;
    return FVSR_OK;
}

fvsr_status fvsr_stream_layer(fvsr_stream* s, int32_t layer, const void* q_lin, const void* k_lin, const void* v_lin,
                              const void* norm_q, const void* norm_k, float eps, void* q_win, void* out,
                              int32_t* kidx, int32_t* kcnt, void* workspace, size_t workspace_bytes,
                              fvsr_stream_t stream) {
    if (!s) return sfail(FVSR_EINVAL, "stream is NULL");
    if (s->chunk < 0) return sfail(FVSR_EINVAL, "no chunk started (fvsr_stream_start_chunk)");
    if (layer < 0 || layer >= s->layers) return sfail(FVSR_EINVAL, "layer out of range");
    fvsr_lcsa_params p;
    fvsr_status st = stream_geometry(s->heads, s->out_h, s->out_w, s->dtype, s->topk_ratio, s->local_range, s->chunk,
                                     &p, nullptr, nullptr);
    if (st != FVSR_OK) return st;
    return fvsr_lcsa_forward_tokens(&p, q_lin, k_lin, v_lin, norm_q, norm_k, eps, s->rope,
                                    s->rope + (size_t)s->max_tokens * 64, s->caches[layer], q_win, out, kidx, kcnt,
                                    workspace, workspace_bytes, stream);
}

}  // extern "C"
