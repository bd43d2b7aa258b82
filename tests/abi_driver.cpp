// abi_driver.cpp — C++ test driver of the C ABI (include/fvsr_lcsa.h), linked against libfvsr_lcsa.so the way a
// non-Python host binds it. Built and run by tests/test_abi_driver.py.
//
//   abi_driver cpu   host-side validation only (no GPU needed): every bad argument returns its status before any
//                    launch, with a message in fvsr_last_error().
//   abi_driver gpu   a small LCSA layer on the device: selection (with and without a workspace), attention, the
//                    streaming forward over a window cache, the streaming driver, and fvsr_device_check.
// Prints one line per failed check and exits non-zero if any failed.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "fvsr_lcsa.h"

static int g_failed = 0;

#define CHECK(cond)                                                         \
    do {                                                                    \
        if (!(cond)) {                                                      \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);     \
            ++g_failed;                                                     \
        }                                                                   \
    } while (0)

#define EXPECT_STATUS(call, want)                                                                          \
    do {                                                                                                   \
        const fvsr_status s_ = (call);                                                                     \
        if (s_ != (want)) {                                                                                \
            std::printf("FAIL %s:%d: %s returned %s, want %s (%s)\n", __FILE__, __LINE__, #call,           \
                        fvsr_status_string(s_), fvsr_status_string(want), fvsr_last_error());              \
            ++g_failed;                                                                                    \
        }                                                                                                  \
    } while (0)

static fvsr_lcsa_params small_params(fvsr_dtype dt) {
    fvsr_lcsa_params p;
    p.heads = 2;
    p.head_dim = 128;
    p.bh = 2;
    p.bw = 4;
    p.q_slices = 1;
    p.kv_slices = 3;
    p.local_range = 3;
    p.topk = 20;
    p.dtype = dt;
    return p;
}

static int run_cpu() {
    CHECK(fvsr_version() > 0);
    for (int s = FVSR_OK; s <= FVSR_EUNSUPPORTED; ++s) {
        const char* m = fvsr_status_string((fvsr_status)s);
        CHECK(m != nullptr && std::strlen(m) > 0);
    }
    fvsr_lcsa_params p = small_params(FVSR_BF16);
    size_t bytes = 0;
    EXPECT_STATUS(fvsr_lcsa_workspace_size(&p, &bytes), FVSR_OK);
    CHECK(bytes > 0);
    EXPECT_STATUS(fvsr_lcsa_workspace_size(nullptr, &bytes), FVSR_EINVAL);
    EXPECT_STATUS(fvsr_lcsa_workspace_size(&p, nullptr), FVSR_EINVAL);
    {
        fvsr_lcsa_params b = p;
        b.head_dim = 64;  // the kernels are head_dim 128 only (SparseAttention.swift:173)
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&b, &bytes), FVSR_EINVAL);
        CHECK(std::strlen(fvsr_last_error()) > 0);
        b = p;
        b.bh = 0;
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&b, &bytes), FVSR_EINVAL);
        b = p;
        b.local_range = 0;
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&b, &bytes), FVSR_EINVAL);
        b = p;
        b.topk = -1;
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&b, &bytes), FVSR_EINVAL);
        b = p;
        b.dtype = 7;
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&b, &bytes), FVSR_EINVAL);
    }
    {  // more key slices need more workspace
        fvsr_lcsa_params b = p;
        size_t more = 0;
        b.kv_slices = 6;
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&b, &more), FVSR_OK);
        CHECK(more > bytes);
    }
    // NULL and misaligned device pointers are refused on the host
    alignas(16) static char fake[256];
    void* ok_ptr = fake;
    void* odd_ptr = fake + 1;
    EXPECT_STATUS(fvsr_lcsa_select(&p, nullptr, ok_ptr, nullptr, (int32_t*)ok_ptr, (int32_t*)ok_ptr, nullptr, nullptr,
                                   ok_ptr, bytes, nullptr),
                  FVSR_EINVAL);
    EXPECT_STATUS(fvsr_lcsa_select(&p, odd_ptr, ok_ptr, nullptr, (int32_t*)ok_ptr, (int32_t*)ok_ptr, nullptr, nullptr,
                                   ok_ptr, bytes, nullptr),
                  FVSR_EINVAL);
    EXPECT_STATUS(fvsr_lcsa_select(&p, ok_ptr, ok_ptr, nullptr, (int32_t*)ok_ptr, (int32_t*)ok_ptr, nullptr, nullptr,
                                   ok_ptr, bytes - 1, nullptr),
                  FVSR_ENOMEM);
    EXPECT_STATUS(fvsr_lcsa_attention(&p, nullptr, ok_ptr, ok_ptr, (int32_t*)ok_ptr, (int32_t*)ok_ptr, ok_ptr, nullptr),
                  FVSR_EINVAL);
    // each buffer at its access width: index lists 4 bytes, the workspace 16
    EXPECT_STATUS(fvsr_lcsa_select(&p, ok_ptr, ok_ptr, nullptr, (int32_t*)(fake + 2), (int32_t*)ok_ptr, nullptr, nullptr,
                                   ok_ptr, bytes, nullptr),
                  FVSR_EINVAL);
    EXPECT_STATUS(fvsr_lcsa_select(&p, ok_ptr, ok_ptr, nullptr, (int32_t*)ok_ptr, (int32_t*)ok_ptr, nullptr, nullptr,
                                   fake + 4, bytes, nullptr),
                  FVSR_EINVAL);
    // block counts that wrap in 32 bits are refused, not taken for a small problem
    {
        fvsr_lcsa_params b = p;
        b.bh = 1 << 16;
        b.bw = 1 << 16;
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&b, &bytes), FVSR_EUNSUPPORTED);
        EXPECT_STATUS(fvsr_lcsa_workspace_size(&p, &bytes), FVSR_OK);
    }
    // item ranges outside the H·Nq items
    const int32_t items = p.heads * p.q_slices * p.bh * p.bw;
    EXPECT_STATUS(fvsr_lcsa_attention_range(&p, ok_ptr, ok_ptr, ok_ptr, (int32_t*)ok_ptr, (int32_t*)ok_ptr, ok_ptr,
                                            items - 1, 2, nullptr, nullptr),
                  FVSR_EINVAL);
    EXPECT_STATUS(fvsr_lcsa_item_order(&p, (int32_t*)ok_ptr, -1, 1, (int32_t*)ok_ptr, nullptr), FVSR_EINVAL);
    EXPECT_STATUS(fvsr_lcsa_schedule_size(&p, items + 1, &bytes), FVSR_EINVAL);
    EXPECT_STATUS(fvsr_lcsa_schedule_size(&p, -3, &bytes), FVSR_EINVAL);
    // cache geometry limits
    fvsr_kv_cache* c = nullptr;
    EXPECT_STATUS(fvsr_kv_cache_create(&p, 0, 1, &c), FVSR_EINVAL);
    EXPECT_STATUS(fvsr_kv_cache_create(&p, 2, 0, &c), FVSR_EINVAL);
    EXPECT_STATUS(fvsr_kv_cache_create(&p, 40, 1, &c), FVSR_EINVAL);
    EXPECT_STATUS(fvsr_kv_cache_create(&p, 2, 1, nullptr), FVSR_EINVAL);
    CHECK(c == nullptr);
    EXPECT_STATUS(fvsr_lcsa_forward(&p, ok_ptr, ok_ptr, ok_ptr, nullptr, ok_ptr, nullptr, nullptr, ok_ptr, bytes,
                                    nullptr),
                  FVSR_EINVAL);
    // token-order entry points: host checks before any launch
    {
        fvsr_lcsa_params b = p;
        b.heads = 17;
        EXPECT_STATUS(fvsr_lcsa_prepare(&b, ok_ptr, ok_ptr, ok_ptr, nullptr, nullptr, 1e-6f, nullptr, nullptr, ok_ptr,
                                        ok_ptr, ok_ptr, nullptr, nullptr, nullptr),
                      FVSR_EUNSUPPORTED);
        EXPECT_STATUS(fvsr_lcsa_prepare(&p, ok_ptr, ok_ptr, ok_ptr, nullptr, nullptr, 1e-6f, (const float*)ok_ptr,
                                        nullptr, ok_ptr, ok_ptr, ok_ptr, nullptr, nullptr, nullptr),
                      FVSR_EINVAL);
        EXPECT_STATUS(fvsr_lcsa_forward_tokens(&p, ok_ptr, ok_ptr, ok_ptr, nullptr, nullptr, 1e-6f, nullptr, nullptr,
                                               nullptr, ok_ptr, ok_ptr, nullptr, nullptr, ok_ptr, bytes, nullptr),
                      FVSR_EINVAL);
    }
    // streaming driver: the reference's chunk schedule and topk rule, host only
    {
        fvsr_lcsa_params g;
        int32_t b = -1, e = -1;
        EXPECT_STATUS(fvsr_stream_chunk_geometry(12, 1152, 1920, FVSR_BF16, 0.0, 11, 0, &g, &b, &e), FVSR_OK);
        CHECK(b == 0 && e == 6 && g.q_slices == 3 && g.bh == 9 && g.bw == 15 && g.topk == 16199);
        EXPECT_STATUS(fvsr_stream_chunk_geometry(12, 1152, 1920, FVSR_BF16, 0.0, 11, 5, &g, &b, &e), FVSR_OK);
        CHECK(b == 14 && e == 16 && g.q_slices == 1);
        EXPECT_STATUS(fvsr_stream_chunk_geometry(12, 1000, 1920, FVSR_BF16, 0.0, 11, 0, &g, &b, &e), FVSR_EINVAL);
        EXPECT_STATUS(fvsr_stream_chunk_geometry(12, 1152, 1920, FVSR_BF16, 0.0, 11, 0, nullptr, &b, &e), FVSR_EINVAL);
        EXPECT_STATUS(fvsr_stream_create(12, 1152, 1920, 30, FVSR_BF16, 0.0, 3.0, 11, nullptr), FVSR_EINVAL);
        fvsr_stream* st = nullptr;
        EXPECT_STATUS(fvsr_stream_create(12, 1152, 1920, 30, FVSR_BF16, 0.0, 0.5, 11, &st), FVSR_EINVAL);
        CHECK(st == nullptr);
        EXPECT_STATUS(fvsr_stream_begin(nullptr), FVSR_EINVAL);
        EXPECT_STATUS(fvsr_stream_destroy(nullptr), FVSR_OK);
    }
    return g_failed;
}

// Deterministic inputs: a 32-bit LCG mapped to [−2, 2), rounded to bf16.
static std::vector<uint16_t> bf16_values(size_t n, uint32_t seed) {
    std::vector<uint16_t> v(n);
    uint32_t x = seed;
    for (size_t i = 0; i < n; ++i) {
        x = x * 1664525u + 1013904223u;
        const float f = ((float)(x >> 8) / 16777216.0f) * 4.0f - 2.0f;
        uint32_t bits;
        std::memcpy(&bits, &f, 4);
        v[i] = (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
    }
    return v;
}

template <typename T>
static T* to_device(const std::vector<T>& h) {
    T* d = nullptr;
    if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) return nullptr;
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}

static int run_gpu() {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        std::printf("FAIL no CUDA device\n");
        return 1;
    }
    const fvsr_lcsa_params p = small_params(FVSR_BF16);
    const int s = p.bh * p.bw, nq = p.q_slices * s, nk = p.kv_slices * s, C = p.heads * 128;
    const size_t lq = (size_t)nq * 128, lk = (size_t)nk * 128;
    uint16_t* q = to_device(bf16_values(lq * C, 1));
    uint16_t* k = to_device(bf16_values(lk * C, 2));
    uint16_t* v = to_device(bf16_values(lk * C, 3));
    size_t ws_bytes = 0;
    EXPECT_STATUS(fvsr_lcsa_workspace_size(&p, &ws_bytes), FVSR_OK);
    void* ws = nullptr;
    int32_t *kidx = nullptr, *kcnt = nullptr, *kidx2 = nullptr, *kcnt2 = nullptr;
    float* probs = nullptr;
    uint16_t* out = nullptr;
    cudaMalloc(&ws, ws_bytes);
    cudaMalloc(&kidx, sizeof(int32_t) * p.heads * nq * nk);
    cudaMalloc(&kcnt, sizeof(int32_t) * p.heads * nq);
    cudaMalloc(&kidx2, sizeof(int32_t) * p.heads * nq * nk);
    cudaMalloc(&kcnt2, sizeof(int32_t) * p.heads * nq);
    cudaMalloc(&probs, sizeof(float) * p.heads * nq * nk);
    cudaMalloc(&out, lq * C * 2);
    CHECK(q && k && v && ws && kidx && kcnt && kidx2 && kcnt2 && probs && out);
    cudaStream_t st;
    cudaStreamCreate(&st);
    fvsr_stream_t fs = reinterpret_cast<fvsr_stream_t>(st);
    EXPECT_STATUS(fvsr_lcsa_select(&p, q, k, nullptr, kidx, kcnt, nullptr, nullptr, ws, ws_bytes, fs), FVSR_OK);
    EXPECT_STATUS(fvsr_lcsa_select_noalloc(&p, q, k, nullptr, kidx2, kcnt2, nullptr, probs, fs), FVSR_OK);
    EXPECT_STATUS(fvsr_lcsa_attention(&p, q, k, v, kidx, kcnt, out, fs), FVSR_OK);
    EXPECT_STATUS(fvsr_device_check(fs), FVSR_OK);
    std::vector<int32_t> hk(p.heads * nq * nk), hc(p.heads * nq), hk2(hk.size()), hc2(hc.size());
    cudaMemcpy(hk.data(), kidx, hk.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hc.data(), kcnt, hc.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hk2.data(), kidx2, hk.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hc2.data(), kcnt2, hc.size() * 4, cudaMemcpyDeviceToHost);
    CHECK(hk == hk2 && hc == hc2);  // the two selection entries agree exactly
    long kept = 0;
    for (int r = 0; r < p.heads * nq; ++r) {
        const int c = hc[r];
        CHECK(c >= 0 && c <= nk);
        kept += c;
        for (int j = 0; j < nk; ++j) {
            const int32_t x = hk[(size_t)r * nk + j];
            if (j < c) {
                CHECK(x >= 0 && x < nk);
                if (j > 0) CHECK(x > hk[(size_t)r * nk + j - 1]);  // ascending key blocks
            } else {
                CHECK(x == -1);
            }
        }
    }
    // joint top-k per (head, slice) row keeps at most topk + ties; at least one block somewhere
    CHECK(kept > 0);
    std::vector<uint16_t> ho(lq * C);
    cudaMemcpy(ho.data(), out, ho.size() * 2, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < ho.size(); i += 97) {
        const uint32_t bits = (uint32_t)ho[i] << 16;
        float f;
        std::memcpy(&f, &bits, 4);
        CHECK(std::isfinite(f) && std::fabs(f) <= 2.0f);  // a convex combination of values in [−2, 2)
    }
    // streaming layer: cache of 2 slices + 1 new slice per call
    fvsr_kv_cache* cache = nullptr;
    EXPECT_STATUS(fvsr_kv_cache_create(&p, 2, 1, &cache), FVSR_OK);
    if (cache) {
        const size_t slice = (size_t)s * 128 * C;
        EXPECT_STATUS(fvsr_kv_cache_append(cache, k, v, 1, fs), FVSR_OK);
        EXPECT_STATUS(fvsr_kv_cache_append(cache, k + slice, v + slice, 1, fs), FVSR_OK);
        int32_t n = 0;
        EXPECT_STATUS(fvsr_kv_cache_slices(cache, &n), FVSR_OK);
        CHECK(n == 2);
        EXPECT_STATUS(fvsr_lcsa_forward(&p, q, k + 2 * slice, v + 2 * slice, cache, out, kidx2, kcnt2, ws, ws_bytes,
                                        fs),
                      FVSR_OK);
        EXPECT_STATUS(fvsr_kv_cache_slices(cache, &n), FVSR_OK);
        CHECK(n == 2);  // appended one, trimmed back to kv_len
        EXPECT_STATUS(fvsr_device_check(fs), FVSR_OK);
        // cache ⊕ current = the same three slices as above in the same order: the same selection
        cudaMemcpy(hc2.data(), kcnt2, hc.size() * 4, cudaMemcpyDeviceToHost);
        CHECK(hc == hc2);
        EXPECT_STATUS(fvsr_kv_cache_destroy(cache), FVSR_OK);
    }
    // streaming driver: two chunks of one block from token-order linear outputs (q, k, v reused as such)
    {
        fvsr_stream* drv = nullptr;
        const int out_h = p.bh * 128, out_w = p.bw * 128;
        EXPECT_STATUS(fvsr_stream_create(p.heads, out_h, out_w, 1, FVSR_BF16, 0.0, 2.0, p.local_range, &drv), FVSR_OK);
        size_t dws = 0;
        if (drv) EXPECT_STATUS(fvsr_stream_workspace_size(drv, &dws), FVSR_OK);
        void* dw = nullptr;
        uint16_t *qwin = nullptr, *tout = nullptr;
        int32_t* tcnt = nullptr;
        const size_t l0 = (size_t)3 * s * 128;  // chunk 0: three slices
        cudaMalloc(&dw, dws);
        cudaMalloc(&qwin, l0 * C * 2);
        cudaMalloc(&tout, l0 * C * 2);
        cudaMalloc(&tcnt, sizeof(int32_t) * p.heads * 3 * s);
        CHECK(drv && dw && qwin && tout && tcnt);
        uint16_t* q0 = to_device(bf16_values(l0 * C, 11));
        uint16_t* k0 = to_device(bf16_values(l0 * C, 12));
        uint16_t* v0 = to_device(bf16_values(l0 * C, 13));
        EXPECT_STATUS(fvsr_stream_layer(drv, 0, q0, k0, v0, nullptr, nullptr, 1e-6f, qwin, tout, nullptr, tcnt, dw, dws,
                                        fs),
                      FVSR_EINVAL);  // no chunk started
        EXPECT_STATUS(fvsr_stream_begin(drv), FVSR_OK);
        EXPECT_STATUS(fvsr_stream_start_chunk(drv, 1, fs), FVSR_EINVAL);  // chunks run in order
        for (int chunk = 0; chunk < 2; ++chunk) {
            EXPECT_STATUS(fvsr_stream_start_chunk(drv, chunk, fs), FVSR_OK);
            EXPECT_STATUS(fvsr_stream_layer(drv, 0, q0, k0, v0, nullptr, nullptr, 1e-6f, qwin, tout, nullptr, tcnt, dw,
                                            dws, fs),
                          FVSR_OK);
            EXPECT_STATUS(fvsr_stream_layer(drv, 1, q0, k0, v0, nullptr, nullptr, 1e-6f, qwin, tout, nullptr, tcnt, dw,
                                            dws, fs),
                          FVSR_EINVAL);  // one block only
            EXPECT_STATUS(fvsr_device_check(fs), FVSR_OK);
            const size_t rows = (size_t)(chunk == 0 ? 3 : 1) * s * 128;
            std::vector<uint16_t> to(rows * C);
            cudaMemcpy(to.data(), tout, to.size() * 2, cudaMemcpyDeviceToHost);
            for (size_t i = 0; i < to.size(); i += 89) {
                const uint32_t bits = (uint32_t)to[i] << 16;
                float f;
                std::memcpy(&f, &bits, 4);
                CHECK(std::isfinite(f) && std::fabs(f) <= 2.0f);
            }
        }
        EXPECT_STATUS(fvsr_stream_destroy(drv), FVSR_OK);
        cudaFree(dw);
        cudaFree(qwin);
        cudaFree(tout);
        cudaFree(tcnt);
        cudaFree(q0);
        cudaFree(k0);
        cudaFree(v0);
    }
    cudaStreamDestroy(st);
    cudaFree(q);
    cudaFree(k);
    cudaFree(v);
    cudaFree(ws);
    cudaFree(kidx);
    cudaFree(kcnt);
    cudaFree(kidx2);
    cudaFree(kcnt2);
    cudaFree(probs);
    cudaFree(out);
    return g_failed;
}

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "cpu";
    const int failed = mode == "gpu" ? run_gpu() : run_cpu();
    if (failed == 0) std::printf("ok %s\n", mode.c_str());
    return failed == 0 ? 0 : 1;
}
