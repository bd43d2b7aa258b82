// select_noalloc.cu — fvsr_lcsa_select for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc: a video app whose engine owns every device buffer under a
// fixed memory budget (the Swift/MLX side hands over only its own tensors), or a real-time streaming thread that
// must not take the device-wide synchronisation an allocation can imply. fvsr_lcsa_select needs scratch (pooled
// queries and keys, the radix-select histograms), which normally comes from a caller-provided workspace. This
// entry point takes it instead from one fixed array compiled into the library: kNoallocScratchBytes of device
// memory that every GPU which loads the library holds until the process exits.
//
// The array is shared by every call on a device and keeps the previous call's contents; what must start at zero
// (the histograms) is cleared on the stream by each call. Calls whose work overlaps on the GPU — on two streams
// at once, or from two threads — race on it, so one caller must order its calls on one stream.
#include <cstdio>
#include <mutex>
#include <vector>

#include "../../include/fvsr_lcsa.h"
#include "common.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = FVSR_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// Device address of the array for the current device. The address is looked up once per device, on that device's
// first call, with that device current; host code never dereferences the symbol itself.
cudaError_t scratch_address(void** out) {
    static std::mutex mu;
    static std::vector<void*> addr(256, nullptr);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= (int)addr.size()) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
    }
    *out = addr[dev];
    return cudaSuccess;
}

}  // namespace

namespace fvsr {
void set_last_error(const char* msg);  // api.cu: the message fvsr_last_error() returns
}

extern "C" fvsr_status fvsr_lcsa_select_noalloc(const fvsr_lcsa_params* p, const void* q, const void* k,
                                                const float* pooled_k, int32_t* kidx, int32_t* kcnt, uint8_t* mask,
                                                float* probs, fvsr_stream_t stream) {
    using namespace fvsr;
    char msg[256];
    // The same argument rules as fvsr_lcsa_select, checked through its workspace query.
    size_t ws_bytes = 0;
    fvsr_status s = fvsr_lcsa_workspace_size(p, &ws_bytes);
    if (s != FVSR_OK) return s;
    if (!q || (!k && !pooled_k) || !kidx || !kcnt || !probs) {
        set_last_error("q, k (or pooled_k), kidx, kcnt and probs are required");
        return FVSR_EINVAL;
    }
    auto misaligned = [](const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) != 0; };
    if (misaligned(q, 16) || misaligned(k, 16) || misaligned(pooled_k, 16)) {
        set_last_error("q, k and pooled_k must be 16-byte aligned");
        return FVSR_EINVAL;
    }
    if (misaligned(kidx, 4) || misaligned(kcnt, 4) || misaligned(probs, 4)) {
        set_last_error("kidx, kcnt and probs must be 4-byte aligned");
        return FVSR_EINVAL;
    }
    const int s_blocks = p->bh * p->bw;
    const int64_t nq = (int64_t)p->q_slices * s_blocks, nk = (int64_t)p->kv_slices * s_blocks;
    const int64_t channels = (int64_t)p->heads * 128;
    const size_t bq = round256(sizeof(float) * nq * channels);
    const size_t bk = pooled_k ? 0 : round256(sizeof(float) * nk * channels);
    const size_t bh = round256(select_hist_bytes(p->heads, p->q_slices));
    if (bq + bk + bh > kNoallocScratchBytes) {
        snprintf(msg, sizeof(msg),
                 "this call needs %zu bytes of scratch; the allocation-free entry point has %zu (use fvsr_lcsa_select)",
                 bq + bk + bh, kNoallocScratchBytes);
        set_last_error(msg);
        return FVSR_EUNSUPPORTED;
    }
    void* base = nullptr;
    if (scratch_address(&base) != cudaSuccess) {
        set_last_error("cudaGetSymbolAddress of the scratch array failed");
        return FVSR_ECUDA;
    }
    unsigned char* b = static_cast<unsigned char*>(base);
    float* pq = reinterpret_cast<float*>(b);
    float* pk = pooled_k ? const_cast<float*>(pooled_k) : reinterpret_cast<float*>(b + bq);
    uint32_t* hist = reinterpret_cast<uint32_t*>(b + bq + bk);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    KvPages pages{};
    pages.s = (int32_t)nk;
    cudaError_t e = launch_pool2(q, nq, pq, nullptr, pooled_k ? nullptr : k, pooled_k ? 0 : nk, pk, p->dtype,
                                 (int)channels, st);
    if (e == cudaSuccess)
        e = launch_select_scores(pq, pk, pages, p->heads, (int)nq, (int)nk, p->bh, p->bw, p->local_range, p->q_slices,
                                 p->topk, probs, hist, st);  // clears the histograms on the stream first
    if (e == cudaSuccess)
        e = launch_select_threshold(probs, p->heads, (int)nq, (int)nk, p->q_slices, p->topk, hist, kidx, kcnt, mask, st);
    if (e != cudaSuccess) {
        snprintf(msg, sizeof(msg), "launch failed: %s", cudaGetErrorString(e));
        set_last_error(msg);
        return FVSR_ECUDA;
    }
    return FVSR_OK;
}
