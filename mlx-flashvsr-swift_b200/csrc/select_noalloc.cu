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
#include <cuda.h>

#include <cstdio>
#include <map>
#include <mutex>

#include "../../include/fvsr_lcsa.h"
#include "common.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = FVSR_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

// The calling thread's current CUDA context (the driver's cuCtxGetCurrent, resolved once through the runtime), or
// NULL when it cannot be read. A __device__ array's address belongs to a context, not to a device number: a host
// that runs its own driver-API context, or one that reset the device, sees a new address.
CUcontext current_context() {
    typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    CUcontext ctx = nullptr;
    if (!fn || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

// Device address of the array in the current context, with the context current; host code never dereferences the
// symbol itself. Outside stream capture it is looked up afresh on every call (a cheap query), so a context that was
// destroyed and re-created, or a host-owned context, always gets its own address. Inside a capture no lookup is made
// (it could load the module, which a capture forbids); the address recorded by this context's last call outside a
// capture is used, and a context with no such call is refused.
cudaError_t scratch_address(cudaStream_t st, void** out) {
    static std::mutex mu;
    static std::map<CUcontext, void*> addr;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess) return e;
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lock(mu);
    if (cs == cudaStreamCaptureStatusNone) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        if (ctx) addr[ctx] = p;
        *out = p;
        return cudaSuccess;
    }
    const auto it = ctx ? addr.find(ctx) : addr.end();
    if (it == addr.end()) return cudaErrorStreamCaptureUnsupported;
    *out = it->second;
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
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    void* base = nullptr;
    const cudaError_t ea = scratch_address(st, &base);
    if (ea == cudaErrorStreamCaptureUnsupported) {
        set_last_error("the first call in a CUDA context must come before any stream capture (it looks the scratch "
                       "array's address up)");
        return FVSR_EINVAL;
    }
    if (ea != cudaSuccess) {
        snprintf(msg, sizeof(msg), "looking up the scratch array's address failed: %s", cudaGetErrorString(ea));
        set_last_error(msg);
        return FVSR_ECUDA;
    }
    unsigned char* b = static_cast<unsigned char*>(base);
    float* pq = reinterpret_cast<float*>(b);
    float* pk = pooled_k ? const_cast<float*>(pooled_k) : reinterpret_cast<float*>(b + bq);
    uint32_t* hist = reinterpret_cast<uint32_t*>(b + bq + bk);
    KvPages pages{};
    pages.s = (int32_t)nk;
    // the pooling launch also clears the histograms (the scratch keeps the previous call's counts), as in
    // fvsr_lcsa_select, so no memset runs in between
    cudaError_t e = launch_pool2(q, nq, pq, nullptr, pooled_k ? nullptr : k, pooled_k ? 0 : nk, pk, p->dtype,
                                 (int)channels, st, hist, select_hist_bytes(p->heads, p->q_slices) / 4);
    if (e == cudaSuccess)
        e = launch_select(pq, pk, pages, p->heads, (int)nq, (int)nk, p->bh, p->bw, p->local_range, p->q_slices,
                          p->topk, probs, hist, kidx, kcnt, mask, nullptr, st);
    if (e != cudaSuccess) {
        snprintf(msg, sizeof(msg), "launch failed: %s", cudaGetErrorString(e));
        set_last_error(msg);
        return FVSR_ECUDA;
    }
    return FVSR_OK;
}
