// Router entry point for callers that cannot allocate device memory.
//
// moe_router_topk needs a caller-provided workspace (a ticket per token plus the logits),
// so its caller must own a device allocator. Some callers have none: a C or FFI host
// (cgo, JNI, plain ctypes without a CUDA array library) that only receives device pointers
// from elsewhere, or a process whose device memory is entirely reserved by another
// framework's allocator so that any further cudaMalloc fails. This file gives those
// callers moe_router_topk_noalloc, which keeps the same scratch in a fixed-size array that
// is part of the library image on each device.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kNoAllocMaxTokens = 256;                               // tickets
constexpr int kNoAllocMaxTokenExperts = 65536;                       // T * E logits
constexpr size_t kTicketBytes = kNoAllocMaxTokens * sizeof(unsigned int);             // 1 KiB
constexpr size_t kLogitBytes = (size_t)kNoAllocMaxTokenExperts * sizeof(uint16_t);    // 128 KiB
constexpr size_t kScratchBytes = kTicketBytes + 2 * kLogitBytes;                      // 257 KiB

}  // namespace

// One copy per device that loads the library, held until the process exits. Shared by
// every call on that device: concurrent calls that overlap on the GPU race on it.
static __device__ __align__(256) unsigned char g_router_noalloc_scratch[kScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
unsigned char *g_scratch_dev[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};   // unique id of the context the address belongs to
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

// unique id of the calling thread's current context, 0 if none is bound
unsigned long long current_ctx_id() {
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    if (g_ctx_get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Device address of this device's copy of the scratch array. In host code the array's name
// is only a host-side handle, so the address is looked up through cudaGetSymbolAddress with
// the device current and cached together with the context it belongs to. A cudaDeviceReset
// between two calls destroys that context and reloads the module at a new address; the
// cached address is then stale, so a changed current context triggers a fresh lookup.
int scratch_for_current_device(unsigned char **out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return moe_set_cuda_error(e);
    if (dev < 0 || dev >= kMaxDevices)
        return moe_set_error(MOE_ENODEV, "router_topk_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_ctx_get_current || !g_ctx_get_id) {
        void *f1 = nullptr, *f2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1);
        if (e != cudaSuccess) return moe_set_cuda_error(e);
        e = cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2);
        if (e != cudaSuccess) return moe_set_cuda_error(e);
        if (q1 != cudaDriverEntryPointSuccess || !f1 || q2 != cudaDriverEntryPointSuccess || !f2)
            return moe_set_error(MOE_ECUDA, "router_topk_noalloc: context queries not available from the driver");
        g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
        g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
    }
    // 0 on a host thread where the runtime has not bound the primary context yet; the
    // symbol lookup below binds it
    unsigned long long id = current_ctx_id();
    if (id == 0 || !g_scratch_dev[dev] || g_scratch_ctx[dev] != id) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_router_noalloc_scratch);
        if (e != cudaSuccess) return moe_set_cuda_error(e);
        id = current_ctx_id();
        if (id == 0) return moe_set_error(MOE_ECUDA, "router_topk_noalloc: no current CUDA context");
        g_scratch_dev[dev] = static_cast<unsigned char *>(p);
        g_scratch_ctx[dev] = id;
    }
    *out = g_scratch_dev[dev];
    return MOE_OK;
}

}  // namespace

extern "C" int moe_router_topk_noalloc(const void *x, int T, int H, int E, int K, const void *w,
                                       const void *w_scales, const void *w_biases, int rbits,
                                       int group_size, int sb_fp16, const void *wn,
                                       const void *wn_scales, const void *wn_biases, int M,
                                       const float *pred_bias, void *out_logits, void *out_probs,
                                       uint32_t *out_inds, void *out_scores, uint32_t *out_pred,
                                       void *stream) {
    if (T <= 0 || E <= 0)
        return moe_set_error(MOE_EINVAL, "router_topk_noalloc: bad sizes T=%d E=%d", T, E);
    if (T > kNoAllocMaxTokens || (size_t)T * (size_t)E > (size_t)kNoAllocMaxTokenExperts)
        return moe_set_error(MOE_EINVAL,
                             "router_topk_noalloc: T=%d E=%d exceeds the static scratch "
                             "(T <= %d and T*E <= %d); use moe_router_topk with a workspace",
                             T, E, kNoAllocMaxTokens, kNoAllocMaxTokenExperts);
    unsigned char *base = nullptr;
    int rc = scratch_for_current_device(&base);
    if (rc) return rc;
    unsigned int *tickets = reinterpret_cast<unsigned int *>(base);
    uint16_t *logits = reinterpret_cast<uint16_t *>(base + kTicketBytes);
    uint16_t *plogits = reinterpret_cast<uint16_t *>(base + kTicketBytes + kLogitBytes);
    // The array keeps whatever the previous call left; the tickets must start at zero.
    cudaError_t e = cudaMemsetAsync(tickets, 0, (size_t)T * sizeof(unsigned int), as_stream(stream));
    if (e != cudaSuccess) return moe_set_cuda_error(e);
    return moe_router_launch(x, T, H, E, K, w, w_scales, w_biases, rbits, group_size, sb_fp16, wn, wn_scales,
                             wn_biases, M, pred_bias, out_logits, out_probs, out_inds, out_scores, out_pred,
                             tickets, logits, M > 0 ? plogits : nullptr, nullptr, nullptr, nullptr, 0, stream);
}
