// Expert fills: copy the experts named by a miss / prefetch list (eid -> slot) from the
// pinned host pool into the device slot buffers. Replaces the reference's pread worker pool
// (mlx-qwen38/expert_io.c:113-356), which read each expert's nine tensors from the SSD
// shard into the MLX slot arrays.
//
// Two ways to run a fill:
//   * moe_fill_slots: a kernel reads the list where the LRU kernel wrote it (device memory)
//     and streams the rows from the host pool through the mapped pinned mapping (PCIe reads
//     issued by the SMs, 16 bytes per thread, several in flight). No host round trip, so
//     the whole LRU step + fill + expert compute sequence can be stream-ordered or captured
//     in a CUDA graph.
//   * moe_fill_slots_host: the list is on the host (the caller already synchronised, as the
//     reference's c_layer_step_decode does): one cudaMemcpyAsync per (expert, tensor) row on
//     the given (copy) stream, i.e. the copy engines.
// A "tensor" is any per-expert row array: the nine MLX tensors (row = one expert's slice),
// or the packed layout (one tensor, row = one whole expert).
#include <mutex>
#include <unordered_set>

#include "common.cuh"

namespace {

constexpr int kFillMaxTensors = 9;

struct FillTensor {
    const unsigned char *src;   // host pool base (device-accessible address), row e at src + e * bytes
    unsigned char *dst;         // slot buffer base, row s at dst + s * bytes
    uint64_t bytes;             // row bytes (multiple of 16)
};

struct FillArgs {
    const int32_t *list;        // {n, eids[stride], slots[stride]}
    int stride, nt, E, cap;
    FillTensor t[kFillMaxTensors];
    uint64_t pre[kFillMaxTensors + 1];   // prefix sums of row bytes / 16
};

__global__ void __launch_bounds__(256) fill_kernel(FillArgs a) {
    const int n = a.list[0];
    if (n <= 0 || n > a.stride) return;
    const uint64_t per = a.pre[a.nt];                 // 16-byte chunks per expert
    const uint64_t total = per * (uint64_t)n;
    const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t base = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; base < total; base += 4 * step) {
        uint4 v[4];
        unsigned char *d[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint64_t c = base + u * step;
            d[u] = nullptr;
            if (c >= total) continue;
            const int i = (int)(c / per);
            uint64_t r = c - (uint64_t)i * per;
            int t = 0;
            while (t + 1 < a.nt && r >= a.pre[t + 1]) ++t;
            r -= a.pre[t];
            const int e = a.list[1 + i], s = a.list[1 + a.stride + i];
            if (e < 0 || e >= a.E || s < 0 || s >= a.cap) {
                atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
                continue;
            }
            const FillTensor &ft = a.t[t];
            v[u] = *reinterpret_cast<const uint4 *>(ft.src + (uint64_t)e * ft.bytes + r * 16);
            d[u] = ft.dst + (uint64_t)s * ft.bytes + r * 16;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (d[u]) *reinterpret_cast<uint4 *>(d[u]) = v[u];
    }
}

int fill_tensors(FillArgs &a, int nt, const void *const *src, void *const *dst, const uint64_t *row_bytes) {
    if (nt <= 0 || nt > kFillMaxTensors) return moe_set_error(MOE_EINVAL, "fill: %d tensors", nt);
    a.nt = nt;
    a.pre[0] = 0;
    for (int t = 0; t < nt; ++t) {
        if (!src[t] || !dst[t] || row_bytes[t] == 0 || row_bytes[t] % 16 ||
            reinterpret_cast<uintptr_t>(src[t]) % 16 || reinterpret_cast<uintptr_t>(dst[t]) % 16)
            return moe_set_error(MOE_EINVAL, "fill: tensor %d needs 16-byte aligned bases and row bytes", t);
        a.t[t] = FillTensor{static_cast<const unsigned char *>(src[t]), static_cast<unsigned char *>(dst[t]),
                            row_bytes[t]};
        a.pre[t + 1] = a.pre[t] + row_bytes[t] / 16;
    }
    return MOE_OK;
}

std::mutex g_src_mu;
std::unordered_set<const void *> g_src_ok;

int check_source(const void *p, int t) {
    {
        std::lock_guard<std::mutex> lk(g_src_mu);
        if (g_src_ok.count(p)) return MOE_OK;
    }
    cudaPointerAttributes pa{};
    MOE_CUDA_TRY(cudaPointerGetAttributes(&pa, p));
    if (pa.type != cudaMemoryTypeHost && pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged)
        return moe_set_error(MOE_EINVAL, "fill_slots: tensor %d source is pageable host memory", t);
    if (pa.type == cudaMemoryTypeHost && pa.devicePointer != p)
        return moe_set_error(MOE_EINVAL, "fill_slots: tensor %d pinned source is not mapped at its host address", t);
    std::lock_guard<std::mutex> lk(g_src_mu);
    g_src_ok.insert(p);
    return MOE_OK;
}

}  // namespace

extern "C" int moe_fill_slots(const int32_t *list, int stride, int E, int cap, int ntensors,
                              const void *const *host_src, void *const *dev_dst, const uint64_t *row_bytes,
                              int num_ctas, void *stream) {
    if (!list || stride <= 0 || E <= 0 || cap <= 0 || !host_src || !dev_dst || !row_bytes)
        return moe_set_error(MOE_EINVAL, "fill_slots: bad arguments");
    FillArgs a{};
    a.list = list;
    a.stride = stride;
    a.E = E;
    a.cap = cap;
    if (int rc = fill_tensors(a, ntensors, host_src, dev_dst, row_bytes)) return rc;
    // the pool must be reachable from the device: pinned (page-locked) host memory, whose
    // device address equals the host address under unified addressing, or device memory.
    // Checked once per base address (later calls may be inside a stream capture).
    for (int t = 0; t < ntensors; ++t)
        if (int rc = check_source(host_src[t], t)) return rc;
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        MOE_CUDA_TRY(cudaGetDevice(&dev));
        MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    }
    const int grid = num_ctas > 0 ? num_ctas : sms;
    fill_kernel<<<grid, 256, 0, as_stream(stream)>>>(a);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" int moe_fill_slots_host(const int32_t *list_host, int stride, int E, int cap, int ntensors,
                                   const void *const *host_src, void *const *dev_dst, const uint64_t *row_bytes,
                                   void *stream) {
    if (!list_host || stride <= 0 || E <= 0 || cap <= 0 || !host_src || !dev_dst || !row_bytes)
        return moe_set_error(MOE_EINVAL, "fill_slots_host: bad arguments");
    FillArgs a{};
    if (int rc = fill_tensors(a, ntensors, host_src, dev_dst, row_bytes)) return rc;
    const int n = list_host[0];
    if (n < 0 || n > stride) return moe_set_error(MOE_EINVAL, "fill_slots_host: list count %d", n);
    for (int i = 0; i < n; ++i) {
        const int e = list_host[1 + i], s = list_host[1 + stride + i];
        if (e < 0 || e >= E || s < 0 || s >= cap)
            return moe_set_error(MOE_EINVAL, "fill_slots_host: entry %d (expert %d -> slot %d)", i, e, s);
        for (int t = 0; t < ntensors; ++t)
            MOE_CUDA_TRY(cudaMemcpyAsync(a.t[t].dst + (uint64_t)s * a.t[t].bytes,
                                         a.t[t].src + (uint64_t)e * a.t[t].bytes, a.t[t].bytes,
                                         cudaMemcpyHostToDevice, as_stream(stream)));
    }
    return MOE_OK;
}
