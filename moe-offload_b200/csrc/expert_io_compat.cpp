// Drop-in replacement of the reference's expert cache C ABI (mlx-qwen38/expert_io.c:428-852:
// c_io_init, c_layer_init, c_layer_step_decode*, c_layer_start_prefetch*, c_layer_load_sync,
// c_layer_get/set_lru_state, c_layer_get_stats, c_get_decode_totals, ...), same names and
// signatures, same calling convention (one calling thread, layer ids 0..63, invalid layer
// ids ignored silently, eids passed in host memory, n_miss returned).
//
// What changes underneath: the cache state lives on the GPU (moe_lru_* in lru.cu) and the
// expert bytes come from a pinned host pool registered per layer instead of an SSD shard.
// Each call stages its host arguments through pinned buffers, runs the one-thread LRU kernel
// on the library's stream, and reads back the miss list; fills are cudaMemcpyAsync on the
// library's copy stream (synchronous for c_layer_step_decode, asynchronous for the _async
// variants and for prefetches, waited by c_layer_wait_demand / c_layer_wait_prefetch or at
// the start of the next call, as the reference's wait_async_batch does). slot_inds_ptr may
// be device memory (written by the kernel) or host memory (written after the read-back).
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/moe_b200.h"

int moe_set_error(int code, const char *fmt, ...);   // errors.cpp

namespace {

constexpr int kMaxLayers = 64;
constexpr int kMaxTensors = 9;
constexpr int kRefExperts = 512;                   // the reference's NUM_EXPERTS
constexpr uint64_t kRefExpertBytes = 1536000ull;   // the reference's EXPERT_BYTES (stats unit)
constexpr int kListMax = 1 + 2 * 2048;

struct CompatLayer {
    bool init = false;
    int E = kRefExperts, cap = 0, nt = 0;
    uint64_t expert_bytes = kRefExpertBytes;
    uint64_t row_bytes[kMaxTensors] = {};
    void *dst[kMaxTensors] = {};
    const void *src[kMaxTensors] = {};
    bool have_pool = false;
    uint32_t *slot_inds = nullptr;
    bool slots_on_device = false;
    void *state = nullptr;
};

struct Compat {
    std::mutex mu;
    bool io = false;
    cudaStream_t st = nullptr, copy = nullptr;
    cudaEvent_t fills = nullptr;
    bool fills_pending = false;
    uint32_t *h_eids = nullptr, *d_eids = nullptr;
    int32_t *h_list = nullptr, *d_list = nullptr, *h_ord = nullptr, *d_ord = nullptr;
    uint32_t *h_slots = nullptr, *d_slots = nullptr;
    uint64_t *h_stats = nullptr, *d_stats = nullptr;
    CompatLayer L[kMaxLayers];
};

Compat g;

bool ok(cudaError_t e) { return e == cudaSuccess; }

bool ensure_io() {
    if (g.io) return true;
    bool good = ok(cudaStreamCreateWithFlags(&g.st, cudaStreamNonBlocking)) &&
                ok(cudaStreamCreateWithFlags(&g.copy, cudaStreamNonBlocking)) &&
                ok(cudaEventCreateWithFlags(&g.fills, cudaEventDisableTiming)) &&
                ok(cudaHostAlloc(&g.h_eids, 64 * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_eids, 64 * 4)) &&
                ok(cudaHostAlloc(&g.h_list, kListMax * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_list, kListMax * 4)) &&
                ok(cudaHostAlloc(&g.h_ord, 2 * 2048 * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_ord, 2 * 2048 * 4)) &&
                ok(cudaHostAlloc(&g.h_slots, 64 * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_slots, 64 * 4)) &&
                ok(cudaHostAlloc(&g.h_stats, 18 * 8, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_stats, 18 * 8));
    g.io = good;
    return good;
}

CompatLayer *layer(int i) {
    if (i < 0 || i >= kMaxLayers || !g.io || !g.L[i].init) return nullptr;
    return &g.L[i];
}

// the reference's wait_async_batch: every call first waits for outstanding fills
void wait_fills() {
    if (g.fills_pending) {
        cudaEventSynchronize(g.fills);
        g.fills_pending = false;
    }
}

// fills of list h_list (stride) on the copy stream; async: leave them pending
void issue_fills(CompatLayer *L, int stride, bool async) {
    if (!L->have_pool || g.h_list[0] <= 0) return;
    if (moe_fill_slots_host(g.h_list, stride, L->E, L->cap, L->nt, L->src, L->dst, L->row_bytes, g.copy) != 0)
        return;
    cudaEventRecord(g.fills, g.copy);
    g.fills_pending = true;
    if (!async) wait_fills();
}

int layer_init(int li, int E, int cap, uint64_t expert_bytes, int nt, const uint64_t *row_bytes,
               const uint64_t *base_ptrs, const uint64_t *host_ptrs, uint64_t slot_inds_ptr) {
    if (li < 0 || li >= kMaxLayers) return MOE_EINVAL;
    if (!ensure_io()) return moe_set_error(MOE_ECUDA, "c_layer_init: CUDA setup failed");
    wait_fills();
    CompatLayer &L = g.L[li];
    if (L.state) cudaFree(L.state);
    L = CompatLayer{};
    L.E = E;
    L.cap = cap;
    L.expert_bytes = expert_bytes;
    L.nt = nt;
    bool pool = host_ptrs != nullptr;
    for (int t = 0; t < nt; ++t) {
        L.row_bytes[t] = row_bytes ? row_bytes[t] : 0;
        L.dst[t] = base_ptrs ? reinterpret_cast<void *>(static_cast<uintptr_t>(base_ptrs[t])) : nullptr;
        L.src[t] = host_ptrs ? reinterpret_cast<const void *>(static_cast<uintptr_t>(host_ptrs[t])) : nullptr;
        pool = pool && L.row_bytes[t] > 0 && L.dst[t] && L.src[t];
    }
    L.have_pool = pool && nt > 0;
    L.slot_inds = reinterpret_cast<uint32_t *>(static_cast<uintptr_t>(slot_inds_ptr));
    if (L.slot_inds) {
        cudaPointerAttributes pa{};
        L.slots_on_device = ok(cudaPointerGetAttributes(&pa, L.slot_inds)) &&
                            (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged ||
                             (pa.type == cudaMemoryTypeHost && pa.devicePointer == L.slot_inds));
        cudaGetLastError();
    }
    const size_t sb = moe_lru_state_bytes(E, cap);
    if (sb == 0) return moe_set_error(MOE_EINVAL, "c_layer_init: E=%d capacity=%d", E, cap);
    if (!ok(cudaMalloc(&L.state, sb))) return moe_set_error(MOE_ENOMEM, "c_layer_init: state allocation");
    if (int rc = moe_lru_init(L.state, E, cap, expert_bytes, g.st)) return rc;
    if (!ok(cudaStreamSynchronize(g.st))) return moe_set_error(MOE_ECUDA, "c_layer_init: sync");
    L.init = true;
    return MOE_OK;
}

}  // namespace

extern "C" {

void c_io_init(int num_threads) {
    (void)num_threads;   // fills run on the copy engines, not on host worker threads
    std::lock_guard<std::mutex> lk(g.mu);
    ensure_io();
}

void c_layer_init(int layer_idx, int fd, int capacity, const uint64_t *base_offsets, const uint64_t *row_bytes,
                  const uint64_t *base_ptrs, uint64_t slot_inds_ptr) {
    (void)fd;
    (void)base_offsets;   // the expert bytes come from a pinned host pool (c_layer_set_host_pool)
    std::lock_guard<std::mutex> lk(g.mu);
    layer_init(layer_idx, kRefExperts, capacity, kRefExpertBytes, kMaxTensors, row_bytes, base_ptrs, nullptr,
               slot_inds_ptr);
}

int c_layer_init_ex(int layer_idx, int num_experts, int capacity, uint64_t expert_bytes, int ntensors,
                    const uint64_t *row_bytes, const uint64_t *base_ptrs, const uint64_t *host_ptrs,
                    uint64_t slot_inds_ptr) {
    if (ntensors < 0 || ntensors > kMaxTensors) return moe_set_error(MOE_EINVAL, "c_layer_init_ex: %d tensors", ntensors);
    std::lock_guard<std::mutex> lk(g.mu);
    return layer_init(layer_idx, num_experts, capacity, expert_bytes, ntensors, row_bytes, base_ptrs, host_ptrs,
                      slot_inds_ptr);
}

void c_layer_set_host_pool(int layer_idx, const uint64_t *host_ptrs) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L || !host_ptrs) return;
    bool pool = L->nt > 0;
    for (int t = 0; t < L->nt; ++t) {
        L->src[t] = reinterpret_cast<const void *>(static_cast<uintptr_t>(host_ptrs[t]));
        pool = pool && L->src[t] && L->row_bytes[t] > 0 && L->dst[t];
    }
    L->have_pool = pool;
}

void c_layer_reset_cache(int layer_idx) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L) return;
    wait_fills();
    moe_lru_reset(L->state, L->E, L->cap, 0, g.st);
    cudaStreamSynchronize(g.st);
}

void c_layer_reset_stats(int layer_idx) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L) return;
    moe_lru_reset(L->state, L->E, L->cap, 1, g.st);
    cudaStreamSynchronize(g.st);
}

void c_layer_wait_prefetch(int layer_idx) {
    (void)layer_idx;
    std::lock_guard<std::mutex> lk(g.mu);
    wait_fills();
}

void c_layer_wait_demand(int layer_idx) {
    (void)layer_idx;
    std::lock_guard<std::mutex> lk(g.mu);
    wait_fills();
}

void c_layer_start_prefetch(int layer_idx, const int32_t *pred_eids, int pred_count, int max_fetch) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L || pred_count < 0 || pred_count > 64) return;
    wait_fills();
    const int mf = (max_fetch > 0 && max_fetch < 32) ? max_fetch : 32;
    if (pred_count > 0) std::memcpy(g.h_eids, pred_eids, (size_t)pred_count * 4);
    cudaMemcpyAsync(g.d_eids, g.h_eids, (size_t)pred_count * 4, cudaMemcpyHostToDevice, g.st);
    if (moe_lru_prefetch(L->state, L->E, L->cap, reinterpret_cast<const int32_t *>(g.d_eids), pred_count, mf,
                         g.d_list, g.st) != 0)
        return;
    cudaMemcpyAsync(g.h_list, g.d_list, (size_t)(1 + 2 * mf) * 4, cudaMemcpyDeviceToHost, g.st);
    cudaStreamSynchronize(g.st);
    issue_fills(L, mf, true);
}

int c_layer_step_decode_ex(int layer_idx, const uint32_t *eids, int k, int async_io) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L || k <= 0 || k > 32) return 0;
    wait_fills();
    std::memcpy(g.h_eids, eids, (size_t)k * 4);
    cudaMemcpyAsync(g.d_eids, g.h_eids, (size_t)k * 4, cudaMemcpyHostToDevice, g.st);
    uint32_t *out = (L->slot_inds && L->slots_on_device) ? L->slot_inds : g.d_slots;
    if (moe_lru_step(L->state, L->E, L->cap, g.d_eids, k, out, g.d_list, g.st) != 0) return 0;
    cudaMemcpyAsync(g.h_list, g.d_list, (size_t)(1 + 2 * k) * 4, cudaMemcpyDeviceToHost, g.st);
    if (L->slot_inds && !L->slots_on_device)
        cudaMemcpyAsync(g.h_slots, g.d_slots, (size_t)k * 4, cudaMemcpyDeviceToHost, g.st);
    if (!ok(cudaStreamSynchronize(g.st))) return 0;
    if (L->slot_inds && !L->slots_on_device) std::memcpy(L->slot_inds, g.h_slots, (size_t)k * 4);
    const int n = g.h_list[0];
    if (n < 0) return 0;
    issue_fills(L, k, async_io != 0);
    return n;
}

int c_layer_step_decode(int layer_idx, const uint32_t *eids, int k) {
    return c_layer_step_decode_ex(layer_idx, eids, k, 0);
}

int c_layer_step_decode10(int layer_idx, uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3, uint32_t e4,
                          uint32_t e5, uint32_t e6, uint32_t e7, uint32_t e8, uint32_t e9) {
    const uint32_t eids[10] = {e0, e1, e2, e3, e4, e5, e6, e7, e8, e9};
    return c_layer_step_decode_ex(layer_idx, eids, 10, 0);
}

int c_layer_step_decode10_async(int layer_idx, uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3, uint32_t e4,
                                uint32_t e5, uint32_t e6, uint32_t e7, uint32_t e8, uint32_t e9) {
    const uint32_t eids[10] = {e0, e1, e2, e3, e4, e5, e6, e7, e8, e9};
    return c_layer_step_decode_ex(layer_idx, eids, 10, 1);
}

void c_layer_start_prefetch10(int layer_idx, int max_fetch, int32_t e0, int32_t e1, int32_t e2, int32_t e3,
                              int32_t e4, int32_t e5, int32_t e6, int32_t e7, int32_t e8, int32_t e9) {
    const int32_t p[10] = {e0, e1, e2, e3, e4, e5, e6, e7, e8, e9};
    c_layer_start_prefetch(layer_idx, p, 10, max_fetch);
}

void c_layer_start_prefetch12(int layer_idx, int max_fetch, int32_t e0, int32_t e1, int32_t e2, int32_t e3,
                              int32_t e4, int32_t e5, int32_t e6, int32_t e7, int32_t e8, int32_t e9, int32_t e10,
                              int32_t e11) {
    const int32_t p[12] = {e0, e1, e2, e3, e4, e5, e6, e7, e8, e9, e10, e11};
    c_layer_start_prefetch(layer_idx, p, 12, max_fetch);
}

void c_layer_load_sync(int layer_idx, const int32_t *eids, const int32_t *slots, int count, int is_prefill) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L || count <= 0 || count > 2048) return;
    wait_fills();
    if (is_prefill) {
        moe_lru_add_stat(L->state, L->E, L->cap, 9, (uint64_t)count * L->expert_bytes, g.st);
        cudaStreamSynchronize(g.st);
    }
    g.h_list[0] = count;
    for (int i = 0; i < count; ++i) {
        g.h_list[1 + i] = eids[i];
        g.h_list[1 + count + i] = slots[i];
    }
    // the reference's I/O accounting of the fill (expert_io.c:186-233): 9 reads per expert and
    // 9 per run of consecutive expert ids
    int runs = 0;
    {
        std::vector<int32_t> s(eids, eids + count);
        std::sort(s.begin(), s.end());
        runs = 1;
        for (int i = 1; i < count; ++i) runs += (s[i] != s[i - 1] + 1) ? 1 : 0;
    }
    moe_lru_add_stat(L->state, L->E, L->cap, 16, (uint64_t)count * 9, g.st);
    moe_lru_add_stat(L->state, L->E, L->cap, 17, (uint64_t)runs * 9, g.st);
    cudaStreamSynchronize(g.st);
    issue_fills(L, count, false);
}

void c_layer_get_lru_state(int layer_idx, int32_t *out_eids, int32_t *out_slots, int *out_count) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L) {
        *out_count = 0;
        return;
    }
    wait_fills();
    if (moe_lru_get_state(L->state, L->E, L->cap, g.d_list, g.st) != 0) {
        *out_count = 0;
        return;
    }
    cudaMemcpyAsync(g.h_list, g.d_list, (size_t)(1 + 2 * L->cap) * 4, cudaMemcpyDeviceToHost, g.st);
    cudaStreamSynchronize(g.st);
    const int n = g.h_list[0];
    for (int i = 0; i < n; ++i) {
        out_eids[i] = g.h_list[1 + i];
        out_slots[i] = g.h_list[1 + L->cap + i];
    }
    *out_count = n;
}

void c_layer_set_lru_state(int layer_idx, const int32_t *ordered_eids, const int32_t *ordered_slots, int count,
                           uint64_t add_prefill_requests, uint64_t add_prefill_hits, uint64_t add_prefill_misses) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L || count < 0 || count > L->cap) return;
    wait_fills();
    if (count > 0) {
        std::memcpy(g.h_ord, ordered_eids, (size_t)count * 4);
        std::memcpy(g.h_ord + 2048, ordered_slots, (size_t)count * 4);
        cudaMemcpyAsync(g.d_ord, g.h_ord, 2 * 2048 * 4, cudaMemcpyHostToDevice, g.st);
    }
    moe_lru_set_state(L->state, L->E, L->cap, g.d_ord, g.d_ord + 2048, count, add_prefill_requests,
                      add_prefill_hits, add_prefill_misses, g.st);
    cudaStreamSynchronize(g.st);
}

void c_layer_get_stats(int layer_idx, uint64_t *out_stats) {
    std::lock_guard<std::mutex> lk(g.mu);
    CompatLayer *L = layer(layer_idx);
    if (!L) return;
    if (moe_lru_get_stats(L->state, L->E, L->cap, g.d_stats, g.st) != 0) return;
    cudaMemcpyAsync(g.h_stats, g.d_stats, 18 * 8, cudaMemcpyDeviceToHost, g.st);
    cudaStreamSynchronize(g.st);
    std::memcpy(out_stats, g.h_stats, 18 * 8);
}

void c_get_decode_totals(int num_layers, uint64_t *out6) {
    uint64_t lru_h = 0, pref_h = 0, dem_m = 0, req = 0, dem_b = 0, pref_b = 0;
    if (num_layers > kMaxLayers) num_layers = kMaxLayers;
    for (int il = 1; il < num_layers; ++il) {     // layer 0 is pinned
        uint64_t s[18] = {};
        if (!layer(il)) continue;
        c_layer_get_stats(il, s);
        lru_h += s[1];
        pref_h += s[2];
        dem_m += s[3];
        req += s[0];
        dem_b += s[4];
        pref_b += s[5];
    }
    out6[0] = lru_h;
    out6[1] = pref_h;
    out6[2] = dem_m;
    out6[3] = req;
    out6[4] = dem_b;
    out6[5] = pref_b;
}

}  // extern "C"
