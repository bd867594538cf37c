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
//
// The newer reference's additions (cpp/third_party/expert_io.c:1002-1396, declared in
// cpp/src/expert_io.h:87-106) are here too: per-token I/O accounting (c_set_io_accounting,
// c_begin_decode_token, c_end_decode_token) kept in one device LruAcct that every layer's LRU
// kernel updates, the single-call scheduled step c_layer_decode_step_sched (demand step of one
// layer protecting its in-flight prefetch, then the next layer's deduplicated prefetch, demand
// fills queued before prefetch fills) and its hit/miss split records (c_layer_get_split_inds).
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
constexpr int kEidsMax = 128;                      // staged eids: a demand step's 16, then 64 predictions
constexpr int kSchedK = 16;                        // the scheduled step's cap on k
constexpr int kPrefList = 128;                     // offset of the prefetch list in the list buffers
constexpr int kFlagSyncDemand = 1, kFlagNoPrefetch = 2, kFlagSplit = 4;   // cpp/src/expert_io.h:8-12

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

// the last hit/miss split of a layer's scheduled step: written only by a split step, kept
// through layer re-initialisation, as the reference's per-layer split arrays are
struct SplitRecord {
    int hit = 0, miss = 0, k = 0;
    uint32_t hit_slots[kSchedK] = {}, miss_slots[kSchedK] = {};
    int32_t inv[kSchedK] = {};
};

// host mirror of the device LruAcct header (lru.cu); counters live only on the device
struct AcctHeader {
    int32_t enabled, cur_token, pad0, pad1;
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
    // per-token accounting: device record (header + 9 counters), its pinned staging copy,
    // the token step counter and the filled bytes of the token in progress
    void *d_acct = nullptr;
    unsigned char *h_acct = nullptr;
    size_t acct_bytes = 0;
    AcctHeader acct{0, -1, 0, 0};
    int32_t token_step = 0;
    uint64_t tok_fill_bytes = 0;
    CompatLayer L[kMaxLayers];
    SplitRecord split[kMaxLayers];
};

Compat g;

bool ok(cudaError_t e) { return e == cudaSuccess; }

bool ensure_io() {
    if (g.io) return true;
    bool good = ok(cudaStreamCreateWithFlags(&g.st, cudaStreamNonBlocking)) &&
                ok(cudaStreamCreateWithFlags(&g.copy, cudaStreamNonBlocking)) &&
                ok(cudaEventCreateWithFlags(&g.fills, cudaEventDisableTiming)) &&
                ok(cudaHostAlloc(&g.h_eids, kEidsMax * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_eids, kEidsMax * 4)) &&
                ok(cudaHostAlloc(&g.h_list, kListMax * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_list, kListMax * 4)) &&
                ok(cudaHostAlloc(&g.h_ord, 2 * 2048 * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_ord, 2 * 2048 * 4)) &&
                ok(cudaHostAlloc(&g.h_slots, 64 * 4, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_slots, 64 * 4)) &&
                ok(cudaHostAlloc(&g.h_stats, 18 * 8, cudaHostAllocDefault)) &&
                ok(cudaMalloc(&g.d_stats, 18 * 8));
    if (good) {
        g.acct_bytes = moe_lru_acct_bytes();
        good = ok(cudaMalloc(&g.d_acct, g.acct_bytes)) &&
               ok(cudaHostAlloc(reinterpret_cast<void **>(&g.h_acct), g.acct_bytes, cudaHostAllocDefault));
        if (good) {
            std::memset(g.h_acct, 0, g.acct_bytes);
            std::memcpy(g.h_acct, &g.acct, sizeof(AcctHeader));
            good = ok(cudaMemcpyAsync(g.d_acct, g.h_acct, g.acct_bytes, cudaMemcpyHostToDevice, g.st)) &&
                   ok(cudaStreamSynchronize(g.st));
        }
    }
    g.io = good;
    return good;
}

// push the host accounting header (and, with zero_counters, cleared counters) to the device
void push_acct(bool zero_counters) {
    if (!g.io) return;
    if (zero_counters) std::memset(g.h_acct, 0, g.acct_bytes);
    std::memcpy(g.h_acct, &g.acct, sizeof(AcctHeader));
    cudaMemcpyAsync(g.d_acct, g.h_acct, zero_counters ? g.acct_bytes : sizeof(AcctHeader), cudaMemcpyHostToDevice,
                    g.st);
    cudaStreamSynchronize(g.st);
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

// fills of a host list {count, eids[stride], slots[stride]} on the copy stream; async: leave
// them pending. With accounting on, their bytes count as the token's read bytes (the
// reference's g_tok_pread_bytes).
void issue_fills(CompatLayer *L, const int32_t *list, int stride, bool async) {
    if (!L->have_pool || list[0] <= 0) return;
    if (moe_fill_slots_host(list, stride, L->E, L->cap, L->nt, L->src, L->dst, L->row_bytes, g.copy) != 0)
        return;
    if (g.acct.enabled) {
        uint64_t eb = 0;
        for (int t = 0; t < L->nt; ++t) eb += L->row_bytes[t];
        g.tok_fill_bytes += (uint64_t)list[0] * eb;
    }
    cudaEventRecord(g.fills, g.copy);
    g.fills_pending = true;
    if (!async) wait_fills();
}

void issue_fills(CompatLayer *L, int stride, bool async) { issue_fills(L, g.h_list, stride, async); }

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
    if (li == 1) {    // the reference's init resets the cache, and layer 1's reset the token count
        g.token_step = 0;
        g.acct.cur_token = -1;
        push_acct(false);
    }
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
    if (layer_idx == 1) {    // cpp/third_party/expert_io.c:570-573: layer 1 restarts the token count
        g.token_step = 0;
        g.acct.cur_token = -1;
        push_acct(false);
    }
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
    if (moe_lru_prefetch_ex(L->state, L->E, L->cap, reinterpret_cast<const int32_t *>(g.d_eids), pred_count, mf,
                            g.d_list, g.d_acct, 0, g.st) != 0)
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
    if (moe_lru_step_ex(L->state, L->E, L->cap, g.d_eids, k, out, g.d_list, g.d_acct, 0, g.st) != 0) return 0;
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

// cpp/third_party/expert_io.c:1002-1008
void c_set_io_accounting(int enabled) {
    std::lock_guard<std::mutex> lk(g.mu);
    if (!ensure_io()) return;
    wait_fills();
    g.acct.enabled = enabled ? 1 : 0;
    if (!g.acct.enabled) g.acct.cur_token = -1;
    push_acct(false);
}

// cpp/third_party/expert_io.c:1010-1024: the token index argument is not used; tokens are
// numbered by a counter that resetting layer 1's cache restarts
void c_begin_decode_token(int token_idx) {
    (void)token_idx;
    std::lock_guard<std::mutex> lk(g.mu);
    if (!ensure_io()) return;
    wait_fills();
    g.acct.cur_token = g.token_step++;
    g.tok_fill_bytes = 0;
    push_acct(true);
}

// cpp/third_party/expert_io.c:1026-1038: {LRU hits, demand misses, prefetch loads, prefetch
// hits, wasted prefetches, demand re-reads <=16 / <=64 tokens, prefetch re-reads <=16 / <=64,
// bytes read}; the bytes are those of the slot fills issued while accounting was on
void c_end_decode_token(uint64_t *out10) {
    std::lock_guard<std::mutex> lk(g.mu);
    if (!out10) return;
    std::memset(out10, 0, 10 * sizeof(uint64_t));
    if (!g.io) return;
    wait_fills();
    cudaMemcpyAsync(g.h_acct, g.d_acct, g.acct_bytes, cudaMemcpyDeviceToHost, g.st);
    if (!ok(cudaStreamSynchronize(g.st))) return;
    std::memcpy(out10, g.h_acct + sizeof(AcctHeader), 9 * sizeof(uint64_t));
    out10[9] = g.tok_fill_bytes;
}

// cpp/third_party/expert_io.c:1040-1042 reports the bytes of the module's static tables; here
// the module's own allocations: every layer's device LRU state plus the staging buffers
uint64_t c_get_native_buffer_bytes(void) {
    std::lock_guard<std::mutex> lk(g.mu);
    if (!g.io) return 0;
    uint64_t b = 2ull * (kEidsMax * 4 + kListMax * 4 + 2 * 2048 * 4 + 64 * 4 + 18 * 8) + 2ull * g.acct_bytes;
    for (int i = 0; i < kMaxLayers; ++i)
        if (g.L[i].init) b += moe_lru_state_bytes(g.L[i].E, g.L[i].cap);
    return b;
}

// cpp/third_party/expert_io.c:1062-1082
void c_layer_get_split_inds(int layer_idx, uint32_t *out_hit_slots, uint32_t *out_miss_slots,
                            int32_t *out_inv_order) {
    std::lock_guard<std::mutex> lk(g.mu);
    if (layer_idx < 0 || layer_idx >= kMaxLayers) return;
    const SplitRecord &r = g.split[layer_idx];
    if (r.hit > 0 && out_hit_slots) std::memcpy(out_hit_slots, r.hit_slots, (size_t)r.hit * 4);
    if (r.miss > 0 && out_miss_slots) std::memcpy(out_miss_slots, r.miss_slots, (size_t)r.miss * 4);
    if (r.k > 0 && out_inv_order) std::memcpy(out_inv_order, r.inv, (size_t)r.k * 4);
}

// cpp/third_party/expert_io.c:1094-1396. One call per layer: the demand step of `layer_idx`
// (k capped at 16; the experts the layer's last prefetch fetched stay protected), then the
// next layer's prefetch of `pred` (duplicates fetched once, at most prefetch_cap), both LRU
// kernels back to back on the library stream with one read-back; demand fills are queued on
// the copy stream before the prefetch fills. Layer 0 (pinned) takes no demand step. Returns
// the demand misses of `layer_idx`. flags: 1 wait for every fill before returning, 2 no
// prefetch, 4 record the hit/miss split for c_layer_get_split_inds.
int c_layer_decode_step_sched(int layer_idx, const int32_t *eids, int k, const int32_t *pred, int n_pred,
                              int next_layer, int prefetch_cap, int flags) {
    std::lock_guard<std::mutex> lk(g.mu);
    if (!g.io) return 0;
    wait_fills();
    CompatLayer *L = (layer_idx > 0) ? layer(layer_idx) : nullptr;
    const bool demand = L && eids && k > 0;
    if (demand && k > kSchedK) k = kSchedK;
    CompatLayer *Ln = (!(flags & kFlagNoPrefetch) && next_layer > 0) ? layer(next_layer) : nullptr;
    const bool pref = Ln && pred && n_pred > 0 && n_pred <= 64 && prefetch_cap > 0;
    const int mf = (prefetch_cap > 0 && prefetch_cap < 32) ? prefetch_cap : 32;
    uint32_t *out = nullptr;
    if (demand) {
        std::memcpy(g.h_eids, eids, (size_t)k * 4);
        out = (L->slot_inds && L->slots_on_device) ? L->slot_inds : g.d_slots;
    }
    if (pref) std::memcpy(reinterpret_cast<int32_t *>(g.h_eids) + 16, pred, (size_t)n_pred * 4);
    if (!demand && !pref) return 0;
    cudaMemcpyAsync(g.d_eids, g.h_eids, (size_t)(16 + (pref ? n_pred : 0)) * 4, cudaMemcpyHostToDevice, g.st);
    if (demand && moe_lru_step_ex(L->state, L->E, L->cap, g.d_eids, k, out, g.d_list, g.d_acct, 1, g.st) != 0)
        return 0;
    if (pref && moe_lru_prefetch_ex(Ln->state, Ln->E, Ln->cap, reinterpret_cast<const int32_t *>(g.d_eids) + 16,
                                    n_pred, mf, g.d_list + kPrefList, g.d_acct, 1, g.st) != 0)
        return 0;
    if (demand) {
        cudaMemcpyAsync(g.h_list, g.d_list, (size_t)(1 + 3 * k) * 4, cudaMemcpyDeviceToHost, g.st);
        if (out != L->slot_inds || (flags & kFlagSplit))
            cudaMemcpyAsync(g.h_slots, out, (size_t)k * 4, cudaMemcpyDeviceToHost, g.st);
    }
    if (pref)
        cudaMemcpyAsync(g.h_list + kPrefList, g.d_list + kPrefList, (size_t)(1 + 2 * mf) * 4, cudaMemcpyDeviceToHost,
                        g.st);
    if (!ok(cudaStreamSynchronize(g.st))) return 0;
    int n_missing = 0;
    if (demand) {
        n_missing = g.h_list[0];
        if (n_missing < 0) return 0;
        if (L->slot_inds && !L->slots_on_device) std::memcpy(L->slot_inds, g.h_slots, (size_t)k * 4);
        if ((flags & kFlagSplit) && n_missing > 0 && n_missing < k) {   // expert_io.c:1256-1275
            const int32_t *hit = g.h_list + 1 + 2 * k;
            SplitRecord &r = g.split[layer_idx];
            int nh = 0, nm = 0;
            const int n_hit = k - n_missing;
            for (int i = 0; i < k; ++i) {
                if (hit[i]) {
                    r.hit_slots[nh] = g.h_slots[i];
                    r.inv[i] = nh++;
                } else {
                    r.miss_slots[nm] = g.h_slots[i];
                    r.inv[i] = n_hit + nm++;
                }
            }
            r.hit = n_hit;
            r.miss = n_missing;
            r.k = k;
        }
        issue_fills(L, g.h_list, k, true);
    }
    if (pref) issue_fills(Ln, g.h_list + kPrefList, mf, true);
    if ((flags & kFlagSyncDemand) || n_missing == 0) wait_fills();
    return n_missing;
}

}  // extern "C"
