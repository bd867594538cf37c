// Per-layer LRU expert-slot cache with its state in device memory.
//
// Semantics are those of the reference's host-side cache (mlx-qwen38/expert_io.c): a doubly
// linked list over slots (head = least recently used), eid -> slot and slot -> eid tables, a
// free stack that pops slots 0, 1, 2, ... after a reset, eviction that walks from the head
// skipping protected experts (falling back to the head), demand steps that count LRU hits,
// prefetch hits and demand misses against a residency snapshot taken by the last prefetch,
// and prefetches that take the first <= max_fetch missing predictions in rank order and
// insert them in reverse rank order. Every operation is inherently sequential (each
// allocation depends on the list state the previous one left), so one thread runs it on a
// shared-memory copy of the layer's state: one launch per call, no host round trip, the
// router's indices read where the router wrote them.
//
// Device state of one layer (moe_lru_state_bytes): a header, then int16 tables and u64
// bitmaps sized by E and cap, then 18 u64 counters in the order of c_layer_get_stats
// (expert_io.c:791-812), then each expert's last eviction token (the newer reference's
// per-token I/O accounting, cpp/third_party/expert_io.c:91-112, 504-520).
//
// Per-token accounting (optional, off unless an LruAcct is passed): the decode token in
// progress and nine counters -- LRU hits, demand misses, prefetch loads, prefetch hits,
// wasted prefetches, demand and prefetch re-reads of experts evicted at most 16 / 64 tokens
// earlier -- shared by every layer of a process, as the reference keeps them.
#include <algorithm>

#include "common.cuh"

namespace {

constexpr int kLruMaxE = 2048;
constexpr int kLruMaxK = 32;        // experts per demand step
constexpr int kLruMaxPred = 64;     // predictions per prefetch call
constexpr int kLruThreads = 128;

struct LruHeader {
    int32_t E, cap, head, tail, free_count, has_snap, pad0, pad1;
    uint64_t expert_bytes;
};

struct LruLayout {
    size_t e2s, s2e, prev, next, freel, pre, pred, fet, stats, last_ev, total;
    MOE_HD LruLayout(int E, int cap) {
        const size_t nb = (size_t)(E + 63) / 64;
        e2s = sizeof(LruHeader);
        s2e = al16(e2s + (size_t)E * 2);
        prev = al16(s2e + (size_t)cap * 2);
        next = al16(prev + (size_t)cap * 2);
        freel = al16(next + (size_t)cap * 2);
        pre = al16(freel + (size_t)cap * 2);
        pred = pre + nb * 8;
        fet = pred + nb * 8;
        stats = fet + nb * 8;
        last_ev = al16(stats + 18 * 8);
        total = al16(last_ev + (size_t)E * 4);
    }
};

// the per-token accounting shared by every layer (moe_lru_acct_bytes)
enum AcctCounter {
    kTokLruHits = 0, kTokDemandMisses, kTokPrefLoads, kTokPrefHits, kTokWasted, kTokDemRe16, kTokDemRe64,
    kTokPrefRe16, kTokPrefRe64, kTokCounters
};
struct LruAcct {
    int32_t enabled, cur_token, pad0, pad1;   // cur_token < 0: no token in progress
    uint64_t c[kTokCounters];
};

enum Stat {
    kDecReq = 0, kDecLruHits, kDecPrefHits, kDecMiss, kDecMissBytes, kDecPrefBytes,
    kPreReq, kPreHits, kPreMiss, kPreMissBytes, kPredHits, kPredActual, kPredTotal,
    kMissPrefHits, kMissPrefActualMisses, kMissPrefFetched, kUncoalesced, kCoalesced
};

// Shared-memory view of one layer's state; loaded and stored by the whole block, operated
// on by thread 0.
struct Lru {
    LruHeader *h;
    int16_t *e2s, *s2e, *prev, *next, *freel;
    uint64_t *pre, *pred, *fet, *stats;
    int32_t *last_ev;
    LruAcct *acct;                       // null or accounting off: nothing recorded
    int nb;

    MOE_D bool accounting() const { return acct && acct->enabled && acct->cur_token >= 0; }
    MOE_D void evicted(int eid) {
        if (accounting()) last_ev[eid] = acct->cur_token;
    }
    // an expert read again: count it against the token it was evicted at
    MOE_D void reread(int eid, int c16, int c64) {
        if (!accounting()) return;
        const int ev = last_ev[eid];
        if (ev >= 0 && acct->cur_token >= ev) {
            const int dist = acct->cur_token - ev;
            if (dist <= 16) ++acct->c[c16];
            if (dist <= 64) ++acct->c[c64];
        }
        last_ev[eid] = -1;
    }

    MOE_D void bind(unsigned char *base, int E, int cap) {
        const LruLayout Ly(E, cap);
        h = reinterpret_cast<LruHeader *>(base);
        e2s = reinterpret_cast<int16_t *>(base + Ly.e2s);
        s2e = reinterpret_cast<int16_t *>(base + Ly.s2e);
        prev = reinterpret_cast<int16_t *>(base + Ly.prev);
        next = reinterpret_cast<int16_t *>(base + Ly.next);
        freel = reinterpret_cast<int16_t *>(base + Ly.freel);
        pre = reinterpret_cast<uint64_t *>(base + Ly.pre);
        pred = reinterpret_cast<uint64_t *>(base + Ly.pred);
        fet = reinterpret_cast<uint64_t *>(base + Ly.fet);
        stats = reinterpret_cast<uint64_t *>(base + Ly.stats);
        last_ev = reinterpret_cast<int32_t *>(base + Ly.last_ev);
        acct = nullptr;
        nb = (E + 63) / 64;
    }

    MOE_D void remove(int s) {
        const int p = prev[s], n = next[s];
        if (p >= 0) next[p] = (int16_t)n; else h->head = n;
        if (n >= 0) prev[n] = (int16_t)p; else h->tail = p;
        prev[s] = -1;
        next[s] = -1;
    }
    MOE_D void append_mru(int s) {
        prev[s] = (int16_t)h->tail;
        next[s] = -1;
        if (h->tail >= 0) next[h->tail] = (int16_t)s; else h->head = s;
        h->tail = s;
    }
    MOE_D void move_to_mru(int s) {
        if (h->tail == s) return;
        remove(s);
        append_mru(s);
    }
    MOE_D void insert(int eid, int s) {
        if (e2s[eid] >= 0) {
            move_to_mru(e2s[eid]);
            return;
        }
        e2s[eid] = (int16_t)s;
        s2e[s] = (int16_t)eid;
        append_mru(s);
    }
    MOE_D static bool has(const uint64_t *bm, int e) { return (bm[e >> 6] >> (e & 63)) & 1ull; }
    // keep: experts that must stay resident even when every resident expert is protected (the
    // scheduled step's own experts, which also protects prefetched ones; with k + fetched > cap
    // the reference's oldest-goes fallback can evict one of the step's experts and then indexes
    // its tables with -1 -- here the oldest expert outside `keep` goes instead)
    MOE_D int alloc(const uint64_t *prot, const uint64_t *keep = nullptr) {
        if (h->free_count > 0) return freel[--h->free_count];
        for (int cur = h->head; cur >= 0; cur = next[cur]) {
            const int eid = s2e[cur];
            if (eid >= 0 && !has(prot, eid)) {
                remove(cur);
                e2s[eid] = -1;
                s2e[cur] = -1;
                evicted(eid);
                return cur;
            }
        }
        int victim = h->head;                   // every resident expert is protected: the oldest goes
        if (keep)
            for (int cur = h->head; cur >= 0; cur = next[cur])
                if (s2e[cur] < 0 || !has(keep, s2e[cur])) {
                    victim = cur;
                    break;
                }
        const int eid = s2e[victim];
        remove(victim);
        if (eid >= 0) {
            e2s[eid] = -1;
            evicted(eid);
        }
        s2e[victim] = -1;
        return victim;
    }
    MOE_D void reset_tables() {
        for (int i = 0; i < h->E; ++i) e2s[i] = -1;
        for (int i = 0; i < h->cap; ++i) s2e[i] = prev[i] = next[i] = -1;
        h->head = h->tail = -1;
        h->has_snap = 0;
    }
};

// The reference's I/O accounting of one fill of n experts (expert_io.c:186-233): nine tensor
// reads per expert, and nine reads per run of consecutive expert ids once sorted (its
// coalesced preadv calls). Counted the same way here so the counters stay comparable.
constexpr int kRefTensors = 9;
MOE_D void count_fill(uint64_t *stats, const int *eids, int n) {
    if (n <= 0) return;
    int s[32];
    for (int i = 0; i < n; ++i) {
        int j = i - 1;
        while (j >= 0 && s[j] > eids[i]) {
            s[j + 1] = s[j];
            --j;
        }
        s[j + 1] = eids[i];
    }
    int runs = 1;
    for (int i = 1; i < n; ++i) runs += (s[i] != s[i - 1] + 1) ? 1 : 0;
    stats[kUncoalesced] += (uint64_t)n * kRefTensors;
    stats[kCoalesced] += (uint64_t)runs * kRefTensors;
}

// whole-block copy of the state between global and shared memory (16-byte multiples)
MOE_D void copy16(void *dst, const void *src, size_t bytes) {
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    for (size_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
}

enum Op {
    kOpReset = 0, kOpResetStats, kOpStep, kOpPrefetch, kOpGetState, kOpSetState, kOpStats, kOpAddStat,
    kOpStepSched, kOpPrefetchSched
};

struct LruArgs {
    unsigned char *state;
    int E, cap, op;
    const uint32_t *eids;      // step: [k] (device)   prefetch: [n] predictions   set: [n] ordered eids
    const int32_t *slots_in;   // set: [n] ordered slots
    int n;                     // k / prediction count / set count (when count_dev is null)
    const int32_t *count_dev;  // set: count on the device (optional)
    int max_fetch;
    uint32_t *out_slots;       // step: [k] slot per expert
    int32_t *out_list;         // step: [1 + 2*k] {n_miss, eids.., slots..}; prefetch: [1 + 2*max] fetched
                               // get: [1 + 2*cap] {count, eids (LRU->MRU).., slots..}
    uint64_t *out_stats;       // stats: [18]
    uint64_t add_req, add_hits, add_misses;
    LruAcct *acct;             // per-token accounting shared by all layers, or null
};

__global__ void __launch_bounds__(kLruThreads) lru_kernel(LruArgs a) {
    extern __shared__ __align__(16) unsigned char sm[];
    const LruLayout Ly(a.E, a.cap);
    copy16(sm, a.state, Ly.total);
    __syncthreads();
    Lru L;
    L.bind(sm, a.E, a.cap);
    L.acct = a.acct;
    if (a.op == kOpPrefetch || a.op == kOpPrefetchSched) {
        // the residency snapshot of expert_io.c:536-541 by every warp at once: 32 experts per
        // ballot, one 32-bit half of a bitmap word per warp step (words past E come out zero)
        const int lane = threadIdx.x & 31;
        uint32_t *pre32 = reinterpret_cast<uint32_t *>(L.pre);
#pragma unroll 1
        for (int base = threadIdx.x - lane; base < L.nb * 64; base += blockDim.x) {
            const int e = base + lane;
            const unsigned bal = __ballot_sync(0xffffffffu, e < a.E && L.e2s[e] >= 0);
            if (lane == 0) pre32[base >> 5] = bal;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        LruHeader *h = L.h;
        const int E = a.E;
        switch (a.op) {
            case kOpReset: {     // expert_io.c:450-468 (+ cpp/third_party/expert_io.c:560)
                L.reset_tables();
                h->free_count = h->cap;
                for (int i = 0; i < h->cap; ++i) L.freel[i] = (int16_t)(h->cap - 1 - i);
                for (int i = 0; i < E; ++i) L.last_ev[i] = -1;
                break;
            }
            case kOpResetStats: {   // expert_io.c:470-495
                for (int i = 0; i < 18; ++i) L.stats[i] = 0;
                break;
            }
            case kOpStep:        // expert_io.c:583-676 (+ accounting, cpp/third_party/expert_io.c:745-806)
            case kOpStepSched: { // cpp/third_party/expert_io.c:1129-1270 (the step half of decode_step_sched)
                const bool sched = a.op == kOpStepSched;
                const int k = a.n;
                L.stats[kDecReq] += (uint64_t)k;
                uint64_t act[kLruMaxE / 64], prot[kLruMaxE / 64];
                for (int b = 0; b < L.nb; ++b) act[b] = 0;
                bool bad = false;
                for (int i = 0; i < k; ++i) {
                    const uint32_t e = a.eids[i];
                    if (e >= (uint32_t)E) { bad = true; continue; }
                    act[e >> 6] |= 1ull << (e & 63);
                }
                if (bad) {
                    atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
                    a.out_list[0] = -1;
                    break;
                }
                // the scheduled step also protects the experts the last prefetch is bringing in
                for (int b = 0; b < L.nb; ++b) prot[b] = act[b] | ((sched && h->has_snap) ? L.fet[b] : 0ull);
                const bool acc = a.acct && a.acct->enabled;
                int miss_e[kLruMaxK], miss_s[kLruMaxK], nm = 0;
                uint8_t hit[kLruMaxK];
                uint64_t tok_lru = 0, tok_pref = 0;
                if (h->has_snap) {
                    uint64_t ov = 0, ta = 0, tp = 0, mh = 0, tam = 0, tf = 0;
                    for (int b = 0; b < L.nb; ++b) {
                        const uint64_t am = act[b] & ~L.pre[b];
                        ov += __popcll(act[b] & L.pred[b]);
                        ta += __popcll(act[b]);
                        tp += __popcll(L.pred[b]);
                        mh += __popcll(am & L.fet[b]);
                        tam += __popcll(am);
                        tf += __popcll(L.fet[b]);
                    }
                    L.stats[kPredHits] += ov;
                    L.stats[kPredActual] += ta;
                    L.stats[kPredTotal] += tp;
                    L.stats[kMissPrefHits] += mh;
                    L.stats[kMissPrefActualMisses] += tam;
                    L.stats[kMissPrefFetched] += tf;
                    for (int i = 0; i < k; ++i) {
                        const int e = (int)a.eids[i];
                        hit[i] = L.e2s[e] >= 0;
                        if (hit[i]) {
                            if (Lru::has(L.pre, e)) { ++L.stats[kDecLruHits]; ++tok_lru; }
                            else { ++L.stats[kDecPrefHits]; ++tok_pref; }
                        } else {
                            ++L.stats[kDecMiss];
                            miss_e[nm++] = e;
                        }
                    }
                    if (acc) {
                        a.acct->c[kTokLruHits] += tok_lru;
                        a.acct->c[kTokPrefHits] += tok_pref;
                        if (tf >= tok_pref) a.acct->c[kTokWasted] += tf - tok_pref;
                        a.acct->c[kTokDemandMisses] += (uint64_t)nm;
                    }
                    h->has_snap = 0;
                } else {
                    for (int i = 0; i < k; ++i) {
                        const int e = (int)a.eids[i];
                        hit[i] = L.e2s[e] >= 0;
                        if (hit[i]) {
                            ++L.stats[kDecLruHits];
                            ++tok_lru;
                        } else {
                            ++L.stats[kDecMiss];
                            miss_e[nm++] = e;
                        }
                    }
                    if (acc) {
                        a.acct->c[kTokLruHits] += tok_lru;
                        a.acct->c[kTokDemandMisses] += (uint64_t)nm;
                    }
                }
                for (int i = 0; i < nm; ++i) {
                    const int s = L.alloc(prot, sched ? act : nullptr);
                    L.reread(miss_e[i], kTokDemRe16, kTokDemRe64);
                    L.insert(miss_e[i], s);
                    miss_s[i] = s;
                }
                L.stats[kDecMissBytes] += (uint64_t)nm * h->expert_bytes;
                count_fill(L.stats, miss_e, nm);
                for (int i = 0; i < k; ++i) {
                    const int s = L.e2s[a.eids[i]];
                    L.move_to_mru(s);
                    a.out_slots[i] = (uint32_t)s;
                }
                a.out_list[0] = nm;
                for (int i = 0; i < nm; ++i) {
                    a.out_list[1 + i] = miss_e[i];
                    a.out_list[1 + k + i] = miss_s[i];
                }
                if (sched)
                    for (int i = 0; i < k; ++i) a.out_list[1 + 2 * k + i] = hit[i];
                break;
            }
            case kOpPrefetch:    // expert_io.c:527-581 (L.pre: the snapshot taken above; + accounting)
            case kOpPrefetchSched: {   // cpp/third_party/expert_io.c:1290-1340: duplicates counted once
                const bool sched = a.op == kOpPrefetchSched;
                for (int b = 0; b < L.nb; ++b) {
                    L.pred[b] = 0;
                    L.fet[b] = 0;
                }
                h->has_snap = 1;
                uint64_t prot[kLruMaxE / 64];
                for (int b = 0; b < L.nb; ++b) prot[b] = 0;
                const int cap_fetch = (a.max_fetch > 0 && a.max_fetch < 32) ? a.max_fetch : 32;
                int miss[32], nm = 0;
                for (int i = 0; i < a.n; ++i) {
                    const int32_t e = (int32_t)a.eids[i];
                    if (e < 0 || e >= E) continue;
                    L.pred[e >> 6] |= 1ull << (e & 63);
                    prot[e >> 6] |= 1ull << (e & 63);
                    if (L.e2s[e] < 0 && nm < cap_fetch && !(sched && Lru::has(L.fet, e))) {
                        miss[nm++] = e;
                        L.fet[e >> 6] |= 1ull << (e & 63);
                    }
                }
                a.out_list[0] = nm;
                count_fill(L.stats, miss, nm);
                for (int i = 0; i < nm; ++i) {      // reverse rank order: the best prediction is newest
                    const int e = miss[nm - 1 - i];
                    const int s = L.alloc(prot);
                    L.reread(e, kTokPrefRe16, kTokPrefRe64);
                    L.insert(e, s);
                    a.out_list[1 + i] = e;
                    a.out_list[1 + a.max_fetch + i] = s;
                }
                if (a.acct && a.acct->enabled) a.acct->c[kTokPrefLoads] += (uint64_t)nm;
                L.stats[kDecPrefBytes] += (uint64_t)nm * h->expert_bytes;
                break;
            }
            case kOpGetState: {  // expert_io.c:726-747
                int cnt = 0;
                for (int cur = h->head; cur >= 0; cur = L.next[cur]) {
                    a.out_list[1 + cnt] = L.s2e[cur];
                    a.out_list[1 + a.cap + cnt] = cur;
                    ++cnt;
                }
                a.out_list[0] = cnt;
                break;
            }
            case kOpSetState: {  // expert_io.c:749-789
                const int cnt = a.count_dev ? *a.count_dev : a.n;
                L.stats[kPreReq] += a.add_req;
                L.stats[kPreHits] += a.add_hits;
                L.stats[kPreMiss] += a.add_misses;
                L.reset_tables();
                uint8_t used[kLruMaxE];
                for (int s = 0; s < h->cap; ++s) used[s] = 0;
                bool bad = cnt < 0 || cnt > h->cap;
                for (int i = 0; i < cnt && !bad; ++i) {
                    const int e = (int)a.eids[i], s = a.slots_in[i];
                    if (e < 0 || e >= E || s < 0 || s >= h->cap) { bad = true; break; }
                    used[s] = 1;
                    L.insert(e, s);
                    L.last_ev[e] = -1;
                }
                if (bad) atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
                h->free_count = 0;
                for (int s = h->cap - 1; s >= 0; --s)
                    if (!used[s]) L.freel[h->free_count++] = (int16_t)s;
                break;
            }
            case kOpStats: {
                for (int i = 0; i < 18; ++i) a.out_stats[i] = L.stats[i];
                break;
            }
            case kOpAddStat: {   // counter a.n += a.add_req (prefill accounting of c_layer_load_sync)
                if (a.n >= 0 && a.n < 18) L.stats[a.n] += a.add_req;
                break;
            }
        }
    }
    __syncthreads();
    if (a.op != kOpGetState && a.op != kOpStats) copy16(a.state, sm, Ly.total);
}

int lru_launch(LruArgs a, void *stream) {
    if (!a.state) return moe_set_error(MOE_EINVAL, "lru: null state");
    const LruLayout Ly(a.E, a.cap);
    // raise the dynamic shared-memory limit once (not per launch: launches may be captured)
    static int configured = 0;
    if (Ly.total > 48 * 1024 && !configured) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(lru_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)LruLayout(kLruMaxE, kLruMaxE).total));
        configured = 1;
    }
    lru_kernel<<<1, kLruThreads, Ly.total, as_stream(stream)>>>(a);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

int check_dims(int E, int cap) {
    if (E <= 0 || E > kLruMaxE || cap <= 0 || cap > E || cap > 32767)
        return moe_set_error(MOE_EINVAL, "lru: bad sizes E=%d cap=%d", E, cap);
    return MOE_OK;
}

// host-side header written by moe_lru_init
__global__ void lru_header_kernel(unsigned char *state, int E, int cap, uint64_t expert_bytes) {
    LruHeader *h = reinterpret_cast<LruHeader *>(state);
    h->E = E;
    h->cap = cap;
    h->expert_bytes = expert_bytes;
}

}  // namespace

extern "C" size_t moe_lru_state_bytes(int E, int cap) {
    if (E <= 0 || E > kLruMaxE || cap <= 0 || cap > E) return 0;
    return LruLayout(E, cap).total;
}

extern "C" int moe_lru_init(void *state, int E, int cap, uint64_t expert_bytes, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    if (!state || reinterpret_cast<uintptr_t>(state) % 16)
        return moe_set_error(MOE_EINVAL, "lru_init: state must be a 16-byte aligned device pointer");
    MOE_CUDA_TRY(cudaMemsetAsync(state, 0, LruLayout(E, cap).total, as_stream(stream)));
    lru_header_kernel<<<1, 1, 0, as_stream(stream)>>>(static_cast<unsigned char *>(state), E, cap, expert_bytes);
    MOE_CUDA_TRY(cudaGetLastError());
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = kOpReset;
    return lru_launch(a, stream);
}

extern "C" int moe_lru_reset(void *state, int E, int cap, int what, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = what == 1 ? kOpResetStats : kOpReset;
    return lru_launch(a, stream);
}

extern "C" size_t moe_lru_acct_bytes(void) { return sizeof(LruAcct); }

extern "C" int moe_lru_step_ex(void *state, int E, int cap, const uint32_t *eids, int k, uint32_t *out_slots,
                               int32_t *out_miss, void *acct, int sched, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    if (k <= 0 || k > kLruMaxK || k > cap || !eids || !out_slots || !out_miss)
        return moe_set_error(MOE_EINVAL, "lru_step: bad arguments (k=%d cap=%d)", k, cap);
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = sched ? kOpStepSched : kOpStep;
    a.eids = eids;
    a.n = k;
    a.out_slots = out_slots;
    a.out_list = out_miss;
    a.acct = static_cast<LruAcct *>(acct);
    return lru_launch(a, stream);
}

extern "C" int moe_lru_step(void *state, int E, int cap, const uint32_t *eids, int k, uint32_t *out_slots,
                            int32_t *out_miss, void *stream) {
    return moe_lru_step_ex(state, E, cap, eids, k, out_slots, out_miss, nullptr, 0, stream);
}

extern "C" int moe_lru_prefetch_ex(void *state, int E, int cap, const int32_t *pred, int n, int max_fetch,
                                   int32_t *out_fetch, void *acct, int sched, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    if (n < 0 || n > kLruMaxPred || (n > 0 && !pred) || !out_fetch || max_fetch <= 0 || max_fetch > 32)
        return moe_set_error(MOE_EINVAL, "lru_prefetch: bad arguments (n=%d max_fetch=%d)", n, max_fetch);
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = sched ? kOpPrefetchSched : kOpPrefetch;
    a.eids = reinterpret_cast<const uint32_t *>(pred);
    a.n = n;
    a.max_fetch = max_fetch;
    a.out_list = out_fetch;
    a.acct = static_cast<LruAcct *>(acct);
    return lru_launch(a, stream);
}

extern "C" int moe_lru_prefetch(void *state, int E, int cap, const int32_t *pred, int n, int max_fetch,
                                int32_t *out_fetch, void *stream) {
    return moe_lru_prefetch_ex(state, E, cap, pred, n, max_fetch, out_fetch, nullptr, 0, stream);
}

extern "C" int moe_lru_get_state(void *state, int E, int cap, int32_t *out, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    if (!out) return moe_set_error(MOE_EINVAL, "lru_get_state: null output");
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = kOpGetState;
    a.out_list = out;
    return lru_launch(a, stream);
}

extern "C" int moe_lru_set_state(void *state, int E, int cap, const int32_t *eids, const int32_t *slots, int n,
                                 uint64_t add_req, uint64_t add_hits, uint64_t add_misses, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    if (n < 0 || n > cap || (n > 0 && (!eids || !slots)))
        return moe_set_error(MOE_EINVAL, "lru_set_state: bad arguments (n=%d cap=%d)", n, cap);
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = kOpSetState;
    a.eids = reinterpret_cast<const uint32_t *>(eids);
    a.slots_in = slots;
    a.n = n;
    a.add_req = add_req;
    a.add_hits = add_hits;
    a.add_misses = add_misses;
    return lru_launch(a, stream);
}

extern "C" int moe_lru_get_stats(void *state, int E, int cap, uint64_t *out18, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    if (!out18) return moe_set_error(MOE_EINVAL, "lru_get_stats: null output");
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = kOpStats;
    a.out_stats = out18;
    return lru_launch(a, stream);
}

extern "C" int moe_lru_add_stat(void *state, int E, int cap, int index, uint64_t value, void *stream) {
    if (int rc = check_dims(E, cap)) return rc;
    if (index < 0 || index >= 18) return moe_set_error(MOE_EINVAL, "lru_add_stat: counter %d", index);
    LruArgs a{};
    a.state = static_cast<unsigned char *>(state);
    a.E = E;
    a.cap = cap;
    a.op = kOpAddStat;
    a.n = index;
    a.add_req = value;
    return lru_launch(a, stream);
}
