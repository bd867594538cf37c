// P1 I/O scheduler with its state in GPU memory.
//
// The reference's qwen38::P1IoScheduler (mlx-qwen38/cpp/src/io_sched.h:46-245, behaviour of
// cpp/src/io_sched.cpp, tested by cpp/tests/test_io_sched.cpp:142-445) keeps per-layer LRU
// slot caches and two read queues (URGENT served before PREFETCH) behind one mutex, drained by
// host worker threads and by callers that wait. Here the whole scheduler -- every layer's LRU
// lists, pin counts and in-flight reads, an op pool, the two task queues -- is one struct in
// device memory, and every method is one launch of a single-warp control kernel that applies
// the call to that state, so the decisions are made where the slots live and the host only
// moves arguments and results. Reads that the control kernel takes from a queue are appended
// to an execute list; a multi-CTA copy kernel then moves those rows from the pinned host pool
// (or device memory) into the slot buffers in list order (the last write to a row wins), and
// rows from a file (the reference's own form) are read by the host from the same list.
//
// Queue model (observable behaviour, identical to the reference's): a read op covers one
// expert into one slot and is split into one task per tensor (prefetch) or, for urgent reads,
// one task per (tensor, run of <= 16 consecutive expert ids); weights (rows above 100,000
// bytes) are queued before scales and biases. An op has started once any of its tasks has
// been taken and is done once all have; a prefetch that has not started can be cancelled
// (its slot handed back to the expert it displaced) or promoted to the urgent queue, one that
// has started can only be used or wasted. Without workers nothing is taken until a caller
// waits (deterministic, used by the differential tests); with workers (init(n), n >= 1) the
// copy engine takes every queued task at the end of each call, one valid schedule of the
// reference's threads. A slot allocation that finds only slots pinned by a GPU reader stops
// the kernel with a continuation record; the host calls the reader-wait callback (which
// unpins) and resumes the call where it stopped.
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <random>
#include <vector>

#include "common.cuh"

namespace {

constexpr int kLayers = 64, kExperts = 512, kTensors = 9;
constexpr int kRun = 16;                    // ops per coalesced urgent task
constexpr uint32_t kOpPool = 1u << 18;      // op records (id -> id % kOpPool)
constexpr int kRing = 1 << 14;              // tasks per queue
constexpr int kExecMax = 1 << 15;           // rows taken by one call
constexpr int kPinList = 1 << 13;           // pins held by step_decode per layer until unpinned
constexpr int kMaxK = 64;                   // experts per step_decode
constexpr int kMaxPred = 32;                // predictions considered per start_prefetch (the cap)
constexpr int kMaxPredIn = 512;             // predictions passed per start_prefetch
constexpr uint64_t kLargeRow = 100000;      // rows above this size are queued first
constexpr uint64_t kDefaultExpertBytes = 1536000;

// per-layer counters (qwen38::P1LayerStats order)
enum Stat {
    kReq, kHits, kUrgent, kIssued, kCancelled, kPromoted, kUsed, kWasted, kPinWaits, kBytes, kIoWait,
    kForced, kPfReq, kPfHits, kPfMiss, kPfBytes, kNumStats
};
static_assert(kNumStats == MOE_P1_STATS, "stat layout");

enum OpFlag : uint32_t { kOpPrefetch = 1, kOpPromoted = 2, kOpCancelled = 4, kOpResolved = 8 };

struct Op {
    int16_t eid, slot, prev_eid, layer;
    uint32_t flags;
    uint16_t ntasks, started, completed, pad;
};

struct Task {
    int16_t layer, tensor;
    uint16_t nops, flags;                   // flags: 1 prefill read (no decode bytes), 2 removed
    uint32_t op[kRun];
};

struct Ring {
    uint32_t head, tail;                    // monotonic; entry i at t[i % kRing]
    Task t[kRing];
};

struct LayerState {
    int32_t init, capacity, ntensors, pad0;
    uint64_t row_bytes[kTensors];
    uint64_t expert_bytes;
    int16_t e2s[kExperts], s2e[kExperts], prv[kExperts], nxt[kExperts], freel[kExperts];
    int16_t head, tail;
    int32_t nfree;
    int32_t pins[kExperts];
    uint32_t io[kExperts];                  // op id of the slot's last read (0: none)
    int32_t npinned;
    int16_t pinned[kPinList];
    int32_t has_snap;
    uint64_t snap[8];                       // residency before the last start_prefetch
    int32_t nlast;
    uint32_t last[kMaxPred];                // unresolved prefetch ops of the last start_prefetch
    int32_t npend;
    uint32_t pend[kMaxK];                   // reads the last step_decode / load_sync waits for
    uint64_t st[kNumStats];
};

struct Exec {
    int16_t layer, tensor, slot, kind;      // kind 0 copy row, 1 scrub the first 64 bytes
    int32_t eid;
};

// progress of a call stopped by a pinned-slot wait (resumed by the same command)
struct Cont {
    int32_t active, phase, idx, pin_counted;
    int32_t nmiss;
    int32_t miss[kMaxPred];
    uint64_t prot[8];
    int32_t nurg;
    uint32_t urg[kMaxK + kMaxPred];
};

struct State {
    LayerState L[kLayers];
    Ring urgent, prefetch;
    Op ops[kOpPool];
    uint32_t next_op;
    int32_t eager;
    int32_t nexec;
    Exec exec[kExecMax];
    Cont cont;
};

enum Cmd {
    kCmdInit = 1, kCmdResize, kCmdResetCache, kCmdResetStats, kCmdPrefetch, kCmdStep, kCmdWaitUrgent,
    kCmdWaitAll, kCmdUnpinLayer, kCmdPin, kCmdUnpin, kCmdPinCount, kCmdFiCount, kCmdForce, kCmdLoadSync,
    kCmdGetLru, kCmdSetLru, kCmdGetStats, kCmdGetTotal, kCmdSetEager
};

struct CmdArgs {
    int32_t cmd, layer, n, m, resume, flag;
    int32_t capacity, ntensors;
    double rate;
    uint64_t row_bytes[kTensors];
    uint64_t add[3];
    int32_t a[kMaxPredIn];                  // eids / predictions / slots
    int32_t b[kExperts];                    // second list (slots)
    double draws[kExperts];
};

enum Status { kOk = 0, kBlockedPin = 1, kErrQueue = -1, kErrStuck = -2, kErrExec = -3, kErrPins = -4 };

struct Result {
    int32_t status, ret, waited, nexec, count, pad;
    int32_t a[kExperts], b[kExperts];
    uint64_t st[kNumStats];
};

// ------------------------------------------------------------------ device helpers (thread 0)

__device__ __forceinline__ bool bit(const uint64_t *bm, int e) { return (bm[e >> 6] >> (e & 63)) & 1ull; }
__device__ __forceinline__ void setbit(uint64_t *bm, int e) { bm[e >> 6] |= 1ull << (e & 63); }

__device__ Op &op_of(State &S, uint32_t id) { return S.ops[id % kOpPool]; }

// an op id older than the pool is treated as done: its record has been reused
__device__ bool op_done(State &S, uint32_t id) {
    if (id == 0 || S.next_op - id >= kOpPool) return true;
    const Op &o = op_of(S, id);
    return o.completed >= o.ntasks;
}

__device__ bool slot_busy(State &S, LayerState &L, int s) { return L.io[s] != 0 && !op_done(S, L.io[s]); }

__device__ uint32_t new_op(State &S, int layer, int eid, int slot, int prev, uint32_t flags, int ntasks) {
    uint32_t id = ++S.next_op;
    if (id == 0) id = ++S.next_op;
    Op &o = op_of(S, id);
    o.eid = (int16_t)eid;
    o.slot = (int16_t)slot;
    o.prev_eid = (int16_t)prev;
    o.layer = (int16_t)layer;
    o.flags = flags;
    o.ntasks = (uint16_t)ntasks;
    o.started = 0;
    o.completed = 0;
    return id;
}

// LRU list: head = least recently used, tail = most recently used
__device__ void lru_unlink(LayerState &L, int s) {
    const int p = L.prv[s], n = L.nxt[s];
    if (p >= 0) L.nxt[p] = (int16_t)n;
    else L.head = (int16_t)n;
    if (n >= 0) L.prv[n] = (int16_t)p;
    else L.tail = (int16_t)p;
    L.prv[s] = L.nxt[s] = -1;
}

__device__ void lru_push_tail(LayerState &L, int s) {
    L.prv[s] = L.tail;
    L.nxt[s] = -1;
    if (L.tail >= 0) L.nxt[L.tail] = (int16_t)s;
    else L.head = (int16_t)s;
    L.tail = (int16_t)s;
}

__device__ void lru_push_head(LayerState &L, int e, int s) {
    L.e2s[e] = (int16_t)s;
    L.s2e[s] = (int16_t)e;
    L.prv[s] = -1;
    L.nxt[s] = L.head;
    if (L.head >= 0) L.prv[L.head] = (int16_t)s;
    else L.tail = (int16_t)s;
    L.head = (int16_t)s;
}

__device__ void lru_touch(LayerState &L, int s) {
    if (L.tail == s) return;
    lru_unlink(L, s);
    lru_push_tail(L, s);
}

__device__ void lru_place(LayerState &L, int e, int s) {      // map e -> s at the MRU end
    if (L.e2s[e] >= 0) {
        lru_touch(L, L.e2s[e]);
        return;
    }
    L.e2s[e] = (int16_t)s;
    L.s2e[s] = (int16_t)e;
    lru_push_tail(L, s);
}

__device__ void forget_slot(LayerState &L, int s) {           // drop s's expert from the cache
    const int e = L.s2e[s];
    lru_unlink(L, s);
    if (e >= 0) L.e2s[e] = -1;
    L.s2e[s] = -1;
    L.io[s] = 0;
}

__device__ void free_push(LayerState &L, int s) {
    if (L.nfree < kExperts) L.freel[L.nfree++] = (int16_t)s;
}

__device__ void clear_lists(LayerState &L, bool pins) {
    for (int i = 0; i < kExperts; ++i) {
        L.e2s[i] = L.s2e[i] = L.prv[i] = L.nxt[i] = -1;
        L.io[i] = 0;
        if (pins) L.pins[i] = 0;
    }
    if (pins) L.npinned = 0;
    L.head = L.tail = -1;
    L.has_snap = 0;
    for (int w = 0; w < 8; ++w) L.snap[w] = 0;
    L.nlast = 0;
    L.npend = 0;
}

__device__ void fill_free_all(LayerState &L) {                // pops return 0, 1, 2, ...
    L.nfree = L.capacity;
    for (int i = 0; i < L.capacity; ++i) L.freel[i] = (int16_t)(L.capacity - 1 - i);
}

// rebuild from an LRU -> MRU ordered list; free slots = the unused ones, smallest popped first
__device__ void place_ordered(LayerState &L, const int32_t *eids, const int32_t *slots, int n) {
    uint8_t used[kExperts];
    for (int s = 0; s < kExperts; ++s) used[s] = 0;
    for (int i = 0; i < n; ++i) {
        const int e = eids[i], s = slots[i];
        if (s >= 0 && s < L.capacity && e >= 0 && e < kExperts) {
            used[s] = 1;
            lru_place(L, e, s);
        }
    }
    L.nfree = 0;
    for (int s = L.capacity - 1; s >= 0; --s)
        if (!used[s]) L.freel[L.nfree++] = (int16_t)s;
}

// ------------------------------------------------------------------ queues and the taking of tasks

__device__ bool ring_push(Ring &R, const Task &t) {
    if (R.tail - R.head >= (uint32_t)kRing) return false;
    R.t[R.tail % kRing] = t;
    ++R.tail;
    return true;
}

// the task is taken: its ops progress, its rows join the execute list, decode bytes are counted
__device__ bool run_task(State &S, const Task &t) {
    LayerState &L = S.L[t.layer];
    for (int k = 0; k < t.nops; ++k) {
        Op &o = op_of(S, t.op[k]);
        if (S.nexec >= kExecMax) return false;
        S.exec[S.nexec++] = Exec{t.layer, t.tensor, o.slot, 0, o.eid};
        ++o.completed;
    }
    if (!(t.flags & 1)) L.st[kBytes] += L.row_bytes[t.tensor] * (uint64_t)t.nops;
    return true;
}

// an urgent task is taken if any of its ops is still wanted
__device__ bool take_urgent(State &S, const Task &t, bool &ok) {
    bool valid = false;
    for (int k = 0; k < t.nops; ++k) {
        Op &o = op_of(S, t.op[k]);
        if (!(o.flags & kOpCancelled)) {
            ++o.started;
            valid = true;
        }
    }
    if (valid) ok = run_task(S, t);
    return valid;
}

// the next task by priority (URGENT, then PREFETCH), taken and run; false if none is left
__device__ bool take_next(State &S, bool &ok) {
    ok = true;
    while (S.urgent.head != S.urgent.tail) {
        const Task t = S.urgent.t[S.urgent.head % kRing];
        ++S.urgent.head;
        if (t.flags & 2) continue;
        if (take_urgent(S, t, ok)) return true;
    }
    while (S.prefetch.head != S.prefetch.tail) {
        const Task t = S.prefetch.t[S.prefetch.head % kRing];
        ++S.prefetch.head;
        if (t.flags & 2) continue;
        Op &o = op_of(S, t.op[0]);
        if (o.flags & (kOpCancelled | kOpPromoted)) continue;
        ++o.started;
        ok = run_task(S, t);
        return true;
    }
    return false;
}

__device__ bool queue_prefetch(State &S, int layer, uint32_t id) {
    LayerState &L = S.L[layer];
    for (int pass = 0; pass < 2; ++pass)
        for (int t = 0; t < L.ntensors; ++t) {
            if ((L.row_bytes[t] > kLargeRow) != (pass == 0)) continue;
            Task tk{};
            tk.layer = (int16_t)layer;
            tk.tensor = (int16_t)t;
            tk.nops = 1;
            tk.op[0] = id;
            if (!ring_push(S.prefetch, tk)) return false;
        }
    return true;
}

// urgent reads of `ops` (distinct experts): sorted by expert, split into runs of consecutive
// ids (<= kRun), one task per (tensor, run), large tensors first
__device__ bool queue_urgent(State &S, int layer, uint32_t *ops, int n, bool prefill) {
    if (n <= 0) return true;
    for (int i = 1; i < n; ++i) {                  // insertion sort by expert id
        const uint32_t v = ops[i];
        const int e = op_of(S, v).eid;
        int j = i - 1;
        while (j >= 0 && op_of(S, ops[j]).eid > e) {
            ops[j + 1] = ops[j];
            --j;
        }
        ops[j + 1] = v;
    }
    LayerState &L = S.L[layer];
    for (int pass = 0; pass < 2; ++pass)
        for (int t = 0; t < L.ntensors; ++t) {
            if ((L.row_bytes[t] > kLargeRow) != (pass == 0)) continue;
            int i = 0;
            while (i < n) {
                Task tk{};
                tk.layer = (int16_t)layer;
                tk.tensor = (int16_t)t;
                tk.flags = prefill ? 1 : 0;
                tk.op[0] = ops[i];
                tk.nops = 1;
                ++i;
                while (i < n && tk.nops < kRun && op_of(S, ops[i]).eid == op_of(S, ops[i - 1]).eid + 1)
                    tk.op[tk.nops++] = ops[i++];
                if (!ring_push(S.urgent, tk)) return false;
            }
        }
    return true;
}

// slot for a new read, evicting the least recently used unprotected, unpinned, idle slot
// (reference alloc_slot_locked): -1 with *status = kBlockedPin when only pinned slots block
__device__ int grab_slot(State &S, int layer, const uint64_t *prot, int *prev, int *status) {
    LayerState &L = S.L[layer];
    if (L.nfree > 0) {
        *prev = -1;
        return L.freel[--L.nfree];
    }
    for (int guard = 0; guard < (1 << 20); ++guard) {
        bool pin_seen = false, io_seen = false;
        for (int s = L.head, g = 0; s >= 0 && g <= kExperts; s = L.nxt[s], ++g) {
            const int e = L.s2e[s];
            const bool p = e >= 0 && bit(prot, e);
            const bool pinned = L.pins[s] > 0, busy = slot_busy(S, L, s);
            if (!p && !pinned && !busy) {
                *prev = e;
                forget_slot(L, s);
                return s;
            }
            pin_seen |= !p && pinned;
            io_seen |= !p && busy;
        }
        if (!pin_seen && !io_seen)
            for (int s = L.head, g = 0; s >= 0 && g <= kExperts; s = L.nxt[s], ++g) {
                pin_seen |= L.pins[s] > 0;
                io_seen |= slot_busy(S, L, s);
            }
        if (pin_seen) {
            if (!S.cont.pin_counted) {
                ++L.st[kPinWaits];
                S.cont.pin_counted = 1;
            }
            *status = kBlockedPin;
            return -1;
        }
        if (io_seen) {
            bool ok = true;
            if (!take_next(S, ok) || !ok) {
                *status = ok ? kErrStuck : kErrExec;
                return -1;
            }
            continue;
        }
        for (int s = L.head, g = 0; s >= 0 && g <= kExperts; s = L.nxt[s], ++g) {       // every slot was protected
            if (L.pins[s] == 0 && !slot_busy(S, L, s)) {
                *prev = L.s2e[s];
                forget_slot(L, s);
                return s;
            }
        }
    }
    *status = kErrStuck;
    return -1;
}

// an unstarted prefetch that is not wanted: cancelled, its slot back to the expert it
// displaced (at the LRU end) or to the free list
__device__ void cancel_prefetch(State &S, LayerState &L, Op &o, bool mark_snapshot) {
    o.flags |= kOpCancelled;
    ++L.st[kCancelled];
    if (L.s2e[o.slot] != o.eid) return;
    lru_unlink(L, o.slot);
    L.e2s[o.eid] = -1;
    L.s2e[o.slot] = -1;
    L.io[o.slot] = 0;
    if (o.prev_eid >= 0 && o.prev_eid < kExperts && L.e2s[o.prev_eid] < 0) {
        lru_push_head(L, o.prev_eid, o.slot);
        if (mark_snapshot) setbit(L.snap, o.prev_eid);
    } else {
        free_push(L, o.slot);
    }
}

// waits (by taking urgent tasks) until every read the last step / load needs is done
__device__ int wait_urgent(State &S, int layer, int *waited) {
    LayerState &L = S.L[layer];
    *waited = 0;
    if (L.npend == 0) return kOk;
    bool pending = false;
    for (int i = 0; i < L.npend; ++i) pending |= !op_done(S, L.pend[i]);
    if (!pending) {
        L.npend = 0;
        return kOk;
    }
    *waited = 1;
    for (;;) {
        bool all = true;
        for (int i = 0; i < L.npend; ++i) all &= op_done(S, L.pend[i]);
        if (all) break;
        bool taken = false, ok = true;
        while (S.urgent.head != S.urgent.tail && !taken) {
            const Task t = S.urgent.t[S.urgent.head % kRing];
            ++S.urgent.head;
            if (t.flags & 2) continue;
            taken = take_urgent(S, t, ok);
            if (!taken) return kErrStuck;             // the reference would wait for a worker here
        }
        if (!ok) return kErrExec;
        if (!taken) return kErrStuck;
    }
    L.npend = 0;
    return kOk;
}

__device__ int wait_all(State &S, int layer, int *waited) {
    int rc = wait_urgent(S, layer, waited);
    if (rc) return rc;
    LayerState &L = S.L[layer];
    if (!L.init) return kOk;
    for (;;) {
        bool all = true;
        for (int s = 0; s < L.capacity && all; ++s)
            if (L.io[s] && !op_done(S, L.io[s]) && !(op_of(S, L.io[s]).flags & kOpCancelled)) all = false;
        if (all) return kOk;
        bool ok = true;
        if (!take_next(S, ok)) return kErrStuck;
        if (!ok) return kErrExec;
    }
}

__device__ int drain_if_eager(State &S) {
    if (!S.eager) return kOk;
    bool ok = true;
    while (take_next(S, ok))
        if (!ok) return kErrExec;
    return kOk;
}

// ------------------------------------------------------------------ the calls

__device__ int do_prefetch(State &S, const CmdArgs &c) {
    LayerState &L = S.L[c.layer];
    Cont &K = S.cont;
    if (!L.init) return kOk;
    if (!c.resume) {
        for (int i = 0; i < L.nlast; ++i) {          // the previous prediction, never consumed
            Op &o = op_of(S, L.last[i]);
            if (o.flags & kOpResolved) continue;
            o.flags |= kOpResolved;
            if (o.started == 0) cancel_prefetch(S, L, o, false);
            else ++L.st[kWasted];
        }
        L.nlast = 0;
        for (int w = 0; w < 8; ++w) L.snap[w] = 0;
        for (int e = 0; e < kExperts; ++e)
            if (L.e2s[e] >= 0) setbit(L.snap, e);
        L.has_snap = 1;
        for (int w = 0; w < 8; ++w) K.prot[w] = 0;
        K.nmiss = 0;
        const int cap = c.flag < kMaxPred ? c.flag : kMaxPred;
        for (int i = 0; i < c.n; ++i) {
            const int e = c.a[i];
            if (e < 0 || e >= kExperts) continue;
            const bool seen = bit(K.prot, e);
            setbit(K.prot, e);
            if (!seen && L.e2s[e] < 0 && K.nmiss < cap) K.miss[K.nmiss++] = e;
        }
        K.idx = 0;
        K.pin_counted = 0;
    }
    // highest-ranked prediction allocated last, so it ends at the MRU end
    for (int i = K.idx; i < K.nmiss; ++i) {
        const int e = K.miss[K.nmiss - 1 - i];
        if (L.e2s[e] >= 0) continue;
        int prev = -1, status = kOk;
        const int s = grab_slot(S, c.layer, K.prot, &prev, &status);
        if (s < 0) {
            K.idx = i;
            return status;
        }
        K.pin_counted = 0;
        lru_place(L, e, s);
        const uint32_t id = new_op(S, c.layer, e, s, prev, kOpPrefetch, L.ntensors);
        L.io[s] = id;
        L.last[L.nlast++] = id;
        ++L.st[kIssued];
        if (!queue_prefetch(S, c.layer, id)) return kErrQueue;
    }
    return kOk;
}

__device__ int do_step(State &S, const CmdArgs &c, Result &r) {
    LayerState &L = S.L[c.layer];
    Cont &K = S.cont;
    const int k = c.n;
    if (!L.init) return kOk;
    uint64_t want[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < k; ++i)
        if (c.a[i] >= 0 && c.a[i] < kExperts) setbit(want, c.a[i]);
    if (!c.resume) {
        L.st[kReq] += (uint64_t)k;
        K.nurg = 0;
        if (L.nlast > 0) {
            for (int i = 0; i < L.nlast; ++i) {      // unwanted predictions first
                Op &o = op_of(S, L.last[i]);
                if ((o.flags & kOpResolved) || bit(want, o.eid)) continue;
                o.flags |= kOpResolved;
                if (o.started == 0) cancel_prefetch(S, L, o, true);
                else ++L.st[kWasted];
            }
            for (int i = 0; i < L.nlast; ++i) {      // then the wanted ones
                Op &o = op_of(S, L.last[i]);
                if ((o.flags & kOpResolved) || !bit(want, o.eid)) continue;
                o.flags |= kOpResolved;
                ++L.st[kUsed];
                if (o.started == 0) {
                    o.flags = (o.flags | kOpPromoted) & ~kOpPrefetch;
                    ++L.st[kPromoted];
                    K.urg[K.nurg++] = L.last[i];
                } else if (o.completed < o.ntasks) {
                    // in flight: its tensors still queued as prefetches move to the urgent queue
                    for (uint32_t q = S.prefetch.head; q != S.prefetch.tail; ++q) {
                        Task &t = S.prefetch.t[q % kRing];
                        if ((t.flags & 2) || t.op[0] != L.last[i]) continue;
                        Task mv = t;
                        t.flags |= 2;
                        if (!ring_push(S.urgent, mv)) return kErrQueue;
                    }
                }
            }
            L.nlast = 0;
        }
        for (uint32_t q = S.prefetch.head; q != S.prefetch.tail; ++q) {   // drop dead prefetch tasks
            Task &t = S.prefetch.t[q % kRing];
            if (t.flags & 2) continue;
            if (op_of(S, t.op[0]).flags & (kOpCancelled | kOpPromoted)) t.flags |= 2;
        }
        for (int w = 0; w < 8; ++w) K.prot[w] = want[w];
        K.idx = 0;
        K.pin_counted = 0;
    }
    for (int i = K.idx; i < k; ++i) {
        const int e = c.a[i];
        if (e < 0 || e >= kExperts) continue;
        if (L.e2s[e] >= 0) {
            if (!L.has_snap || bit(L.snap, e)) ++L.st[kHits];
            continue;
        }
        int prev = -1, status = kOk;
        const int s = grab_slot(S, c.layer, K.prot, &prev, &status);
        if (s < 0) {
            K.idx = i;
            return status;
        }
        K.pin_counted = 0;
        ++L.st[kUrgent];
        lru_place(L, e, s);
        const uint32_t id = new_op(S, c.layer, e, s, prev, 0, L.ntensors);
        L.io[s] = id;
        K.urg[K.nurg++] = id;
    }
    L.has_snap = 0;
    if (!queue_urgent(S, c.layer, K.urg, K.nurg, false)) return kErrQueue;
    L.npend = 0;
    for (int i = 0; i < k; ++i) {
        const int s = L.e2s[c.a[i]];
        lru_touch(L, s);
        r.a[i] = s;
        ++L.pins[s];
        if (L.npinned >= kPinList) return kErrPins;
        L.pinned[L.npinned++] = (int16_t)s;
        if (slot_busy(S, L, s)) L.pend[L.npend++] = L.io[s];
    }
    r.ret = L.npend;
    return kOk;
}

// resident unpinned slots in LRU order: the draws force_invalidate needs
__device__ int fi_candidates(LayerState &L) {
    int n = 0;
    for (int s = L.head, g = 0; s >= 0 && g <= kExperts; s = L.nxt[s], ++g)
        if (L.pins[s] == 0 && L.s2e[s] >= 0) ++n;
    return n;
}

__device__ int do_force(State &S, const CmdArgs &c, Result &r) {
    LayerState &L = S.L[c.layer];
    r.ret = 0;
    if (!L.init || c.rate <= 0.0) return kOk;
    int16_t chosen[kExperts];
    int nch = 0, j = 0;
    for (int s = L.head, g = 0; s >= 0 && g <= kExperts; s = L.nxt[s], ++g) {
        if (L.pins[s] > 0 || L.s2e[s] < 0) continue;
        if (c.rate >= 1.0 || (j < c.n && c.draws[j++] < c.rate)) chosen[nch++] = (int16_t)s;
    }
    int n = 0;
    for (int i = 0; i < nch; ++i) {
        const int s = chosen[i];
        if (L.pins[s] > 0) continue;
        const int e = L.s2e[s];
        if (e < 0) continue;
        const uint32_t a = L.io[s];
        if (a && !op_done(S, a) && !(op_of(S, a).flags & kOpCancelled)) {
            Op &o = op_of(S, a);
            if ((o.flags & kOpPrefetch) && o.started == 0) {
                o.flags |= kOpResolved | kOpCancelled;
                ++L.st[kCancelled];
            } else {
                while (!op_done(S, a) && !(op_of(S, a).flags & kOpCancelled)) {
                    bool ok = true;
                    if (!take_next(S, ok)) return kErrStuck;
                    if (!ok) return kErrExec;
                }
            }
        }
        for (int q = 0; q < L.nlast; ++q) {
            Op &o = op_of(S, L.last[q]);
            if (!(o.flags & kOpResolved) && o.slot == s) {
                o.flags |= kOpResolved;
                ++L.st[kWasted];
            }
        }
        forget_slot(L, s);
        L.snap[e >> 6] &= ~(1ull << (e & 63));
        if (L.row_bytes[0] > 0) {
            if (S.nexec >= kExecMax) return kErrExec;
            S.exec[S.nexec++] = Exec{(int16_t)c.layer, 0, (int16_t)s, 1, e};
        }
        free_push(L, s);
        ++n;
    }
    L.st[kForced] += (uint64_t)n;
    r.ret = n;
    return kOk;
}

__global__ void p1_control(State *S, const CmdArgs *cp, Result *rp) {
    if (threadIdx.x != 0) return;
    const CmdArgs &c = *cp;
    Result &r = *rp;
    r.status = kOk;
    r.ret = 0;
    r.waited = 0;
    S->nexec = 0;
    LayerState &L = S->L[c.layer & (kLayers - 1)];
    int rc = kOk;
    switch (c.cmd) {
    case kCmdInit:
        L.init = 1;
        L.capacity = c.capacity;
        L.ntensors = c.ntensors;
        L.expert_bytes = 0;
        for (int t = 0; t < kTensors; ++t) {
            L.row_bytes[t] = t < c.ntensors ? c.row_bytes[t] : 0;
            L.expert_bytes += L.row_bytes[t];
        }
        if (L.expert_bytes == 0) L.expert_bytes = kDefaultExpertBytes;
        clear_lists(L, true);
        fill_free_all(L);
        for (int i = 0; i < kNumStats; ++i) L.st[i] = 0;
        break;
    case kCmdResize:
        L.capacity = c.capacity;
        clear_lists(L, true);
        place_ordered(L, c.a, c.b, c.n);
        break;
    case kCmdResetCache:
        clear_lists(L, true);
        fill_free_all(L);
        break;
    case kCmdResetStats:
        for (int i = 0; i < kNumStats; ++i) L.st[i] = 0;
        break;
    case kCmdPrefetch:
        rc = do_prefetch(*S, c);
        if (rc == kOk) rc = drain_if_eager(*S);
        break;
    case kCmdStep:
        rc = do_step(*S, c, r);
        if (rc == kOk) rc = drain_if_eager(*S);
        break;
    case kCmdWaitUrgent:
        rc = wait_urgent(*S, c.layer, &r.waited);
        break;
    case kCmdWaitAll:
        rc = wait_all(*S, c.layer, &r.waited);
        break;
    case kCmdUnpinLayer:
        for (int i = 0; i < L.npinned; ++i)
            if (L.pins[L.pinned[i]] > 0) --L.pins[L.pinned[i]];
        L.npinned = 0;
        break;
    case kCmdPin:
    case kCmdUnpin:
        for (int i = 0; i < c.n; ++i) {
            const int s = c.a[i];
            if (s < 0 || s >= kExperts) continue;
            if (c.cmd == kCmdPin) ++L.pins[s];
            else if (L.pins[s] > 0) --L.pins[s];
        }
        break;
    case kCmdPinCount:
        r.ret = (c.n >= 0 && c.n < kExperts) ? L.pins[c.n] : 0;
        break;
    case kCmdFiCount:
        r.ret = L.init ? fi_candidates(L) : 0;
        break;
    case kCmdForce:
        rc = do_force(*S, c, r);
        if (rc == kOk) rc = drain_if_eager(*S);
        break;
    case kCmdLoadSync: {
        if (!L.init) break;
        if (c.flag) L.st[kPfBytes] += (uint64_t)c.n * L.expert_bytes;
        uint32_t ids[kExperts];
        L.npend = 0;
        for (int i = 0; i < c.n; ++i) {
            ids[i] = new_op(*S, c.layer, c.a[i], c.b[i], -1, 0, L.ntensors);
            L.io[c.b[i]] = ids[i];
            if (L.npend < kMaxK) L.pend[L.npend++] = ids[i];
        }
        uint32_t sorted[kExperts];
        for (int i = 0; i < c.n; ++i) sorted[i] = ids[i];
        if (!queue_urgent(*S, c.layer, sorted, c.n, c.flag != 0)) {
            rc = kErrQueue;
            break;
        }
        // every op, not just the first kMaxK, must be done before the call returns
        rc = drain_if_eager(*S);
        if (rc == kOk) rc = wait_urgent(*S, c.layer, &r.waited);
        for (int i = 0; rc == kOk && i < c.n; ++i)
            while (!op_done(*S, ids[i])) {
                bool ok = true;
                if (!take_next(*S, ok)) {
                    rc = kErrStuck;
                    break;
                }
                if (!ok) rc = kErrExec;
            }
        break;
    }
    case kCmdGetLru: {
        int n = 0;
        for (int s = L.head, g = 0; s >= 0 && g <= kExperts; s = L.nxt[s], ++g) {
            r.a[n] = L.s2e[s];
            r.b[n] = s;
            ++n;
        }
        r.count = n;
        break;
    }
    case kCmdSetLru:
        L.st[kPfReq] += c.add[0];
        L.st[kPfHits] += c.add[1];
        L.st[kPfMiss] += c.add[2];
        clear_lists(L, false);
        place_ordered(L, c.a, c.b, c.n);
        break;
    case kCmdGetStats:
        for (int i = 0; i < kNumStats; ++i) r.st[i] = L.st[i];
        break;
    case kCmdGetTotal:
        for (int i = 0; i < kNumStats; ++i) r.st[i] = 0;
        for (int l = 1; l < c.n && l < kLayers; ++l) {
            if (!S->L[l].init) continue;
            for (int i = 0; i < kNumStats; ++i) r.st[i] += S->L[l].st[i];
        }
        break;
    case kCmdSetEager:
        S->eager = c.flag;
        break;
    default:
        break;
    }
    if (rc == kBlockedPin) S->cont.active = 1;
    else S->cont.active = 0;
    r.status = rc;
    r.nexec = S->nexec;
}

// ------------------------------------------------------------------ row copies on the device

struct LayerIo {
    uint64_t src[kTensors], dst[kTensors], rb[kTensors];
    int32_t device_copy;                    // 1: pool -> slots by the copy kernel
    int32_t num_experts, capacity, pad;     // bounds of the pool and of the slot buffers
};

// rows of the execute list whose layer copies on the device; a row written again later in the
// list is skipped (the later write wins), a scrub only if no later copy rewrites that row
__global__ void p1_copy_rows(const State *S, const LayerIo *io, int scrubs) {
    const int n = S->nexec;
    for (int i = blockIdx.y; i < n; i += gridDim.y) {
        const Exec x = S->exec[i];
        const LayerIo &d = io[x.layer];
        if (!d.device_copy || x.kind != scrubs || x.tensor >= kTensors || d.dst[x.tensor] == 0 ||
            (!scrubs && d.src[x.tensor] == 0) || x.slot < 0 || x.slot >= d.capacity ||
            (!scrubs && (x.eid < 0 || x.eid >= d.num_experts)))
            continue;
        bool later = false;
        for (int j = i + 1; j < n && !later; ++j) {
            const Exec y = S->exec[j];
            later = y.kind == 0 && y.layer == x.layer && y.slot == x.slot && y.tensor == x.tensor;
        }
        if (later) continue;
        const uint64_t rb = d.rb[x.tensor];
        unsigned char *dst = reinterpret_cast<unsigned char *>(d.dst[x.tensor]) + (uint64_t)x.slot * rb;
        if (scrubs) {
            const uint64_t m = rb < 64 ? rb : 64;
            for (uint64_t b = threadIdx.x; b < m; b += blockDim.x)
                if (blockIdx.x == 0) dst[b] = 0xA5;
            continue;
        }
        const unsigned char *src = reinterpret_cast<const unsigned char *>(d.src[x.tensor]) + (uint64_t)x.eid * rb;
        const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | rb) & 15) == 0;
        if (vec) {
            const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
            uint4 *d4 = reinterpret_cast<uint4 *>(dst);
            const uint64_t n4 = rb / 16;
            for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < n4; b += (uint64_t)gridDim.x * blockDim.x)
                d4[b] = s4[b];
        } else {
            for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < rb; b += (uint64_t)gridDim.x * blockDim.x)
                dst[b] = src[b];
        }
    }
}

// ------------------------------------------------------------------ host side

struct LayerHost {
    int source;                              // 0 none, 1 file, 2 pool
    int fd;
    int ntensors;
    int capacity;
    int num_experts;                         // rows in the pool (pool sources)
    bool dst_device;
    uint64_t off[kTensors], rb[kTensors], src[kTensors], dst[kTensors];
    uint32_t *slot_inds;                     // host array the slot ids of step_decode go to
};

struct Sched {
    std::mutex mu;
    int device = 0;
    cudaStream_t stream = nullptr;
    State *d_state = nullptr;
    CmdArgs *d_cmd = nullptr, *h_cmd = nullptr;
    Result *d_res = nullptr, *h_res = nullptr;
    Exec *h_exec = nullptr;
    LayerIo *d_io = nullptr;
    LayerIo h_io[kLayers]{};
    LayerHost lay[kLayers]{};
    uint64_t io_wait_ns[kLayers]{};
    uint64_t copy_errors = 0;
    uint64_t launches = 0;                   // control + copy kernels launched so far
    int workers = 6;                         // the reference's default before init()
    bool running = false;
    void (*reader_fn)(void *, int) = nullptr;
    void *reader_user = nullptr;
    std::mt19937_64 rng;
    std::vector<unsigned char> staging;
};

// host-side rows of the execute list (file sources, host destinations), in list order
void host_rows(Sched &h, int nexec) {
    for (int i = 0; i < nexec; ++i) {
        const Exec &x = h.h_exec[i];
        const LayerHost &L = h.lay[x.layer];
        if (h.h_io[x.layer].device_copy || L.source == 0 || x.tensor >= L.ntensors) continue;
        const uint64_t rb = L.rb[x.tensor];
        if (rb == 0 || L.dst[x.tensor] == 0) continue;
        unsigned char *dst = reinterpret_cast<unsigned char *>(L.dst[x.tensor]) + (uint64_t)x.slot * rb;
        if (x.kind == 1) {
            const size_t m = std::min<uint64_t>(64, rb);
            if (L.dst_device) {
                std::vector<unsigned char> a5(m, 0xA5);
                if (cudaMemcpy(dst, a5.data(), m, cudaMemcpyHostToDevice) != cudaSuccess) ++h.copy_errors;
            } else {
                std::memset(dst, 0xA5, m);
            }
            continue;
        }
        if (x.slot < 0 || x.slot >= L.capacity || (L.source == 2 && (x.eid < 0 || x.eid >= L.num_experts))) {
            ++h.copy_errors;
            continue;
        }
        unsigned char *tgt = dst;
        if (L.dst_device) {
            h.staging.resize(rb);
            tgt = h.staging.data();
        }
        if (L.source == 1) {
            uint64_t done = 0;
            while (done < rb) {
                const ssize_t n = ::pread(L.fd, tgt + done, rb - done, (off_t)(L.off[x.tensor] + (uint64_t)x.eid * rb + done));
                if (n <= 0) break;
                done += (uint64_t)n;
            }
            if (done < rb) ++h.copy_errors;
        } else {
            std::memcpy(tgt, reinterpret_cast<const unsigned char *>(L.src[x.tensor]) + (uint64_t)x.eid * rb, rb);
        }
        if (L.dst_device && cudaMemcpy(dst, tgt, rb, cudaMemcpyHostToDevice) != cudaSuccess) ++h.copy_errors;
    }
}

// one call: control kernel (resumed after reader waits), the device row copies, results back
int run(Sched &h, std::unique_lock<std::mutex> &lock) {
    MOE_CUDA_TRY(cudaSetDevice(h.device));
    h.h_cmd->resume = 0;
    for (int round = 0;; ++round) {
        MOE_CUDA_TRY(cudaMemcpyAsync(h.d_cmd, h.h_cmd, sizeof(CmdArgs), cudaMemcpyHostToDevice, h.stream));
        p1_control<<<1, 32, 0, h.stream>>>(h.d_state, h.d_cmd, h.d_res);
        MOE_CUDA_TRY(cudaGetLastError());
        ++h.launches;
        MOE_CUDA_TRY(cudaMemcpyAsync(h.h_res, h.d_res, sizeof(Result), cudaMemcpyDeviceToHost, h.stream));
        MOE_CUDA_TRY(cudaStreamSynchronize(h.stream));
        const int nexec = h.h_res->nexec;
        if (nexec > 0) {
            // device rows run behind the call on the stream (later calls, and every wait, are
            // ordered after them); rows the host moves need the list back now
            p1_copy_rows<<<dim3(16, std::min(nexec, 1024)), 256, 0, h.stream>>>(h.d_state, h.d_io, 0);
            p1_copy_rows<<<dim3(1, std::min(nexec, 1024)), 64, 0, h.stream>>>(h.d_state, h.d_io, 1);
            MOE_CUDA_TRY(cudaGetLastError());
            h.launches += 2;
            bool host_side = false;
            for (int l = 0; l < kLayers && !host_side; ++l) host_side = h.lay[l].source != 0 && !h.h_io[l].device_copy;
            if (host_side) {
                MOE_CUDA_TRY(cudaMemcpyAsync(h.h_exec,
                                             reinterpret_cast<const char *>(h.d_state) + offsetof(State, exec),
                                             sizeof(Exec) * (size_t)nexec, cudaMemcpyDeviceToHost, h.stream));
                MOE_CUDA_TRY(cudaStreamSynchronize(h.stream));
                host_rows(h, nexec);
            }
        }
        const int st = h.h_res->status;
        if (st == kOk) return MOE_OK;
        if (st != kBlockedPin)
            return moe_set_error(MOE_EIO, "p1 scheduler: %s (call %d, layer %d)",
                                 st == kErrQueue ? "task queue full" : st == kErrExec ? "execute list full"
                                 : st == kErrPins ? "too many pins held" : "a read can never complete",
                                 h.h_cmd->cmd, h.h_cmd->layer);
        // only slots pinned by a reader block the allocation: let the reader finish and unpin
        if (!h.reader_fn || round > 100000)
            return moe_set_error(MOE_ETIMEDOUT, "p1 scheduler: every evictable slot of layer %d is pinned",
                                 h.h_cmd->layer);
        const CmdArgs saved = *h.h_cmd;
        auto fn = h.reader_fn;
        void *user = h.reader_user;
        const int layer = h.h_cmd->layer;
        lock.unlock();
        fn(user, layer);
        lock.lock();
        *h.h_cmd = saved;
        h.h_cmd->resume = 1;
    }
}

int simple(Sched &h, int cmd, int layer) {
    std::unique_lock<std::mutex> lock(h.mu);
    std::memset(h.h_cmd, 0, offsetof(CmdArgs, a));
    h.h_cmd->cmd = cmd;
    h.h_cmd->layer = layer;
    return run(h, lock);
}

bool bad_layer(int layer) { return layer < 0 || layer >= kLayers; }

int wait_all_locked(Sched &h, std::unique_lock<std::mutex> &lock, int layer) {
    std::memset(h.h_cmd, 0, offsetof(CmdArgs, a));
    h.h_cmd->cmd = kCmdWaitUrgent;
    h.h_cmd->layer = layer;
    const auto t0 = std::chrono::steady_clock::now();
    int rc = run(h, lock);
    if (rc) return rc;
    if (h.h_res->waited)
        h.io_wait_ns[layer] += (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                   std::chrono::steady_clock::now() - t0).count();
    h.h_cmd->cmd = kCmdWaitAll;
    return run(h, lock);
}

int push_io(Sched &h, int layer) {
    LayerIo &d = h.h_io[layer];
    const LayerHost &L = h.lay[layer];
    for (int t = 0; t < kTensors; ++t) {
        d.src[t] = L.src[t];
        d.dst[t] = L.dst[t];
        d.rb[t] = t < L.ntensors ? L.rb[t] : 0;
    }
    d.device_copy = (L.source == 2 && L.dst_device) ? 1 : 0;
    d.num_experts = L.num_experts;
    d.capacity = L.capacity;
    MOE_CUDA_TRY(cudaMemcpy(h.d_io + layer, &d, sizeof(LayerIo), cudaMemcpyHostToDevice));
    return MOE_OK;
}

}  // namespace

// ------------------------------------------------------------------ C ABI (include/moe_b200.h)

extern "C" void *moe_p1_create(void) {
    Sched *h = new (std::nothrow) Sched();
    if (!h) return nullptr;
    bool ok = cudaGetDevice(&h->device) == cudaSuccess &&
              cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaMalloc(&h->d_state, sizeof(State)) == cudaSuccess &&
              cudaMemsetAsync(h->d_state, 0, sizeof(State), h->stream) == cudaSuccess &&
              cudaMalloc(&h->d_cmd, sizeof(CmdArgs)) == cudaSuccess &&
              cudaMalloc(&h->d_res, sizeof(Result)) == cudaSuccess &&
              cudaMalloc(&h->d_io, sizeof(LayerIo) * kLayers) == cudaSuccess &&
              cudaMemsetAsync(h->d_io, 0, sizeof(LayerIo) * kLayers, h->stream) == cudaSuccess &&
              cudaMallocHost(&h->h_cmd, sizeof(CmdArgs)) == cudaSuccess &&
              cudaMallocHost(&h->h_res, sizeof(Result)) == cudaSuccess &&
              cudaMallocHost(&h->h_exec, sizeof(Exec) * kExecMax) == cudaSuccess &&
              cudaStreamSynchronize(h->stream) == cudaSuccess;
    if (!ok) {
        moe_set_error(MOE_ENOMEM, "p1 scheduler: device state allocation failed");
        if (h->d_state) cudaFree(h->d_state);
        if (h->d_cmd) cudaFree(h->d_cmd);
        if (h->d_res) cudaFree(h->d_res);
        if (h->d_io) cudaFree(h->d_io);
        if (h->h_cmd) cudaFreeHost(h->h_cmd);
        if (h->h_res) cudaFreeHost(h->h_res);
        if (h->h_exec) cudaFreeHost(h->h_exec);
        if (h->stream) cudaStreamDestroy(h->stream);
        delete h;
        return nullptr;
    }
    return h;
}

extern "C" void moe_p1_destroy(void *hp) {
    Sched *h = static_cast<Sched *>(hp);
    if (!h) return;
    cudaSetDevice(h->device);
    cudaStreamSynchronize(h->stream);
    cudaFree(h->d_state);
    cudaFree(h->d_cmd);
    cudaFree(h->d_res);
    cudaFree(h->d_io);
    cudaFreeHost(h->h_cmd);
    cudaFreeHost(h->h_res);
    cudaFreeHost(h->h_exec);
    cudaStreamDestroy(h->stream);
    delete h;
}

#define P1_HANDLE(hp)                                                                   \
    Sched *h = static_cast<Sched *>(hp);                                                \
    if (!h) return moe_set_error(MOE_EINVAL, "p1 scheduler: null handle");

// workers = the copy engine taking every queued task at the end of each call
extern "C" int moe_p1_init(void *hp, int num_threads) {
    P1_HANDLE(hp);
    std::unique_lock<std::mutex> lock(h->mu);
    if (h->running) return MOE_OK;
    h->workers = std::clamp(num_threads, 1, 32);
    h->running = true;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdSetEager;
    h->h_cmd->flag = 1;
    return run(*h, lock);
}

extern "C" int moe_p1_shutdown(void *hp) {
    P1_HANDLE(hp);
    std::unique_lock<std::mutex> lock(h->mu);
    if (!h->running) return MOE_OK;
    h->running = false;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdSetEager;
    h->h_cmd->flag = 0;
    return run(*h, lock);
}

extern "C" int moe_p1_num_threads(void *hp) {
    Sched *h = static_cast<Sched *>(hp);
    return h ? h->workers : 0;
}

extern "C" int moe_p1_set_wait_reader_callback(void *hp, void (*fn)(void *, int), void *user) {
    P1_HANDLE(hp);
    std::unique_lock<std::mutex> lock(h->mu);
    h->reader_fn = fn;
    h->reader_user = user;
    return MOE_OK;
}

static int layer_setup(Sched *h, int layer, int capacity, int num_tensors, const uint64_t *row_bytes) {
    std::unique_lock<std::mutex> lock(h->mu);
    int rc = wait_all_locked(*h, lock, layer);
    if (rc) return rc;
    h->lay[layer].capacity = std::clamp(capacity, 1, kExperts);
    rc = push_io(*h, layer);
    if (rc) return rc;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdInit;
    h->h_cmd->layer = layer;
    h->h_cmd->capacity = std::clamp(capacity, 1, kExperts);
    h->h_cmd->ntensors = std::clamp(num_tensors, 1, kTensors);
    for (int t = 0; t < h->h_cmd->ntensors; ++t) h->h_cmd->row_bytes[t] = row_bytes[t];
    h->io_wait_ns[layer] = 0;
    return run(*h, lock);
}

extern "C" int moe_p1_layer_init(void *hp, int layer, int fd, int capacity, int num_tensors,
                                 const uint64_t *base_offsets, const uint64_t *row_bytes, const uint64_t *base_ptrs,
                                 uint64_t slot_inds_ptr) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    if (!base_offsets || !row_bytes || !base_ptrs) return moe_set_error(MOE_EINVAL, "p1 layer_init: null array");
    LayerHost &L = h->lay[layer];
    {
        std::unique_lock<std::mutex> lock(h->mu);
        int rc = wait_all_locked(*h, lock, layer);
        if (rc) return rc;
        L = LayerHost{};
        L.source = 1;
        L.fd = fd;
        L.ntensors = std::clamp(num_tensors, 1, kTensors);
        for (int t = 0; t < L.ntensors; ++t) {
            L.off[t] = base_offsets[t];
            L.rb[t] = row_bytes[t];
            L.dst[t] = base_ptrs[t];
        }
        L.slot_inds = reinterpret_cast<uint32_t *>(static_cast<uintptr_t>(slot_inds_ptr));
    }
    return layer_setup(h, layer, capacity, num_tensors, row_bytes);
}

extern "C" int moe_p1_layer_init_pool(void *hp, int layer, int capacity, int num_tensors, int num_experts,
                                      const uint64_t *src_ptrs, const uint64_t *row_bytes, const uint64_t *slot_ptrs,
                                      uint64_t slot_inds_ptr, int slots_on_device, int device) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    if (!src_ptrs || !row_bytes || !slot_ptrs) return moe_set_error(MOE_EINVAL, "p1 layer_init_pool: null array");
    if (num_experts <= 0 || num_experts > kExperts)
        return moe_set_error(MOE_EINVAL, "p1 layer_init_pool: %d experts in the pool (1..%d)", num_experts, kExperts);
    if (slots_on_device && device != h->device)
        return moe_set_error(MOE_EINVAL, "p1 layer_init_pool: slots on device %d, scheduler on device %d", device,
                             h->device);
    LayerHost &L = h->lay[layer];
    {
        std::unique_lock<std::mutex> lock(h->mu);
        int rc = wait_all_locked(*h, lock, layer);
        if (rc) return rc;
        L = LayerHost{};
        L.source = 2;
        L.fd = -1;
        L.num_experts = num_experts;
        L.dst_device = slots_on_device != 0;
        L.ntensors = std::clamp(num_tensors, 1, kTensors);
        for (int t = 0; t < L.ntensors; ++t) {
            L.src[t] = src_ptrs[t];
            L.rb[t] = row_bytes[t];
            L.dst[t] = slot_ptrs[t];
        }
        L.slot_inds = reinterpret_cast<uint32_t *>(static_cast<uintptr_t>(slot_inds_ptr));
    }
    return layer_setup(h, layer, capacity, num_tensors, row_bytes);
}

extern "C" int moe_p1_resize_layer(void *hp, int layer, int new_capacity, const uint64_t *new_base_ptrs,
                                   uint64_t slot_inds_ptr, const int32_t *ordered_eids, const int32_t *ordered_slots,
                                   int count) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    if (!new_base_ptrs || (count > 0 && (!ordered_eids || !ordered_slots)) || count > kExperts)
        return moe_set_error(MOE_EINVAL, "p1 resize_layer: bad arrays");
    std::unique_lock<std::mutex> lock(h->mu);
    int rc = wait_all_locked(*h, lock, layer);
    if (rc) return rc;
    LayerHost &L = h->lay[layer];
    for (int t = 0; t < L.ntensors; ++t) L.dst[t] = new_base_ptrs[t];
    L.slot_inds = reinterpret_cast<uint32_t *>(static_cast<uintptr_t>(slot_inds_ptr));
    L.capacity = std::clamp(new_capacity, 1, kExperts);
    rc = push_io(*h, layer);
    if (rc) return rc;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdResize;
    h->h_cmd->layer = layer;
    h->h_cmd->capacity = std::clamp(new_capacity, 1, kExperts);
    h->h_cmd->n = std::max(count, 0);
    for (int i = 0; i < h->h_cmd->n; ++i) {
        h->h_cmd->a[i] = ordered_eids[i];
        h->h_cmd->b[i] = ordered_slots[i];
    }
    return run(*h, lock);
}

extern "C" int moe_p1_reset_cache(void *hp, int layer) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    std::unique_lock<std::mutex> lock(h->mu);
    int rc = wait_all_locked(*h, lock, layer);
    if (rc) return rc;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdResetCache;
    h->h_cmd->layer = layer;
    return run(*h, lock);
}

extern "C" int moe_p1_reset_stats(void *hp, int layer) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    std::unique_lock<std::mutex> lock(h->mu);
    h->io_wait_ns[layer] = 0;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdResetStats;
    h->h_cmd->layer = layer;
    return run(*h, lock);
}

extern "C" int moe_p1_start_prefetch(void *hp, int layer, const int32_t *pred_eids, int pred_count, int max_fetch) {
    P1_HANDLE(hp);
    if (bad_layer(layer) || !pred_eids || pred_count <= 0 || max_fetch <= 0) return MOE_OK;
    if (pred_count > kMaxPredIn) return moe_set_error(MOE_EINVAL, "p1 start_prefetch: %d predictions (max %d)",
                                                      pred_count, kMaxPredIn);
    std::unique_lock<std::mutex> lock(h->mu);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdPrefetch;
    h->h_cmd->layer = layer;
    h->h_cmd->n = pred_count;
    h->h_cmd->flag = max_fetch;
    std::memcpy(h->h_cmd->a, pred_eids, sizeof(int32_t) * (size_t)pred_count);
    return run(*h, lock);
}

extern "C" int moe_p1_step_decode(void *hp, int layer, const uint32_t *eids, int k, uint32_t *out_slots) {
    P1_HANDLE(hp);
    if (bad_layer(layer) || !eids || k <= 0) return 0;
    if (k > kMaxK) return moe_set_error(MOE_EINVAL, "p1 step_decode: k=%d (max %d)", k, kMaxK);
    for (int i = 0; i < k; ++i)
        if (eids[i] >= (uint32_t)kExperts) return moe_set_error(MOE_EINVAL, "p1 step_decode: expert %u", eids[i]);
    std::unique_lock<std::mutex> lock(h->mu);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdStep;
    h->h_cmd->layer = layer;
    h->h_cmd->n = k;
    for (int i = 0; i < k; ++i) h->h_cmd->a[i] = (int32_t)eids[i];
    const int rc = run(*h, lock);
    if (rc) return rc;
    uint32_t *dst = h->lay[layer].slot_inds;
    for (int i = 0; i < k; ++i) {
        if (dst) dst[i] = (uint32_t)h->h_res->a[i];
        if (out_slots) out_slots[i] = (uint32_t)h->h_res->a[i];
    }
    return h->h_res->ret;
}

extern "C" int moe_p1_wait_layer_urgent(void *hp, int layer) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    std::unique_lock<std::mutex> lock(h->mu);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdWaitUrgent;
    h->h_cmd->layer = layer;
    const auto t0 = std::chrono::steady_clock::now();
    const int rc = run(*h, lock);
    if (rc == MOE_OK && h->h_res->waited)
        h->io_wait_ns[layer] += (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                    std::chrono::steady_clock::now() - t0).count();
    return rc;
}

extern "C" int moe_p1_wait_layer_all(void *hp, int layer) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    std::unique_lock<std::mutex> lock(h->mu);
    return wait_all_locked(*h, lock, layer);
}

extern "C" int moe_p1_wait_all(void *hp) {
    P1_HANDLE(hp);
    std::unique_lock<std::mutex> lock(h->mu);
    for (int l = 0; l < kLayers; ++l) {
        const int rc = wait_all_locked(*h, lock, l);
        if (rc) return rc;
    }
    return MOE_OK;
}

extern "C" int moe_p1_unpin_layer_slots(void *hp, int layer) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    return simple(*h, kCmdUnpinLayer, layer);
}

static int pin_cmd(Sched *h, int cmd, int layer, const uint32_t *slots, int count) {
    if (bad_layer(layer) || !slots || count <= 0) return MOE_OK;
    std::unique_lock<std::mutex> lock(h->mu);
    for (int i0 = 0; i0 < count; i0 += kMaxPredIn) {
        std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
        h->h_cmd->cmd = cmd;
        h->h_cmd->layer = layer;
        h->h_cmd->n = std::min(count - i0, kMaxPredIn);
        for (int i = 0; i < h->h_cmd->n; ++i) h->h_cmd->a[i] = (int32_t)std::min<uint32_t>(slots[i0 + i], 1u << 30);
        const int rc = run(*h, lock);
        if (rc) return rc;
    }
    return MOE_OK;
}

extern "C" int moe_p1_pin_slots(void *hp, int layer, const uint32_t *slots, int count) {
    P1_HANDLE(hp);
    return pin_cmd(h, kCmdPin, layer, slots, count);
}

extern "C" int moe_p1_unpin_slots(void *hp, int layer, const uint32_t *slots, int count) {
    P1_HANDLE(hp);
    return pin_cmd(h, kCmdUnpin, layer, slots, count);
}

extern "C" int moe_p1_get_slot_pin_count(void *hp, int layer, int slot) {
    P1_HANDLE(hp);
    if (bad_layer(layer) || slot < 0 || slot >= kExperts) return 0;
    std::unique_lock<std::mutex> lock(h->mu);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdPinCount;
    h->h_cmd->layer = layer;
    h->h_cmd->n = slot;
    const int rc = run(*h, lock);
    return rc ? rc : h->h_res->ret;
}

extern "C" int moe_p1_seed(void *hp, uint64_t seed) {
    P1_HANDLE(hp);
    std::unique_lock<std::mutex> lock(h->mu);
    h->rng.seed(seed);
    return MOE_OK;
}

// the uniform draws come from the handle's std::mt19937_64 on the host, one per resident
// unpinned slot in LRU order (none when rate >= 1), the same sequence the reference draws
extern "C" int moe_p1_force_invalidate(void *hp, int layer, double rate) {
    P1_HANDLE(hp);
    if (bad_layer(layer) || rate <= 0.0) return 0;
    std::unique_lock<std::mutex> lock(h->mu);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdFiCount;
    h->h_cmd->layer = layer;
    int rc = run(*h, lock);
    if (rc) return rc;
    const int n = h->h_res->ret;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdForce;
    h->h_cmd->layer = layer;
    h->h_cmd->rate = rate;
    h->h_cmd->n = rate >= 1.0 ? 0 : n;
    std::uniform_real_distribution<double> dist(0.0, 1.0);
    for (int i = 0; i < h->h_cmd->n; ++i) h->h_cmd->draws[i] = dist(h->rng);
    rc = run(*h, lock);
    return rc ? rc : h->h_res->ret;
}

extern "C" int moe_p1_load_sync(void *hp, int layer, const int32_t *eids, const int32_t *slots, int count,
                                int is_prefill) {
    P1_HANDLE(hp);
    if (bad_layer(layer) || count <= 0) return MOE_OK;
    if (!eids || !slots || count > kExperts) return moe_set_error(MOE_EINVAL, "p1 load_sync: bad arrays");
    std::unique_lock<std::mutex> lock(h->mu);
    int rc = wait_all_locked(*h, lock, layer);
    if (rc) return rc;
    for (int i = 0; i < count; ++i)
        if (eids[i] < 0 || eids[i] >= kExperts || slots[i] < 0 || slots[i] >= h->lay[layer].capacity)
            return moe_set_error(MOE_EINVAL, "p1 load_sync: expert %d slot %d (capacity %d)", eids[i], slots[i],
                                 h->lay[layer].capacity);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdLoadSync;
    h->h_cmd->layer = layer;
    h->h_cmd->n = count;
    h->h_cmd->flag = is_prefill ? 1 : 0;
    std::memcpy(h->h_cmd->a, eids, sizeof(int32_t) * (size_t)count);
    std::memcpy(h->h_cmd->b, slots, sizeof(int32_t) * (size_t)count);
    const auto t0 = std::chrono::steady_clock::now();
    rc = run(*h, lock);
    if (rc == MOE_OK && h->h_res->waited)
        h->io_wait_ns[layer] += (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                    std::chrono::steady_clock::now() - t0).count();
    return rc;
}

extern "C" int moe_p1_get_lru_state(void *hp, int layer, int32_t *out_eids, int32_t *out_slots, int *out_count) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) {
        if (out_count) *out_count = 0;
        return MOE_OK;
    }
    if (!out_eids || !out_slots || !out_count) return moe_set_error(MOE_EINVAL, "p1 get_lru_state: null output");
    std::unique_lock<std::mutex> lock(h->mu);
    int rc = wait_all_locked(*h, lock, layer);
    if (rc) return rc;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdGetLru;
    h->h_cmd->layer = layer;
    rc = run(*h, lock);
    if (rc) return rc;
    const int n = h->h_res->count;
    std::memcpy(out_eids, h->h_res->a, sizeof(int32_t) * (size_t)n);
    std::memcpy(out_slots, h->h_res->b, sizeof(int32_t) * (size_t)n);
    *out_count = n;
    return MOE_OK;
}

extern "C" int moe_p1_set_lru_state(void *hp, int layer, const int32_t *ordered_eids, const int32_t *ordered_slots,
                                    int count, uint64_t add_prefill_requests, uint64_t add_prefill_hits,
                                    uint64_t add_prefill_misses) {
    P1_HANDLE(hp);
    if (bad_layer(layer)) return MOE_OK;
    if ((count > 0 && (!ordered_eids || !ordered_slots)) || count > kExperts)
        return moe_set_error(MOE_EINVAL, "p1 set_lru_state: bad arrays");
    std::unique_lock<std::mutex> lock(h->mu);
    int rc = wait_all_locked(*h, lock, layer);
    if (rc) return rc;
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdSetLru;
    h->h_cmd->layer = layer;
    h->h_cmd->n = std::max(count, 0);
    h->h_cmd->add[0] = add_prefill_requests;
    h->h_cmd->add[1] = add_prefill_hits;
    h->h_cmd->add[2] = add_prefill_misses;
    for (int i = 0; i < h->h_cmd->n; ++i) {
        h->h_cmd->a[i] = ordered_eids[i];
        h->h_cmd->b[i] = ordered_slots[i];
    }
    return run(*h, lock);
}

extern "C" int moe_p1_get_layer_stats(void *hp, int layer, uint64_t *out) {
    P1_HANDLE(hp);
    if (!out) return moe_set_error(MOE_EINVAL, "p1 get_layer_stats: null output");
    if (bad_layer(layer)) {
        std::memset(out, 0, sizeof(uint64_t) * kNumStats);
        return MOE_OK;
    }
    std::unique_lock<std::mutex> lock(h->mu);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdGetStats;
    h->h_cmd->layer = layer;
    const int rc = run(*h, lock);
    if (rc) return rc;
    std::memcpy(out, h->h_res->st, sizeof(uint64_t) * kNumStats);
    out[kIoWait] = h->io_wait_ns[layer];
    return MOE_OK;
}

extern "C" int moe_p1_get_total_stats(void *hp, int num_layers, uint64_t *out) {
    P1_HANDLE(hp);
    if (!out) return moe_set_error(MOE_EINVAL, "p1 get_total_stats: null output");
    std::unique_lock<std::mutex> lock(h->mu);
    std::memset(h->h_cmd, 0, offsetof(CmdArgs, a));
    h->h_cmd->cmd = kCmdGetTotal;
    h->h_cmd->n = num_layers;
    const int rc = run(*h, lock);
    if (rc) return rc;
    std::memcpy(out, h->h_res->st, sizeof(uint64_t) * kNumStats);
    uint64_t w = 0;
    for (int l = 1; l < std::min(num_layers, kLayers); ++l) w += h->io_wait_ns[l];
    out[kIoWait] = w;
    return MOE_OK;
}

extern "C" uint64_t moe_p1_copy_errors(void *hp) {
    Sched *h = static_cast<Sched *>(hp);
    return h ? h->copy_errors : 0;
}

extern "C" uint64_t moe_p1_launches(void *hp) {
    Sched *h = static_cast<Sched *>(hp);
    return h ? h->launches : 0;
}
