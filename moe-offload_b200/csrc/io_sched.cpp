// P1 I/O scheduler of the reference's offload engine (mlx-qwen38/cpp/src/io_sched.h:46-245,
// io_sched.cpp), built for a B200 host: the expert bytes come from a pinned host pool (or
// from the reference's expert file through pread) and land in slot buffers in device memory
// (cudaMemcpyAsync on a per-thread non-blocking stream) or in host memory.
//
// Observable behaviour kept from the reference, call for call:
//   - two queues: URGENT (demand misses, promoted prefetches, synchronous loads) is always
//     served before PREFETCH; worker threads and any caller that waits help drain them;
//   - start_prefetch: resolves the layer's previous unconsumed prefetches (not started ->
//     cancelled, slot handed back to the expert it displaced; started -> wasted), snapshots
//     residency, protects every prediction, fetches the first max_fetch (<= 32) missing ones,
//     allocating slots in reverse rank order (the best prediction ends up most recent);
//   - step_decode: cancels unneeded unstarted prefetches, promotes needed unstarted ones to
//     URGENT, moves the queued tensor copies of needed in-flight ones to URGENT, counts hits
//     against the pre-prefetch snapshot, reads demand misses as coalesced runs of consecutive
//     expert ids (<= 16 per copy task, large tensors before scales/biases), then moves the k
//     slots to MRU, pins them, writes the slot ids and returns the number still loading;
//   - slot allocation: free stack first (lowest slot first on a fresh layer), then the least
//     recent slot that is neither protected, pinned nor loading; when only pinned slots block
//     it counts one pin wait and calls the reader-wait callback (or waits for an unpin), when
//     only loading slots block it executes queued copies itself;
//   - force_invalidate (forced-miss stress, std::mt19937_64 + uniform_real_distribution),
//     load_sync, get/set_lru_state, resize_layer, per-layer and total statistics.
// Layer ids outside 0..63 are ignored as in the reference; the C ABI below adds status codes
// and a handle. Without init() there are no worker threads: queued copies then run only inside
// the calls that wait for them, which makes every result deterministic.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

#include <unistd.h>

#include <cuda_runtime.h>

#include "../../include/moe_b200.h"

int moe_set_error(int code, const char *fmt, ...);   // errors.cpp

namespace {

constexpr int kLayers = 64;
constexpr int kExperts = 512;
constexpr int kTensors = 9;
constexpr int kRun = 16;                        // copies per coalesced task
constexpr int kMaxPrefetch = 32;
constexpr uint64_t kDefaultExpertBytes = 1536000ull;
constexpr uint64_t kLargeRow = 100000ull;       // tensors with larger rows are copied first

struct Op {
    int layer = 0, eid = -1, slot = -1, prev_eid = -1;
    bool prefetch = false, promoted = false, cancelled = false, resolved = false, done = false;
    int started = 0, completed = 0, total = 0;
};
using OpPtr = std::shared_ptr<Op>;

struct Seg {
    uint64_t src = 0;       // file offset or host address
    void *dst = nullptr;
    size_t len = 0;
    OpPtr op;
};

struct Task {
    int layer = 0;
    bool prefill = false;
    int nseg = 0;
    Seg seg[kRun];
};

struct Stats {
    uint64_t v[MOE_P1_STATS] = {};
};
enum {
    S_DECODE_REQ, S_HITS, S_URGENT, S_PF_ISSUED, S_PF_CANCELLED, S_PF_PROMOTED, S_PF_USED, S_PF_WASTED,
    S_PIN_WAITS, S_BYTES, S_IO_WAIT_NS, S_FORCED, S_PRE_REQ, S_PRE_HITS, S_PRE_MISSES, S_PRE_BYTES
};
static_assert(S_PRE_BYTES + 1 == MOE_P1_STATS, "stats layout");

struct Layer {
    bool init = false;
    int fd = -1;                       // >= 0: rows come from this file (pread)
    int cap = 0, nt = kTensors;
    uint64_t src[kTensors] = {};       // file offsets (fd >= 0) or host pool addresses of expert 0
    uint64_t rb[kTensors] = {};
    char *dst[kTensors] = {};
    bool dst_dev = false;
    int device = 0;
    uint32_t *slot_out = nullptr;      // host array receiving step_decode's slot ids
    uint64_t expert_bytes = kDefaultExpertBytes;

    int16_t e2s[kExperts], s2e[kExperts], prv[kExperts], nxt[kExperts];
    int16_t head = -1, tail = -1;
    std::vector<int16_t> free_stack;   // top = back
    int pins[kExperts] = {};
    std::vector<int16_t> reader_pins;  // slots pinned by step_decode for the current reader
    OpPtr io[kExperts];

    bool snap = false;
    uint64_t snap_bm[8] = {};
    std::vector<OpPtr> last_prefetch, pending;
    Stats st;
    std::atomic<uint64_t> bytes{0};
};

inline bool bm_has(const uint64_t *bm, int e) { return (bm[e >> 6] >> (e & 63)) & 1ull; }
inline void bm_set(uint64_t *bm, int e) { bm[e >> 6] |= 1ull << (e & 63); }
inline void bm_clear(uint64_t *bm, int e) { bm[e >> 6] &= ~(1ull << (e & 63)); }

// one non-blocking stream per thread that executes device copies, released with the thread
struct TlsStream {
    cudaStream_t s = nullptr;
    int dev = -1;
    ~TlsStream() {
        if (s) cudaStreamDestroy(s);
    }
};
thread_local TlsStream tls_stream;

class Scheduler {
public:
    ~Scheduler() { shutdown(); }

    void init(int threads) {
        std::unique_lock<std::mutex> lk(mu_);
        if (running_) return;
        nthreads_ = std::clamp(threads, 1, 32);     // as the reference: init(0) still starts one worker
        stop_ = false;
        urgent_.clear();
        prefetch_.clear();
        for (int i = 0; i < nthreads_; ++i) workers_.emplace_back([this] { worker(); });
        running_ = true;
    }

    void shutdown() {
        std::vector<std::thread> ws;
        {
            std::unique_lock<std::mutex> lk(mu_);
            if (!running_) return;
            stop_ = true;
            work_cv_.notify_all();
            done_cv_.notify_all();
            ws.swap(workers_);
            running_ = false;
        }
        for (auto &w : ws)
            if (w.joinable()) w.join();
    }

    void set_reader_wait(void (*fn)(void *, int), void *user) {
        std::unique_lock<std::mutex> lk(mu_);
        reader_fn_ = fn;
        reader_user_ = user;
    }

    void layer_init(int l, int fd, int cap, int nt, const uint64_t *src, const uint64_t *rb, const uint64_t *dst,
                    uint64_t slot_out, int dst_dev, int device) {
        if (!valid(l)) return;
        wait_layer_all(l);
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        L.init = true;
        L.fd = fd;
        L.cap = std::clamp(cap, 1, kExperts);
        L.nt = std::clamp(nt, 1, kTensors);
        uint64_t sum = 0;
        for (int t = 0; t < L.nt; ++t) {
            L.src[t] = src[t];
            L.rb[t] = rb[t];
            L.dst[t] = reinterpret_cast<char *>(static_cast<uintptr_t>(dst[t]));
            sum += rb[t];
        }
        L.expert_bytes = sum ? sum : kDefaultExpertBytes;
        L.dst_dev = dst_dev != 0;
        L.device = device;
        L.slot_out = reinterpret_cast<uint32_t *>(static_cast<uintptr_t>(slot_out));
        clear_map(L, true);
        fresh_free_stack(L);
        L.st = Stats{};
        L.bytes.store(0, std::memory_order_relaxed);
    }

    void resize_layer(int l, int cap, const uint64_t *dst, uint64_t slot_out, const int32_t *eids,
                      const int32_t *slots, int n) {
        if (!valid(l)) return;
        wait_layer_all(l);
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        L.cap = std::clamp(cap, 1, kExperts);
        for (int t = 0; t < L.nt; ++t) L.dst[t] = reinterpret_cast<char *>(static_cast<uintptr_t>(dst[t]));
        L.slot_out = reinterpret_cast<uint32_t *>(static_cast<uintptr_t>(slot_out));
        clear_map(L, true);
        rebuild(L, eids, slots, n);
    }

    void reset_cache(int l) {
        if (!valid(l)) return;
        wait_layer_all(l);
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        clear_map(L, true);
        fresh_free_stack(L);
    }

    void reset_stats(int l) {
        if (!valid(l)) return;
        std::unique_lock<std::mutex> lk(mu_);
        L_[l].st = Stats{};
        L_[l].bytes.store(0, std::memory_order_relaxed);
    }

    void start_prefetch(int l, const int32_t *pred, int n, int max_fetch) {
        if (!valid(l) || !pred || n <= 0 || max_fetch <= 0) return;
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        if (!L.init) return;
        for (auto &op : L.last_prefetch) {
            if (!op || op->resolved) continue;
            op->resolved = true;
            if (op->started == 0) {
                op->cancelled = true;
                L.st.v[S_PF_CANCELLED]++;
                give_back(L, *op, false);
            } else {
                L.st.v[S_PF_WASTED]++;
            }
        }
        L.last_prefetch.clear();

        std::memset(L.snap_bm, 0, sizeof(L.snap_bm));
        for (int e = 0; e < kExperts; ++e)
            if (L.e2s[e] >= 0) bm_set(L.snap_bm, e);
        L.snap = true;

        uint64_t protect[8] = {};
        int want[kMaxPrefetch];
        int nwant = 0;
        const int limit = std::min(max_fetch, kMaxPrefetch);
        for (int i = 0; i < n; ++i) {
            const int e = pred[i];
            if (e < 0 || e >= kExperts) continue;
            const bool seen = bm_has(protect, e);
            bm_set(protect, e);
            if (!seen && L.e2s[e] < 0 && nwant < limit) want[nwant++] = e;
        }
        if (!nwant) return;
        for (int i = nwant - 1; i >= 0; --i) {          // reverse rank: the best ends most recent
            const int e = want[i];
            if (L.e2s[e] >= 0) continue;
            int prev = -1;
            const int s = alloc(l, lk, protect, &prev);
            map_mru(L, e, s);
            OpPtr op = std::make_shared<Op>();
            op->layer = l;
            op->eid = e;
            op->slot = s;
            op->prev_eid = prev;
            op->prefetch = true;
            op->total = L.nt;
            L.io[s] = op;
            L.last_prefetch.push_back(op);
            L.st.v[S_PF_ISSUED]++;
            queue_prefetch(l, L, op);
        }
        work_cv_.notify_all();
    }

    int step_decode(int l, const uint32_t *eids, int k, uint32_t *out) {
        if (!valid(l) || !eids || k <= 0) return 0;
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        if (!L.init) return 0;
        L.st.v[S_DECODE_REQ] += (uint64_t)k;
        uint64_t need[8] = {};
        for (int i = 0; i < k; ++i)
            if (eids[i] < (uint32_t)kExperts) bm_set(need, (int)eids[i]);

        std::vector<OpPtr> urgent_ops;
        if (!L.last_prefetch.empty()) {
            for (auto &op : L.last_prefetch) {          // unneeded first: their slots come back
                if (!op || op->resolved || bm_has(need, op->eid)) continue;
                op->resolved = true;
                if (op->started == 0) {
                    op->cancelled = true;
                    L.st.v[S_PF_CANCELLED]++;
                    give_back(L, *op, true);
                } else {
                    L.st.v[S_PF_WASTED]++;
                }
            }
            for (auto &op : L.last_prefetch) {
                if (!op || op->resolved || !bm_has(need, op->eid)) continue;
                op->resolved = true;
                L.st.v[S_PF_USED]++;
                if (op->started == 0) {
                    op->promoted = true;
                    op->prefetch = false;
                    L.st.v[S_PF_PROMOTED]++;
                    urgent_ops.push_back(op);
                } else if (!op->done) {
                    for (auto it = prefetch_.begin(); it != prefetch_.end();) {
                        if (it->seg[0].op == op) {
                            urgent_.push_back(std::move(*it));
                            it = prefetch_.erase(it);
                        } else {
                            ++it;
                        }
                    }
                }
            }
            L.last_prefetch.clear();
        }
        for (auto it = prefetch_.begin(); it != prefetch_.end();) {
            const OpPtr &op = it->seg[0].op;
            if (!op || op->cancelled || op->promoted) it = prefetch_.erase(it);
            else ++it;
        }

        uint64_t protect[8];
        std::memcpy(protect, need, sizeof(protect));
        for (int i = 0; i < k; ++i) {
            const int e = (int)eids[i];
            if (e < 0 || e >= kExperts) continue;
            if (L.e2s[e] >= 0) {
                if (!L.snap || bm_has(L.snap_bm, e)) L.st.v[S_HITS]++;
                continue;
            }
            L.st.v[S_URGENT]++;
            int prev = -1;
            const int s = alloc(l, lk, protect, &prev);
            map_mru(L, e, s);
            OpPtr op = std::make_shared<Op>();
            op->layer = l;
            op->eid = e;
            op->slot = s;
            op->prev_eid = prev;
            op->total = L.nt;
            L.io[s] = op;
            urgent_ops.push_back(op);
        }
        L.snap = false;
        if (!urgent_ops.empty()) queue_urgent(l, L, urgent_ops, false);

        L.pending.clear();
        for (int i = 0; i < k; ++i) {
            const int s = L.e2s[(int)eids[i]];
            to_mru(L, s);
            if (L.slot_out) L.slot_out[i] = (uint32_t)s;
            if (out) out[i] = (uint32_t)s;
            L.pins[s]++;
            L.reader_pins.push_back((int16_t)s);
            if (L.io[s] && !L.io[s]->done) L.pending.push_back(L.io[s]);
        }
        if (!L.pending.empty() || !urgent_ops.empty()) work_cv_.notify_all();
        return (int)L.pending.size();
    }

    void wait_layer_urgent(int l) {
        if (!valid(l)) return;
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        if (L.pending.empty()) return;
        if (all_done(L.pending)) {
            L.pending.clear();
            return;
        }
        const auto t0 = std::chrono::steady_clock::now();
        const std::vector<OpPtr> wait_for = L.pending;
        while (!all_done(wait_for)) {
            if (!urgent_.empty()) {                     // help: run the next urgent copy here
                Task task = std::move(urgent_.front());
                urgent_.pop_front();
                if (mark_started(task)) {
                    lk.unlock();
                    execute(task);
                    lk.lock();
                    continue;
                }
            }
            done_cv_.wait(lk);
        }
        L.st.v[S_IO_WAIT_NS] += (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                    std::chrono::steady_clock::now() - t0).count();
        L.pending.clear();
    }

    void wait_layer_all(int l) {
        if (!valid(l)) return;
        wait_layer_urgent(l);
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        if (!L.init) return;
        for (;;) {
            bool busy = false;
            for (int s = 0; s < L.cap && !busy; ++s)
                busy = L.io[s] && !L.io[s]->done && !L.io[s]->cancelled;
            if (!busy) return;
            help_or_wait(lk);
        }
    }

    void wait_all() {
        for (int l = 0; l < kLayers; ++l) wait_layer_all(l);
    }

    void unpin_layer(int l) {
        if (!valid(l)) return;
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        if (L.reader_pins.empty()) return;
        for (int16_t s : L.reader_pins)
            if (s >= 0 && s < kExperts && L.pins[s] > 0) L.pins[s]--;
        L.reader_pins.clear();
        done_cv_.notify_all();
    }

    void pin(int l, const uint32_t *slots, int n, int delta) {
        if (!valid(l) || !slots || n <= 0) return;
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        for (int i = 0; i < n; ++i) {
            const uint32_t s = slots[i];
            if (s >= (uint32_t)kExperts) continue;
            if (delta > 0) L.pins[s]++;
            else if (L.pins[s] > 0) L.pins[s]--;
        }
        if (delta < 0) done_cv_.notify_all();
    }

    int pin_count(int l, int s) {
        if (!valid(l) || s < 0 || s >= kExperts) return 0;
        std::unique_lock<std::mutex> lk(mu_);
        return L_[l].pins[s];
    }

    int force_invalidate(int l, double rate) {
        if (!valid(l) || rate <= 0.0) return 0;
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        if (!L.init) return 0;
        std::uniform_real_distribution<double> u(0.0, 1.0);
        std::vector<int16_t> order, chosen;
        for (int16_t s = L.head; s >= 0; s = L.nxt[s]) order.push_back(s);
        for (int16_t s : order) {
            if (L.pins[s] > 0 || L.s2e[s] < 0) continue;
            if (rate >= 1.0 || u(rng_) < rate) chosen.push_back(s);
        }
        int dropped = 0;
        for (int16_t s : chosen) {
            if (L.pins[s] > 0 || L.s2e[s] < 0) continue;
            OpPtr active = L.io[s];
            if (active && !active->done && !active->cancelled) {
                if (active->prefetch && active->started == 0) {
                    active->resolved = true;
                    active->cancelled = true;
                    L.st.v[S_PF_CANCELLED]++;
                } else {
                    while (!active->done && !active->cancelled) help_or_wait(lk);
                }
            }
            if (L.pins[s] > 0 || L.s2e[s] < 0) continue;   // state may have moved while unlocked
            const int e = L.s2e[s];
            for (auto &op : L.last_prefetch)
                if (op && !op->resolved && op->slot == s) {
                    op->resolved = true;
                    L.st.v[S_PF_WASTED]++;
                }
            unlink(L, s);
            L.e2s[e] = -1;
            L.s2e[s] = -1;
            L.io[s].reset();
            bm_clear(L.snap_bm, e);
            scrub(L, s);
            L.free_stack.push_back(s);
            dropped++;
        }
        L.st.v[S_FORCED] += (uint64_t)dropped;
        return dropped;
    }

    void load_sync(int l, const int32_t *eids, const int32_t *slots, int n, bool prefill) {
        if (!valid(l) || n <= 0) return;
        wait_layer_all(l);
        {
            std::unique_lock<std::mutex> lk(mu_);
            Layer &L = L_[l];
            if (!L.init) return;
            if (prefill) L.st.v[S_PRE_BYTES] += (uint64_t)n * L.expert_bytes;
            std::vector<OpPtr> ops;
            ops.reserve(n);
            for (int i = 0; i < n; ++i) {
                OpPtr op = std::make_shared<Op>();
                op->layer = l;
                op->eid = eids[i];
                op->slot = slots[i];
                op->total = L.nt;
                L.io[op->slot] = op;
                ops.push_back(op);
            }
            queue_urgent(l, L, ops, prefill);
            L.pending = ops;
            work_cv_.notify_all();
        }
        wait_layer_urgent(l);
    }

    int lru_state(int l, int32_t *eids, int32_t *slots) {
        if (!valid(l)) return 0;
        wait_layer_all(l);
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        int n = 0;
        for (int16_t s = L.head; s >= 0; s = L.nxt[s]) {
            eids[n] = L.s2e[s];
            slots[n] = s;
            ++n;
        }
        return n;
    }

    void set_lru_state(int l, const int32_t *eids, const int32_t *slots, int n, uint64_t req, uint64_t hits,
                       uint64_t misses) {
        if (!valid(l)) return;
        wait_layer_all(l);
        std::unique_lock<std::mutex> lk(mu_);
        Layer &L = L_[l];
        L.st.v[S_PRE_REQ] += req;
        L.st.v[S_PRE_HITS] += hits;
        L.st.v[S_PRE_MISSES] += misses;
        clear_map(L, false);
        rebuild(L, eids, slots, n);
    }

    void stats(int l, uint64_t *out) {
        std::memset(out, 0, sizeof(uint64_t) * MOE_P1_STATS);
        if (!valid(l)) return;
        std::unique_lock<std::mutex> lk(mu_);
        std::memcpy(out, L_[l].st.v, sizeof(uint64_t) * MOE_P1_STATS);
        out[S_BYTES] = L_[l].bytes.load(std::memory_order_relaxed);
    }

    // sums layers 1..n-1 (layer 0 is the pinned layer in the reference's engine)
    void total_stats(int n, uint64_t *out) {
        std::memset(out, 0, sizeof(uint64_t) * MOE_P1_STATS);
        std::unique_lock<std::mutex> lk(mu_);
        for (int l = 1; l < std::min(n, kLayers); ++l) {
            const Layer &L = L_[l];
            if (!L.init) continue;
            for (int i = 0; i < MOE_P1_STATS; ++i)
                out[i] += (i == S_BYTES) ? L.bytes.load(std::memory_order_relaxed) : L.st.v[i];
        }
    }

    void seed(uint64_t s) {
        std::unique_lock<std::mutex> lk(mu_);
        rng_.seed(s);
    }

    int threads() const { return nthreads_; }

private:
    static bool valid(int l) { return l >= 0 && l < kLayers; }

    static bool all_done(const std::vector<OpPtr> &ops) {
        for (const auto &op : ops)
            if (op && !op->done) return false;
        return true;
    }

    // ---- LRU list over slots (head = least recent)
    static void unlink(Layer &L, int16_t s) {
        const int16_t p = L.prv[s], n = L.nxt[s];
        (p >= 0 ? L.nxt[p] : L.head) = n;
        (n >= 0 ? L.prv[n] : L.tail) = p;
        L.prv[s] = L.nxt[s] = -1;
    }
    static void push_tail(Layer &L, int16_t s) {
        L.prv[s] = L.tail;
        L.nxt[s] = -1;
        (L.tail >= 0 ? L.nxt[L.tail] : L.head) = s;
        L.tail = s;
    }
    static void push_head(Layer &L, int e, int16_t s) {
        L.e2s[e] = s;
        L.s2e[s] = (int16_t)e;
        L.prv[s] = -1;
        L.nxt[s] = L.head;
        (L.head >= 0 ? L.prv[L.head] : L.tail) = s;
        L.head = s;
    }
    static void to_mru(Layer &L, int16_t s) {
        if (L.tail == s) return;
        unlink(L, s);
        push_tail(L, s);
    }
    // maps e -> s at MRU; an expert already resident just moves to MRU
    static void map_mru(Layer &L, int e, int16_t s) {
        if (L.e2s[e] >= 0) {
            to_mru(L, L.e2s[e]);
            return;
        }
        L.e2s[e] = s;
        L.s2e[s] = (int16_t)e;
        push_tail(L, s);
    }

    static void clear_map(Layer &L, bool pins_too) {
        for (int i = 0; i < kExperts; ++i) {
            L.e2s[i] = L.s2e[i] = L.prv[i] = L.nxt[i] = -1;
            if (pins_too) L.pins[i] = 0;
            L.io[i].reset();
        }
        if (pins_too) L.reader_pins.clear();
        L.head = L.tail = -1;
        L.snap = false;
        std::memset(L.snap_bm, 0, sizeof(L.snap_bm));
        L.last_prefetch.clear();
        L.pending.clear();
    }
    static void fresh_free_stack(Layer &L) {
        L.free_stack.clear();
        for (int s = L.cap - 1; s >= 0; --s) L.free_stack.push_back((int16_t)s);
    }
    // inserts (eid, slot) pairs LRU -> MRU; unused slots go to the free stack, lowest on top
    static void rebuild(Layer &L, const int32_t *eids, const int32_t *slots, int n) {
        std::vector<uint8_t> used(kExperts, 0);
        for (int i = 0; i < n; ++i) {
            const int e = eids[i], s = slots[i];
            if (s < 0 || s >= L.cap || e < 0 || e >= kExperts) continue;
            used[s] = 1;
            map_mru(L, e, (int16_t)s);
        }
        L.free_stack.clear();
        for (int s = L.cap - 1; s >= 0; --s)
            if (!used[s]) L.free_stack.push_back((int16_t)s);
    }

    // an unstarted prefetch that is dropped hands its slot back: to the expert it displaced (as
    // least recent, if that expert is not resident elsewhere) or to the free stack
    static void give_back(Layer &L, const Op &op, bool mark_snapshot) {
        if (L.s2e[op.slot] != op.eid) return;
        unlink(L, (int16_t)op.slot);
        L.e2s[op.eid] = -1;
        L.s2e[op.slot] = -1;
        L.io[op.slot].reset();
        if (op.prev_eid >= 0 && op.prev_eid < kExperts && L.e2s[op.prev_eid] < 0) {
            push_head(L, op.prev_eid, (int16_t)op.slot);
            if (mark_snapshot) bm_set(L.snap_bm, op.prev_eid);
        } else {
            L.free_stack.push_back((int16_t)op.slot);
        }
    }

    static bool loading(const Layer &L, int16_t s) { return L.io[s] && !L.io[s]->done; }

    int16_t take_slot(Layer &L, int16_t s, int *prev) {
        const int e = L.s2e[s];
        unlink(L, s);
        if (e >= 0) L.e2s[e] = -1;
        L.s2e[s] = -1;
        L.io[s].reset();
        if (prev) *prev = e;
        return s;
    }

    int16_t alloc(int l, std::unique_lock<std::mutex> &lk, const uint64_t *protect, int *prev) {
        Layer &L = L_[l];
        if (!L.free_stack.empty()) {
            const int16_t s = L.free_stack.back();
            L.free_stack.pop_back();
            if (prev) *prev = -1;
            return s;
        }
        bool counted = false;
        for (;;) {
            bool blocked_pin = false, blocked_io = false;
            for (int16_t s = L.head; s >= 0; s = L.nxt[s]) {
                const int e = L.s2e[s];
                const bool prot = e >= 0 && bm_has(protect, e);
                if (prot) continue;
                if (L.pins[s] == 0 && !loading(L, s)) return take_slot(L, s, prev);
                blocked_pin |= L.pins[s] > 0;
                blocked_io |= loading(L, s);
            }
            if (!blocked_pin && !blocked_io)
                for (int16_t s = L.head; s >= 0; s = L.nxt[s]) {   // every slot protected
                    blocked_pin |= L.pins[s] > 0;
                    blocked_io |= loading(L, s);
                }
            if (blocked_pin) {
                if (!counted) {
                    L.st.v[S_PIN_WAITS]++;
                    counted = true;
                }
                if (reader_fn_) {
                    auto fn = reader_fn_;
                    void *user = reader_user_;
                    lk.unlock();
                    fn(user, l);
                    lk.lock();
                } else {
                    done_cv_.wait(lk);
                }
                continue;
            }
            if (blocked_io) {
                help_or_wait(lk);
                continue;
            }
            for (int16_t s = L.head; s >= 0; s = L.nxt[s])         // protected, but free to take
                if (L.pins[s] == 0 && !loading(L, s)) return take_slot(L, s, prev);
        }
    }

    // ---- copy tasks
    void queue_prefetch(int l, Layer &L, const OpPtr &op) {
        for (int pass = 0; pass < 2; ++pass)
            for (int t = 0; t < L.nt; ++t) {
                if ((L.rb[t] > kLargeRow) != (pass == 0)) continue;
                Task task;
                task.layer = l;
                task.nseg = 1;
                task.seg[0] = Seg{L.src[t] + (uint64_t)op->eid * L.rb[t], L.dst[t] + (uint64_t)op->slot * L.rb[t],
                                  (size_t)L.rb[t], op};
                prefetch_.push_back(std::move(task));
            }
    }

    // demand reads: runs of consecutive expert ids (at most kRun per task), one task per
    // (tensor, run), the large tensors of every run before the small ones
    void queue_urgent(int l, Layer &L, const std::vector<OpPtr> &ops, bool prefill) {
        if (ops.empty()) return;
        std::vector<OpPtr> by_eid = ops;
        std::sort(by_eid.begin(), by_eid.end(), [](const OpPtr &a, const OpPtr &b) { return a->eid < b->eid; });
        std::vector<std::pair<size_t, size_t>> runs;   // (first, count)
        size_t first = 0;
        for (size_t i = 1; i <= by_eid.size(); ++i) {
            const bool cut = i == by_eid.size() || by_eid[i]->eid != by_eid[i - 1]->eid + 1 || i - first >= (size_t)kRun;
            if (cut) {
                runs.emplace_back(first, i - first);
                first = i;
            }
        }
        for (int pass = 0; pass < 2; ++pass)
            for (int t = 0; t < L.nt; ++t) {
                if ((L.rb[t] > kLargeRow) != (pass == 0)) continue;
                for (const auto &r : runs) {
                    Task task;
                    task.layer = l;
                    task.prefill = prefill;
                    task.nseg = (int)r.second;
                    for (size_t j = 0; j < r.second; ++j) {
                        const OpPtr &op = by_eid[r.first + j];
                        task.seg[j] = Seg{L.src[t] + (uint64_t)op->eid * L.rb[t],
                                          L.dst[t] + (uint64_t)op->slot * L.rb[t], (size_t)L.rb[t], op};
                    }
                    urgent_.push_back(std::move(task));
                }
            }
    }

    static bool mark_started(Task &task) {
        bool any = false;
        for (int j = 0; j < task.nseg; ++j)
            if (task.seg[j].op && !task.seg[j].op->cancelled) {
                task.seg[j].op->started++;
                any = true;
            }
        return any;
    }

    // next task: URGENT first (tasks whose copies were all cancelled are dropped), then PREFETCH
    // (cancelled or promoted ones dropped)
    bool pop(Task &out) {
        while (!urgent_.empty()) {
            out = std::move(urgent_.front());
            urgent_.pop_front();
            if (mark_started(out)) return true;
        }
        while (!prefetch_.empty()) {
            out = std::move(prefetch_.front());
            prefetch_.pop_front();
            const OpPtr &op = out.seg[0].op;
            if (!op || op->cancelled || op->promoted) continue;
            op->started++;
            return true;
        }
        return false;
    }

    void help_or_wait(std::unique_lock<std::mutex> &lk) {
        Task task;
        if (pop(task)) {
            lk.unlock();
            execute(task);
            lk.lock();
        } else {
            done_cv_.wait(lk);
        }
    }

    void worker() {
        for (;;) {
            Task task;
            {
                std::unique_lock<std::mutex> lk(mu_);
                while (!stop_ && !pop(task)) work_cv_.wait(lk);
                if (stop_ && task.nseg == 0) return;
            }
            execute(task);
        }
    }

    // copies one task's rows (without the lock), then completes its operations
    void execute(Task &task) {
        const Layer &L = L_[task.layer];
        uint64_t moved = 0;
        bool failed = false;
        if (L.dst_dev && L.fd < 0) {
            moved = copy_rows_to_device(L, task, failed);   // all rows of the task, one sync
        } else {
            for (int j = 0; j < task.nseg; ++j) moved += copy_row(L, task.seg[j], failed);
        }
        if (!task.prefill && moved) L_[task.layer].bytes.fetch_add(moved, std::memory_order_relaxed);
        if (failed) copy_errors_.fetch_add(1, std::memory_order_relaxed);
        std::unique_lock<std::mutex> lk(mu_);
        bool any_done = false;
        for (int j = 0; j < task.nseg; ++j) {
            const OpPtr &op = task.seg[j].op;
            if (!op) continue;
            if (++op->completed >= op->total) {
                op->done = true;
                any_done = true;
            }
        }
        if (any_done) done_cv_.notify_all();
    }

    static uint64_t read_file(int fd, char *dst, size_t len, uint64_t off) {
        uint64_t got = 0;
        while (len > 0) {
            const ssize_t r = ::pread(fd, dst, len, (off_t)off);
            if (r <= 0) break;
            dst += r;
            len -= (size_t)r;
            off += (uint64_t)r;
            got += (uint64_t)r;
        }
        return got;
    }

    static cudaStream_t thread_stream(int dev) {
        if (tls_stream.s && tls_stream.dev == dev) return tls_stream.s;
        if (tls_stream.s) cudaStreamDestroy(tls_stream.s);
        tls_stream.s = nullptr;
        if (cudaSetDevice(dev) != cudaSuccess) return nullptr;
        if (cudaStreamCreateWithFlags(&tls_stream.s, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
        tls_stream.dev = dev;
        return tls_stream.s;
    }

    uint64_t copy_rows_to_device(const Layer &L, const Task &task, bool &failed) {
        cudaStream_t st = thread_stream(L.device);
        if (!st) {
            failed = true;
            return 0;
        }
        uint64_t moved = 0;
        for (int j = 0; j < task.nseg; ++j) {
            const Seg &sg = task.seg[j];
            if (cudaMemcpyAsync(sg.dst, reinterpret_cast<const void *>(static_cast<uintptr_t>(sg.src)), sg.len,
                                cudaMemcpyHostToDevice, st) != cudaSuccess) {
                failed = true;
                break;
            }
            moved += sg.len;
        }
        if (cudaStreamSynchronize(st) != cudaSuccess) failed = true;
        return failed ? 0 : moved;
    }

    uint64_t copy_row(const Layer &L, const Seg &sg, bool &failed) {
        if (!L.dst_dev) {
            if (L.fd >= 0) return read_file(L.fd, static_cast<char *>(sg.dst), sg.len, sg.src);
            std::memcpy(sg.dst, reinterpret_cast<const void *>(static_cast<uintptr_t>(sg.src)), sg.len);
            return sg.len;
        }
        cudaStream_t st = thread_stream(L.device);
        if (!st) {
            failed = true;
            return 0;
        }
        const void *src = reinterpret_cast<const void *>(static_cast<uintptr_t>(sg.src));
        std::vector<char> bounce;
        uint64_t got = sg.len;
        if (L.fd >= 0) {                                  // file rows go through host memory
            bounce.resize(sg.len);
            got = read_file(L.fd, bounce.data(), sg.len, sg.src);
            src = bounce.data();
        }
        if (cudaMemcpyAsync(sg.dst, src, got, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess) {
            failed = true;
            return 0;
        }
        return got;
    }

    void scrub(Layer &L, int16_t s) {
        if (!L.dst[0] || !L.rb[0]) return;
        const size_t n = (size_t)std::min<uint64_t>(64, L.rb[0]);
        char *p = L.dst[0] + (uint64_t)s * L.rb[0];
        if (L.dst_dev) {
            cudaStream_t st = thread_stream(L.device);
            if (st) {
                cudaMemsetAsync(p, 0xA5, n, st);
                cudaStreamSynchronize(st);
            }
        } else {
            std::memset(p, 0xA5, n);
        }
    }

    std::mutex mu_;
    std::condition_variable work_cv_, done_cv_;
    std::deque<Task> urgent_, prefetch_;
    Layer L_[kLayers];
    std::vector<std::thread> workers_;
    int nthreads_ = 6;
    bool running_ = false, stop_ = false;
    void (*reader_fn_)(void *, int) = nullptr;
    void *reader_user_ = nullptr;
    std::mt19937_64 rng_;

public:
    std::atomic<uint64_t> copy_errors_{0};
};

Scheduler *H(void *h) { return static_cast<Scheduler *>(h); }

}  // namespace

// ------------------------------------------------------------------ C ABI (include/moe_b200.h)

extern "C" void *moe_p1_create(void) { return new (std::nothrow) Scheduler(); }

extern "C" void moe_p1_destroy(void *h) { delete H(h); }

extern "C" int moe_p1_init(void *h, int num_threads) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_init: null handle");
    H(h)->init(num_threads);
    return MOE_OK;
}

extern "C" int moe_p1_shutdown(void *h) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_shutdown: null handle");
    H(h)->shutdown();
    return MOE_OK;
}

extern "C" int moe_p1_num_threads(void *h) { return h ? H(h)->threads() : 0; }

extern "C" int moe_p1_set_wait_reader_callback(void *h, void (*fn)(void *, int), void *user) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_set_wait_reader_callback: null handle");
    H(h)->set_reader_wait(fn, user);
    return MOE_OK;
}

extern "C" int moe_p1_layer_init(void *h, int layer, int fd, int capacity, int num_tensors,
                                 const uint64_t *base_offsets, const uint64_t *row_bytes, const uint64_t *base_ptrs,
                                 uint64_t slot_inds_ptr) {
    if (!h || !base_offsets || !row_bytes || !base_ptrs)
        return moe_set_error(MOE_EINVAL, "p1_layer_init: null pointer");
    H(h)->layer_init(layer, fd, capacity, num_tensors, base_offsets, row_bytes, base_ptrs, slot_inds_ptr, 0, 0);
    return MOE_OK;
}

extern "C" int moe_p1_layer_init_pool(void *h, int layer, int capacity, int num_tensors, const uint64_t *src_ptrs,
                                      const uint64_t *row_bytes, const uint64_t *slot_ptrs, uint64_t slot_inds_ptr,
                                      int slots_on_device, int device) {
    if (!h || !src_ptrs || !row_bytes || !slot_ptrs)
        return moe_set_error(MOE_EINVAL, "p1_layer_init_pool: null pointer");
    H(h)->layer_init(layer, -1, capacity, num_tensors, src_ptrs, row_bytes, slot_ptrs, slot_inds_ptr,
                     slots_on_device, device);
    return MOE_OK;
}

extern "C" int moe_p1_resize_layer(void *h, int layer, int new_capacity, const uint64_t *new_base_ptrs,
                                   uint64_t slot_inds_ptr, const int32_t *ordered_eids, const int32_t *ordered_slots,
                                   int count) {
    if (!h || !new_base_ptrs || (count > 0 && (!ordered_eids || !ordered_slots)))
        return moe_set_error(MOE_EINVAL, "p1_resize_layer: null pointer");
    H(h)->resize_layer(layer, new_capacity, new_base_ptrs, slot_inds_ptr, ordered_eids, ordered_slots, count);
    return MOE_OK;
}

extern "C" int moe_p1_reset_cache(void *h, int layer) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_reset_cache: null handle");
    H(h)->reset_cache(layer);
    return MOE_OK;
}

extern "C" int moe_p1_reset_stats(void *h, int layer) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_reset_stats: null handle");
    H(h)->reset_stats(layer);
    return MOE_OK;
}

extern "C" int moe_p1_start_prefetch(void *h, int layer, const int32_t *pred_eids, int pred_count, int max_fetch) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_start_prefetch: null handle");
    H(h)->start_prefetch(layer, pred_eids, pred_count, max_fetch);
    return MOE_OK;
}

extern "C" int moe_p1_step_decode(void *h, int layer, const uint32_t *eids, int k, uint32_t *out_slots) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_step_decode: null handle");
    for (int i = 0; eids && i < k; ++i)
        if (eids[i] >= (uint32_t)kExperts) return moe_set_error(MOE_EINVAL, "p1_step_decode: eid %u out of range", eids[i]);
    return H(h)->step_decode(layer, eids, k, out_slots);
}

extern "C" int moe_p1_wait_layer_urgent(void *h, int layer) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_wait_layer_urgent: null handle");
    H(h)->wait_layer_urgent(layer);
    return MOE_OK;
}

extern "C" int moe_p1_wait_layer_all(void *h, int layer) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_wait_layer_all: null handle");
    H(h)->wait_layer_all(layer);
    return MOE_OK;
}

extern "C" int moe_p1_wait_all(void *h) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_wait_all: null handle");
    H(h)->wait_all();
    return MOE_OK;
}

extern "C" int moe_p1_unpin_layer_slots(void *h, int layer) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_unpin_layer_slots: null handle");
    H(h)->unpin_layer(layer);
    return MOE_OK;
}

extern "C" int moe_p1_pin_slots(void *h, int layer, const uint32_t *slots, int count) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_pin_slots: null handle");
    H(h)->pin(layer, slots, count, +1);
    return MOE_OK;
}

extern "C" int moe_p1_unpin_slots(void *h, int layer, const uint32_t *slots, int count) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_unpin_slots: null handle");
    H(h)->pin(layer, slots, count, -1);
    return MOE_OK;
}

extern "C" int moe_p1_get_slot_pin_count(void *h, int layer, int slot) { return h ? H(h)->pin_count(layer, slot) : 0; }

extern "C" int moe_p1_seed(void *h, uint64_t seed) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_seed: null handle");
    H(h)->seed(seed);
    return MOE_OK;
}

extern "C" int moe_p1_force_invalidate(void *h, int layer, double rate) {
    if (!h) return moe_set_error(MOE_EINVAL, "p1_force_invalidate: null handle");
    return H(h)->force_invalidate(layer, rate);
}

extern "C" int moe_p1_load_sync(void *h, int layer, const int32_t *eids, const int32_t *slots, int count,
                                int is_prefill) {
    if (!h || (count > 0 && (!eids || !slots))) return moe_set_error(MOE_EINVAL, "p1_load_sync: null pointer");
    for (int i = 0; i < count; ++i)
        if (eids[i] < 0 || eids[i] >= kExperts || slots[i] < 0 || slots[i] >= kExperts)
            return moe_set_error(MOE_EINVAL, "p1_load_sync: eid %d / slot %d out of range", eids[i], slots[i]);
    H(h)->load_sync(layer, eids, slots, count, is_prefill != 0);
    return MOE_OK;
}

extern "C" int moe_p1_get_lru_state(void *h, int layer, int32_t *out_eids, int32_t *out_slots, int *out_count) {
    if (!h || !out_eids || !out_slots || !out_count) return moe_set_error(MOE_EINVAL, "p1_get_lru_state: null pointer");
    *out_count = H(h)->lru_state(layer, out_eids, out_slots);
    return MOE_OK;
}

extern "C" int moe_p1_set_lru_state(void *h, int layer, const int32_t *ordered_eids, const int32_t *ordered_slots,
                                    int count, uint64_t add_prefill_requests, uint64_t add_prefill_hits,
                                    uint64_t add_prefill_misses) {
    if (!h || (count > 0 && (!ordered_eids || !ordered_slots)))
        return moe_set_error(MOE_EINVAL, "p1_set_lru_state: null pointer");
    H(h)->set_lru_state(layer, ordered_eids, ordered_slots, count, add_prefill_requests, add_prefill_hits,
                        add_prefill_misses);
    return MOE_OK;
}

extern "C" int moe_p1_get_layer_stats(void *h, int layer, uint64_t *out) {
    if (!h || !out) return moe_set_error(MOE_EINVAL, "p1_get_layer_stats: null pointer");
    H(h)->stats(layer, out);
    return MOE_OK;
}

extern "C" int moe_p1_get_total_stats(void *h, int num_layers, uint64_t *out) {
    if (!h || !out) return moe_set_error(MOE_EINVAL, "p1_get_total_stats: null pointer");
    H(h)->total_stats(num_layers, out);
    return MOE_OK;
}

extern "C" uint64_t moe_p1_copy_errors(void *h) {
    return h ? H(h)->copy_errors_.load(std::memory_order_relaxed) : 0;
}
