// Test infrastructure only (the checker, never the product): a C entry point per method of the
// reference's P1 I/O scheduler, qwen38::P1IoScheduler (mlx-qwen38/cpp/src/io_sched.h:46-245),
// compiled together with the unmodified reference source mlx-qwen38/cpp/src/io_sched.cpp into
// oracle/_ref/libref_iosched.so (oracle/Makefile). The functions have the signatures of the
// library's moe_p1_* functions (include/moe_b200.h) with the prefix ref_p1_, so the parity
// tests drive both with the same calls. Rows come from a file (the reference's only source).
#include <cstdint>
#include <cstring>
#include <random>

#include "io_sched.h"

namespace {
struct RefHandle {
    qwen38::P1IoScheduler sched;
    std::mt19937_64 rng;
    void (*fn)(void *, int) = nullptr;
    void *user = nullptr;
};
RefHandle *R(void *h) { return static_cast<RefHandle *>(h); }

void stats_out(const qwen38::P1LayerStats &s, uint64_t *o) {
    const uint64_t v[16] = {s.decode_requests, s.lru_hits, s.urgent_reads, s.prefetch_issued,
                            s.prefetch_cancelled, s.prefetch_promoted, s.prefetch_used, s.prefetch_wasted,
                            s.pin_waits, s.bytes, s.io_wait_ns, s.forced_invalidations,
                            s.prefill_requests, s.prefill_lru_hits, s.prefill_demand_misses, s.prefill_demand_bytes};
    std::memcpy(o, v, sizeof(v));
}
}  // namespace

extern "C" {
void *ref_p1_create(void) { return new RefHandle(); }
void ref_p1_destroy(void *h) { delete R(h); }
int ref_p1_init(void *h, int n) { R(h)->sched.init(n); return 0; }
int ref_p1_shutdown(void *h) { R(h)->sched.shutdown(); return 0; }
int ref_p1_num_threads(void *h) { return R(h)->sched.num_threads(); }
int ref_p1_set_wait_reader_callback(void *h, void (*fn)(void *, int), void *user) {
    RefHandle *r = R(h);
    r->fn = fn;
    r->user = user;
    if (fn) r->sched.set_wait_reader_callback([r](int l) { r->fn(r->user, l); });
    else r->sched.set_wait_reader_callback(nullptr);
    return 0;
}
int ref_p1_layer_init(void *h, int l, int fd, int cap, int nt, const uint64_t *off, const uint64_t *rb,
                      const uint64_t *ptrs, uint64_t slot_inds) {
    R(h)->sched.layer_init(l, fd, cap, nt, off, rb, ptrs, slot_inds);
    return 0;
}
int ref_p1_resize_layer(void *h, int l, int cap, const uint64_t *ptrs, uint64_t slot_inds, const int32_t *eids,
                        const int32_t *slots, int n) {
    R(h)->sched.resize_layer(l, cap, ptrs, slot_inds, eids, slots, n);
    return 0;
}
int ref_p1_reset_cache(void *h, int l) { R(h)->sched.reset_cache(l); return 0; }
int ref_p1_reset_stats(void *h, int l) { R(h)->sched.reset_stats(l); return 0; }
int ref_p1_start_prefetch(void *h, int l, const int32_t *pred, int n, int max_fetch) {
    R(h)->sched.start_prefetch(l, pred, n, max_fetch);
    return 0;
}
int ref_p1_step_decode(void *h, int l, const uint32_t *eids, int k, uint32_t *out) {
    return R(h)->sched.step_decode(l, eids, k, out);
}
int ref_p1_wait_layer_urgent(void *h, int l) { R(h)->sched.wait_layer_urgent(l); return 0; }
int ref_p1_wait_layer_all(void *h, int l) { R(h)->sched.wait_layer_all(l); return 0; }
int ref_p1_wait_all(void *h) { R(h)->sched.wait_all(); return 0; }
int ref_p1_unpin_layer_slots(void *h, int l) { R(h)->sched.unpin_layer_slots(l); return 0; }
int ref_p1_pin_slots(void *h, int l, const uint32_t *s, int n) { R(h)->sched.pin_slots(l, s, n); return 0; }
int ref_p1_unpin_slots(void *h, int l, const uint32_t *s, int n) { R(h)->sched.unpin_slots(l, s, n); return 0; }
int ref_p1_get_slot_pin_count(void *h, int l, int s) { return R(h)->sched.get_slot_pin_count(l, s); }
int ref_p1_seed(void *h, uint64_t seed) { R(h)->rng.seed(seed); return 0; }
int ref_p1_force_invalidate(void *h, int l, double rate) { return R(h)->sched.force_invalidate(l, rate, R(h)->rng); }
int ref_p1_load_sync(void *h, int l, const int32_t *eids, const int32_t *slots, int n, int prefill) {
    R(h)->sched.load_sync(l, eids, slots, n, prefill != 0);
    return 0;
}
int ref_p1_get_lru_state(void *h, int l, int32_t *eids, int32_t *slots, int *n) {
    R(h)->sched.get_lru_state(l, eids, slots, n);
    return 0;
}
int ref_p1_set_lru_state(void *h, int l, const int32_t *eids, const int32_t *slots, int n, uint64_t a, uint64_t b,
                         uint64_t c) {
    R(h)->sched.set_lru_state(l, eids, slots, n, a, b, c);
    return 0;
}
int ref_p1_get_layer_stats(void *h, int l, uint64_t *o) { stats_out(R(h)->sched.get_layer_stats(l), o); return 0; }
int ref_p1_get_total_stats(void *h, int n, uint64_t *o) { stats_out(R(h)->sched.get_total_stats(n), o); return 0; }
}
