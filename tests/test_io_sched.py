"""P1 I/O scheduler (moe_offload_b200.io_sched; state and decisions on the GPU, csrc/p1_device.cu)
against the reference's own scheduler (mlx-qwen38/cpp/src/io_sched.cpp, built into
oracle/_ref/libref_iosched.so by oracle/Makefile). Rows are read from a synthetic expert file
into host slot buffers. The reference's runs of its own scenarios need no GPU; every run of
ours is marked gpu (its scheduler state lives in device memory).

The first three tests restate the scenarios of the reference's test_io_sched.cpp:142-445
(queued cancel + promote with exact counters, pin waits through the reader callback, a
multi-threaded stress run with resizes and forced invalidation). The differential test runs
identical random call sequences through both schedulers with no worker threads (then both are
deterministic) and requires the same slots, pending counts, LRU orders, statistics and slot
bytes after every call."""
import ctypes
import os
import random
import threading
import time

import numpy as np
import pytest

from moe_offload_b200.io_sched import P1IoScheduler

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libref_iosched.so")

N_LAYERS = 4           # layers 1..4
N_EXPERTS = 32
# one tensor above the reference's 100,000-byte threshold, so copies are ordered large-first
ROW_BYTES = [131072, 256, 256, 1024, 256, 256, 1024, 256, 256]
NT = len(ROW_BYTES)


def _row(layer, eid, t):
    rng = np.random.default_rng((layer * 1000 + eid) * 16 + t)
    return rng.integers(0, 256, ROW_BYTES[t], dtype=np.uint8)


@pytest.fixture(scope="module")
def expert_file(tmp_path_factory):
    path = tmp_path_factory.mktemp("p1") / "experts.bin"
    offsets = {}
    off = 0
    with open(path, "wb") as f:
        for l in range(1, N_LAYERS + 1):
            offsets[l] = []
            for t in range(NT):
                offsets[l].append(off)
                for e in range(N_EXPERTS):
                    f.write(_row(l, e, t).tobytes())
                off += N_EXPERTS * ROW_BYTES[t]
    fd = os.open(path, os.O_RDONLY)
    yield fd, offsets
    os.close(fd)


@pytest.fixture(scope="module")
def ref_lib():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_iosched.so not built (needs the reference sources)")
    return ctypes.CDLL(REF_LIB)


def _impls(ref_lib):
    return [("ours", lambda: P1IoScheduler()), ("reference", lambda: P1IoScheduler(ref_lib, prefix="ref_p1_"))]


class Slots:
    """Host slot buffers of one layer (one array per tensor) and its slot-id output array."""

    def __init__(self, cap, k_max=16):
        self.cap = cap
        self.bufs = [np.full(cap * rb, 0xCD, dtype=np.uint8) for rb in ROW_BYTES]
        self.slot_inds = np.zeros(k_max, dtype=np.uint32)

    def ptrs(self):
        return [b.ctypes.data for b in self.bufs]

    def inds_ptr(self):
        return self.slot_inds.ctypes.data

    def verify(self, layer, eid, slot):
        assert 0 <= slot < self.cap
        for t, rb in enumerate(ROW_BYTES):
            got = self.bufs[t][slot * rb:(slot + 1) * rb]
            assert np.array_equal(got, _row(layer, eid, t)), f"layer {layer} eid {eid} slot {slot} tensor {t}"


def _init_layer(s, fd, offsets, layer, slots):
    s.layer_init(layer, fd, slots.cap, NT, offsets[layer], ROW_BYTES, slots.ptrs(), slots.inds_ptr())


@pytest.mark.parametrize("which", [pytest.param("ours", marks=pytest.mark.gpu), "reference"])
def test_cancel_and_promote(expert_file, ref_lib, which):
    fd, offsets = expert_file
    s = dict(_impls(ref_lib))[which]()
    # no init(): no worker threads, so the prefetches stay queued until step_decode (the
    # reference's test calls init(0), which its clamp turns into one worker: a race it wins
    # almost always)
    buf = Slots(4)
    _init_layer(s, fd, offsets, 1, buf)
    s.load_sync(1, [0, 1, 2, 3], [0, 1, 2, 3], True)
    s.set_lru_state(1, [0, 1, 2, 3], [0, 1, 2, 3], 4, 0, 4)
    s.unpin_layer_slots(1)
    for e in range(4):
        buf.verify(1, e, e)
    s.start_prefetch(1, [10, 11, 12], 3)
    n, slots = s.step_decode(1, [0, 10, 20, 21])
    assert n > 0
    s.wait_layer_urgent(1)
    for e, sl in zip([0, 10, 20, 21], slots):
        buf.verify(1, e, sl)
    assert list(buf.slot_inds[:4]) == slots
    s.unpin_layer_slots(1)
    st = s.get_layer_stats(1)
    assert (st["prefetch_issued"], st["prefetch_cancelled"], st["prefetch_promoted"], st["prefetch_used"],
            st["urgent_reads"]) == (3, 2, 1, 1, 2)
    s.close()


@pytest.mark.parametrize("which", [pytest.param("ours", marks=pytest.mark.gpu), "reference"])
def test_pin_waits_and_reader_callback(expert_file, ref_lib, which):
    fd, offsets = expert_file
    s = dict(_impls(ref_lib))[which]()
    s.init(4)
    buf = Slots(6)
    _init_layer(s, fd, offsets, 1, buf)
    s.load_sync(1, list(range(6)), list(range(6)), True)
    s.set_lru_state(1, list(range(6)), list(range(6)), 6, 0, 6)
    done = threading.Event()
    reader = {}

    def wait_reader(layer):
        if "t" in reader:
            reader["t"].join()
        assert done.is_set()
        s.unpin_layer_slots(layer)

    s.set_wait_reader_callback(wait_reader)
    eids = [0, 1, 2, 3]
    n, slots = s.step_decode(1, eids)
    if n > 0:
        s.wait_layer_urgent(1)

    def gpu():
        time.sleep(0.015)
        for e, sl in zip(eids, slots):
            buf.verify(1, e, sl)
        done.set()

    reader["t"] = threading.Thread(target=gpu)
    reader["t"].start()
    # four slots stay pinned by the reader, two are free: the third prefetch must wait for it
    s.start_prefetch(1, [10, 11, 12], 3)
    s.wait_layer_all(1)
    assert s.get_layer_stats(1)["pin_waits"] >= 1
    assert done.is_set()
    s.close()


@pytest.mark.parametrize("which", [pytest.param("ours", marks=pytest.mark.gpu), "reference"])
def test_high_concurrency_stress(expert_file, ref_lib, which):
    fd, offsets = expert_file
    cap0, k, m, pcap, steps = 12, 4, 6, 3, 250
    s = dict(_impls(ref_lib))[which]()
    s.init(8)
    s.seed(123456789)
    bufs = {}
    for l in range(1, N_LAYERS + 1):
        bufs[l] = Slots(cap0)
        _init_layer(s, fd, offsets, l, bufs[l])
        s.load_sync(l, list(range(cap0)), list(range(cap0)), True)
        s.set_lru_state(l, list(range(cap0)), list(range(cap0)), cap0, 0, cap0)
    readers = {l: None for l in bufs}
    locks = {l: threading.Lock() for l in bufs}
    errors = []

    def wait_reader(l):
        with locks[l]:
            t, readers[l] = readers[l], None
        if t is not None:
            t.join()
        s.unpin_layer_slots(l)

    s.set_wait_reader_callback(wait_reader)
    rng = random.Random(7)
    verified = 0
    for step in range(steps):
        if step in (100, 160):
            new_cap = 8 if step == 100 else 14
            for l in bufs:
                wait_reader(l)
                s.wait_layer_all(l)
                le, ls = s.get_lru_state(l)
                keep = min(len(le), new_cap)
                nb = Slots(new_cap)
                for i in range(keep):
                    old = ls[len(le) - keep + i]
                    for t, rb in enumerate(ROW_BYTES):
                        nb.bufs[t][i * rb:(i + 1) * rb] = bufs[l].bufs[t][old * rb:(old + 1) * rb]
                bufs[l] = nb
                s.resize_layer(l, new_cap, nb.ptrs(), nb.inds_ptr(), le[len(le) - keep:], list(range(keep)))
        for l in bufs:
            eids = rng.sample(range(N_EXPERTS), k)
            pred = rng.sample(range(N_EXPERTS), m)
            wait_reader(l)
            if step % 3 == 1:
                s.force_invalidate(l, 0.30)
            n, slots = s.step_decode(l, eids)
            if n > 0:
                s.wait_layer_urgent(l)
            buf = bufs[l]

            def gpu(l=l, eids=eids, slots=slots, buf=buf):
                try:
                    for e, sl in zip(eids, slots):
                        buf.verify(l, e, sl)
                except AssertionError as exc:       # reported by the main thread
                    errors.append(str(exc))

            t = threading.Thread(target=gpu)
            with locks[l]:
                readers[l] = t
            t.start()
            verified += k
            if l + 1 in bufs:
                s.start_prefetch(l + 1, pred, pcap)
    for l in bufs:
        wait_reader(l)
    s.wait_all()
    assert not errors, errors[:3]
    tot = s.get_total_stats(N_LAYERS + 1)
    assert tot["decode_requests"] == steps * N_LAYERS * k
    assert tot["urgent_reads"] > 0 and tot["prefetch_issued"] > 0
    assert tot["prefetch_cancelled"] + tot["prefetch_wasted"] + tot["prefetch_used"] == tot["prefetch_issued"]
    assert tot["forced_invalidations"] > 0 and tot["bytes"] > 0
    s.close()


def _cmp_stats(a, b, where):
    a = {k: v for k, v in a.items() if k != "io_wait_ns"}
    b = {k: v for k, v in b.items() if k != "io_wait_ns"}
    assert a == b, f"{where}: {a} vs {b}"


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [1, 2, 3, 4, 5, 6])
def test_differential_against_reference(expert_file, ref_lib, seed):
    """Same random calls, no workers: every observable result equal to the reference's."""
    fd, offsets = expert_file
    rng = random.Random(seed)
    layers = [1, 2, 3]
    caps = {l: rng.randint(6, 12) for l in layers}
    sides = []
    for name, make in _impls(ref_lib):
        s = make()                  # no init(): no workers, both schedulers deterministic
        s.seed(99 + seed)
        bufs = {l: Slots(caps[l]) for l in layers}
        for l in layers:
            _init_layer(s, fd, offsets, l, bufs[l])
        s.set_wait_reader_callback(lambda layer, s=s: s.unpin_layer_slots(layer))
        sides.append((name, s, bufs))

    def both(fn):
        return [fn(s, bufs) for _, s, bufs in sides]

    for step in range(600):
        l = rng.choice(layers)
        op = rng.random()
        if op < 0.30:
            preds = rng.sample(range(N_EXPERTS), rng.randint(1, 8))
            if rng.random() < 0.1:
                preds.insert(rng.randrange(len(preds) + 1), -1)     # skipped by both
            mf = rng.randint(1, 4)
            both(lambda s, b: s.start_prefetch(l, preds, mf))
        elif op < 0.65:
            eids = rng.sample(range(N_EXPERTS), rng.randint(2, 4))
            out = both(lambda s, b: s.step_decode(l, eids))
            assert out[0] == out[1], f"step {step} layer {l} eids {eids}: {out}"
            assert np.array_equal(sides[0][2][l].slot_inds[:len(eids)], sides[1][2][l].slot_inds[:len(eids)])
            if rng.random() < 0.8:
                both(lambda s, b: s.wait_layer_urgent(l))
                for _, s, bufs in sides:
                    for e, sl in zip(eids, out[0][1]):
                        bufs[l].verify(l, e, sl)
        elif op < 0.75:
            both(lambda s, b: s.unpin_layer_slots(l))
        elif op < 0.80:
            rate = rng.choice([0.2, 0.5, 1.0])
            out = both(lambda s, b: s.force_invalidate(l, rate))
            assert out[0] == out[1], f"step {step}: force_invalidate {out}"
        elif op < 0.88:
            out = both(lambda s, b: s.get_lru_state(l))
            assert out[0] == out[1], f"step {step} layer {l}: LRU {out}"
            for _, s, bufs in sides:
                for e, sl in zip(*out[0]):
                    bufs[l].verify(l, e, sl)
        elif op < 0.95:
            out = both(lambda s, b: s.get_layer_stats(l))
            _cmp_stats(out[0], out[1], f"step {step} layer {l}")
        elif op < 0.96:
            # resize to a new capacity, keeping the most recent experts in slots 0.. of new buffers
            new_cap = rng.randint(6, 12)
            both(lambda s, b: s.wait_layer_all(l))
            le, ls = both(lambda s, b: s.get_lru_state(l))[0]
            keep = min(len(le), new_cap)
            for _, s, bufs in sides:
                nb = Slots(new_cap)
                for i in range(keep):
                    old = ls[len(le) - keep + i]
                    for t, rb in enumerate(ROW_BYTES):
                        nb.bufs[t][i * rb:(i + 1) * rb] = bufs[l].bufs[t][old * rb:(old + 1) * rb]
                bufs[l] = nb
                s.resize_layer(l, new_cap, nb.ptrs(), nb.inds_ptr(), le[len(le) - keep:], list(range(keep)))
        elif op < 0.98:
            # a prefill-style synchronous load of two non-resident experts into the two least
            # recent slots, then the rebuilt LRU order
            le, ls = both(lambda s, b: s.get_lru_state(l))[0]
            if len(le) >= 2:
                fresh = [e for e in rng.sample(range(N_EXPERTS), N_EXPERTS) if e not in le][:2]
                slots2 = ls[:2]
                both(lambda s, b: s.load_sync(l, fresh, slots2, True))
                order_e, order_s = le[2:] + fresh, ls[2:] + slots2
                both(lambda s, b: s.set_lru_state(l, order_e, order_s, 2, 1, 1))
                for _, s, bufs in sides:
                    for e, sl in zip(fresh, slots2):
                        bufs[l].verify(l, e, sl)
        else:
            both(lambda s, b: s.reset_cache(l))
    for l in layers:
        both(lambda s, b: s.wait_layer_all(l))
        out = both(lambda s, b: s.get_layer_stats(l))
        _cmp_stats(out[0], out[1], f"final layer {l}")
        out = both(lambda s, b: s.get_lru_state(l))
        assert out[0] == out[1], f"final layer {l}: LRU {out}"
    tot = both(lambda s, b: s.get_total_stats(N_LAYERS + 1))
    _cmp_stats(tot[0], tot[1], "totals")
    assert tot[0]["decode_requests"] > 0 and tot[0]["prefetch_issued"] > 0
    for _, s, _ in sides:
        s.close()


@pytest.mark.gpu
def test_step_decode_rejects_bad_expert_ids():
    from moe_offload_b200._lib import MoeError
    s = P1IoScheduler()
    s.init(0)
    assert s.num_threads() == 1                 # the reference's clamp
    with pytest.raises(MoeError):
        s.step_decode(1, [3, 600])
    s.close()
