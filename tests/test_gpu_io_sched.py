"""P1 I/O scheduler with device slot buffers: expert rows copied from a pinned host pool into
slot buffers in HBM by the scheduler's copy kernel (the rows its control kernel took from the
queues). The decisions are compared with the reference scheduler (mlx-qwen38/cpp/src/
io_sched.cpp, file -> host buffers) on identical calls; the device bytes are read back and
compared with the pool."""
import ctypes
import os
import random

import numpy as np
import pytest
import torch

from moe_offload_b200.io_sched import P1IoScheduler

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libref_iosched.so")
ROW_BYTES = [131072, 256, 256, 1024, 256, 256, 1024, 256, 256]
NT = len(ROW_BYTES)
N_EXPERTS = 32
LAYERS = [1, 2]


def _row(layer, eid, t):
    rng = np.random.default_rng((layer * 1000 + eid) * 16 + t + 7)
    return rng.integers(0, 256, ROW_BYTES[t], dtype=np.uint8)


@pytest.fixture(scope="module")
def pool():
    """Pinned host pool per (layer, tensor): [N_EXPERTS, row] rows, and the same rows in a file."""
    import tempfile
    d = tempfile.mkdtemp()
    path = os.path.join(d, "experts.bin")
    host, offsets = {}, {}
    off = 0
    with open(path, "wb") as f:
        for l in LAYERS:
            host[l], offsets[l] = [], []
            for t, rb in enumerate(ROW_BYTES):
                rows = np.stack([_row(l, e, t) for e in range(N_EXPERTS)])
                pt = torch.from_numpy(rows).pin_memory()
                host[l].append(pt)
                offsets[l].append(off)
                f.write(rows.tobytes())
                off += N_EXPERTS * rb
    fd = os.open(path, os.O_RDONLY)
    yield host, fd, offsets
    os.close(fd)


class DevSlots:
    def __init__(self, cap, dev):
        self.cap = cap
        self.bufs = [torch.full((cap * rb,), 0xCD, dtype=torch.uint8, device=dev) for rb in ROW_BYTES]
        self.slot_inds = np.zeros(16, dtype=np.uint32)

    def ptrs(self):
        return [b.data_ptr() for b in self.bufs]

    def verify(self, layer, eid, slot):
        for t, rb in enumerate(ROW_BYTES):
            got = self.bufs[t][slot * rb:(slot + 1) * rb].cpu().numpy()
            assert np.array_equal(got, _row(layer, eid, t)), f"layer {layer} eid {eid} slot {slot} tensor {t}"


class HostSlots:
    def __init__(self, cap):
        self.cap = cap
        self.bufs = [np.full(cap * rb, 0xCD, dtype=np.uint8) for rb in ROW_BYTES]
        self.slot_inds = np.zeros(16, dtype=np.uint32)

    def ptrs(self):
        return [b.ctypes.data for b in self.bufs]


def test_device_slots_match_reference_decisions(pool):
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_iosched.so not built")
    host, fd, offsets = pool
    dev = torch.device("cuda", 0)
    ours, ref = P1IoScheduler(), P1IoScheduler(ctypes.CDLL(REF_LIB), prefix="ref_p1_")   # no workers
    rng = random.Random(5)
    caps = {l: rng.randint(6, 10) for l in LAYERS}
    dbufs = {l: DevSlots(caps[l], dev) for l in LAYERS}
    hbufs = {l: HostSlots(caps[l]) for l in LAYERS}
    for l in LAYERS:
        ours.layer_init_pool(l, caps[l], [p.data_ptr() for p in host[l]], ROW_BYTES, dbufs[l].ptrs(),
                             dbufs[l].slot_inds.ctypes.data, on_device=True, device=0,
                             num_experts=N_EXPERTS)
        ref.layer_init(l, fd, caps[l], NT, offsets[l], ROW_BYTES, hbufs[l].ptrs(), hbufs[l].slot_inds.ctypes.data)
    for s in (ours, ref):
        s.seed(17)
        s.set_wait_reader_callback(lambda layer, s=s: s.unpin_layer_slots(layer))
    for step in range(300):
        l = rng.choice(LAYERS)
        op = rng.random()
        if op < 0.35:
            preds = rng.sample(range(N_EXPERTS), rng.randint(1, 8))
            mf = rng.randint(1, 4)
            ours.start_prefetch(l, preds, mf)
            ref.start_prefetch(l, preds, mf)
        elif op < 0.75:
            eids = rng.sample(range(N_EXPERTS), rng.randint(2, 4))
            a, b = ours.step_decode(l, eids), ref.step_decode(l, eids)
            assert a == b, f"step {step}: {a} vs {b}"
            ours.wait_layer_urgent(l)
            ref.wait_layer_urgent(l)
            for e, sl in zip(eids, a[1]):
                dbufs[l].verify(l, e, sl)
        elif op < 0.85:
            ours.unpin_layer_slots(l)
            ref.unpin_layer_slots(l)
        elif op < 0.9:
            assert ours.force_invalidate(l, 0.5) == ref.force_invalidate(l, 0.5)
        else:
            a, b = ours.get_lru_state(l), ref.get_lru_state(l)
            assert a == b
            for e, sl in zip(*a):
                dbufs[l].verify(l, e, sl)
    for l in LAYERS:
        a = {k: v for k, v in ours.get_layer_stats(l).items() if k != "io_wait_ns"}
        b = {k: v for k, v in ref.get_layer_stats(l).items() if k != "io_wait_ns"}
        assert a == b
    assert ours.copy_errors() == 0
    ours.close()
    ref.close()


def test_device_slots_threaded(pool):
    """Eight copy workers filling device slots while prefetches are cancelled and promoted."""
    host, _, _ = pool
    dev = torch.device("cuda", 0)
    s = P1IoScheduler()
    s.init(8)
    s.seed(3)
    cap, k = 10, 4
    bufs = {l: DevSlots(cap, dev) for l in LAYERS}
    for l in LAYERS:
        s.layer_init_pool(l, cap, [p.data_ptr() for p in host[l]], ROW_BYTES, bufs[l].ptrs(),
                          bufs[l].slot_inds.ctypes.data, on_device=True, device=0, num_experts=N_EXPERTS)
    s.set_wait_reader_callback(lambda layer: s.unpin_layer_slots(layer))
    rng = random.Random(11)
    for step in range(120):
        for l in LAYERS:
            s.unpin_layer_slots(l)
            if step % 4 == 3:
                s.force_invalidate(l, 0.3)
            eids = rng.sample(range(N_EXPERTS), k)
            n, slots = s.step_decode(l, eids)
            if n:
                s.wait_layer_urgent(l)
            for e, sl in zip(eids, slots):
                bufs[l].verify(l, e, sl)
            if l + 1 in LAYERS:                 # consumed by the next layer's step_decode
                s.start_prefetch(l + 1, rng.sample(range(N_EXPERTS), 6), 3)
    s.wait_all()
    tot = s.get_total_stats(max(LAYERS) + 1)
    assert tot["decode_requests"] == 120 * len(LAYERS) * k
    assert tot["prefetch_cancelled"] + tot["prefetch_wasted"] + tot["prefetch_used"] == tot["prefetch_issued"]
    assert tot["bytes"] > 0 and s.copy_errors() == 0
    s.close()
