"""The GPU-resident LRU expert-slot cache against the reference's own cache (expert_io.c):
bit-exact hit/miss counts, slot ids, counters and LRU order. The drop-in C ABI replays the
committed reference trace and runs side by side with the reference library; the device API
(moe_lru_*, indices on the device) replays the same trace; fills and the cached layer's
outputs are checked against the pool and the resident path."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libexpert_io_ref.so")
u64 = ctypes.c_uint64


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def lib(dev):
    from moe_offload_b200 import _lib
    return _lib.load()


def _replay_dropin(L, lru_trace, layer_base):
    """Runs the trace's call sequence (tests/golden/make_golden.py) through the c_* ABI."""
    E, K, M, CAP, PCAP, NL, STEPS = (int(v) for v in lru_trace["params"])
    bufs = {}
    zeros9 = (u64 * 9)()
    for l in range(NL):
        bufs[l] = (ctypes.c_uint32 * 16)()
        L.c_layer_init(layer_base + l, -1, CAP, zeros9, zeros9, zeros9, ctypes.addressof(bufs[l]))
    mid = int(lru_trace["set_state_at"][0])
    n_miss, slots = [], []
    for i in range(len(lru_trace["layers"])):
        l = int(lru_trace["layers"][i])
        eids = (ctypes.c_uint32 * K)(*[int(v) for v in lru_trace["eids"][i]])
        n_miss.append(L.c_layer_step_decode_ex(layer_base + l, eids, K, 1))
        slots.append(list(bufs[l])[:K])
        pred = lru_trace["preds"][i]
        if pred[0] >= 0:
            L.c_layer_start_prefetch(layer_base + l + 1, (ctypes.c_int32 * M)(*[int(v) for v in pred]), M, PCAP)
        if i == mid:
            oe, os_, cnt = (ctypes.c_int32 * 512)(), (ctypes.c_int32 * 512)(), ctypes.c_int(0)
            L.c_layer_get_lru_state(layer_base + 1, oe, os_, ctypes.byref(cnt))
            keep = list(oe)[: cnt.value][-40:]
            L.c_layer_set_lru_state(layer_base + 1, (ctypes.c_int32 * 40)(*keep),
                                    (ctypes.c_int32 * 40)(*range(40)), 40, u64(400), u64(350), u64(12))
    stats, order = [], []
    for l in range(NL):
        st = (u64 * 18)()
        L.c_layer_get_stats(layer_base + l, st)
        stats.append(list(st))
        oe, os_, cnt = (ctypes.c_int32 * 512)(), (ctypes.c_int32 * 512)(), ctypes.c_int(0)
        L.c_layer_get_lru_state(layer_base + l, oe, os_, ctypes.byref(cnt))
        snap = np.full((2, 512), -1, dtype=np.int32)
        snap[0, : cnt.value] = list(oe)[: cnt.value]
        snap[1, : cnt.value] = list(os_)[: cnt.value]
        order.append(snap)
    return np.array(n_miss), np.array(slots), np.array(stats, dtype=np.uint64), np.stack(order)


def test_dropin_abi_replays_reference_trace(lib, lru_trace):
    n_miss, slots, stats, order = _replay_dropin(lib, lru_trace, layer_base=0)
    assert np.array_equal(n_miss, lru_trace["n_miss"]), "miss counts differ"
    assert np.array_equal(slots, lru_trace["slots"]), "slot ids differ"
    assert np.array_equal(stats, lru_trace["stats"]), "counters differ"
    assert np.array_equal(order, lru_trace["lru_state"]), "final LRU order differs"
    tot = (u64 * 6)()
    lib.c_get_decode_totals(int(lru_trace["params"][5]), tot)
    assert list(tot) == [int(v) for v in lru_trace["totals"]]


def test_device_api_replays_reference_trace(dev, lib, lru_trace):
    """moe_lru_* with the indices and lists in device memory (no host staging)."""
    from moe_offload_b200._lib import call
    E, K, M, CAP, PCAP, NL, STEPS = (int(v) for v in lru_trace["params"])
    nb = int(call("moe_lru_state_bytes", E, CAP))
    states = [torch.empty(nb, dtype=torch.uint8, device=dev) for _ in range(NL)]
    s = torch.cuda.current_stream(dev).cuda_stream
    for st in states:
        call("moe_lru_init", st.data_ptr(), E, CAP, 1536000, s)
    eids = torch.from_numpy(lru_trace["eids"].astype(np.int32)).to(dev)
    preds = torch.from_numpy(lru_trace["preds"].astype(np.int32)).to(dev)
    nsteps = len(lru_trace["layers"])
    out_slots = torch.zeros((nsteps, K), dtype=torch.int32, device=dev)
    out_miss = torch.zeros((nsteps, 1 + 2 * K), dtype=torch.int32, device=dev)
    pref = torch.zeros((nsteps, 1 + 2 * PCAP), dtype=torch.int32, device=dev)
    mid = int(lru_trace["set_state_at"][0])
    for i in range(nsteps):
        l = int(lru_trace["layers"][i])
        call("moe_lru_step", states[l].data_ptr(), E, CAP, eids[i].data_ptr(), K, out_slots[i].data_ptr(),
             out_miss[i].data_ptr(), s)
        if lru_trace["preds"][i][0] >= 0:
            call("moe_lru_prefetch", states[l + 1].data_ptr(), E, CAP, preds[i].data_ptr(), M, PCAP,
                 pref[i].data_ptr(), s)
        if i == mid:
            st = torch.empty(1 + 2 * CAP, dtype=torch.int32, device=dev)
            call("moe_lru_get_state", states[1].data_ptr(), E, CAP, st.data_ptr(), s)
            o = st.cpu().tolist()
            keep = o[1:1 + o[0]][-40:]
            ke = torch.tensor(keep, dtype=torch.int32, device=dev)
            ks = torch.arange(40, dtype=torch.int32, device=dev)
            call("moe_lru_set_state", states[1].data_ptr(), E, CAP, ke.data_ptr(), ks.data_ptr(), 40, 400, 350, 12, s)
    torch.cuda.synchronize()
    assert np.array_equal(out_miss[:, 0].cpu().numpy(), lru_trace["n_miss"])
    assert np.array_equal(out_slots.cpu().numpy(), lru_trace["slots"])
    for l in range(NL):
        st = torch.empty(18, dtype=torch.int64, device=dev)
        call("moe_lru_get_stats", states[l].data_ptr(), E, CAP, st.data_ptr(), s)
        assert np.array_equal(st.cpu().numpy().astype(np.uint64), lru_trace["stats"][l]), f"layer {l} counters"
        o = torch.empty(1 + 2 * CAP, dtype=torch.int32, device=dev)
        call("moe_lru_get_state", states[l].data_ptr(), E, CAP, o.data_ptr(), s)
        o = o.cpu().numpy()
        n = o[0]
        assert np.array_equal(o[1:1 + n], lru_trace["lru_state"][l, 0, :n])
        assert np.array_equal(o[1 + CAP:1 + CAP + n], lru_trace["lru_state"][l, 1, :n])
    # the miss lists name the missing experts in request order with their new slots
    i = int(np.argmax(lru_trace["n_miss"]))
    m = out_miss[i].cpu().numpy()
    n = m[0]
    missing = m[1:1 + n]
    assert set(missing) <= set(lru_trace["eids"][i])
    for e, sl in zip(missing, m[1 + K:1 + K + n]):
        assert sl == lru_trace["slots"][i][list(lru_trace["eids"][i]).index(e)]


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built (oracle/_ref)")
@pytest.mark.parametrize("cap,max_fetch,seed", [(12, 3, 1), (16, 0, 2), (10, 8, 3), (40, 3, 4)])
def test_dropin_matches_reference_library_live(lib, cap, max_fetch, seed):
    """Same random calls into the reference library and ours: small caches, so eviction
    often finds every resident expert protected (the fall-back to the oldest slot)."""
    ref = ctypes.CDLL(REF_LIB)
    rng = np.random.default_rng(seed)
    K, M = 10, 12
    zeros9 = (u64 * 9)()
    bref, bour = (ctypes.c_uint32 * 16)(), (ctypes.c_uint32 * 16)()
    lid = 40 + seed
    ref.c_layer_init(lid, -1, cap, zeros9, zeros9, zeros9, u64(ctypes.addressof(bref)))
    lib.c_layer_init(lid, -1, cap, zeros9, zeros9, zeros9, ctypes.addressof(bour))
    hot = rng.permutation(512)[:48]
    for step in range(300):
        eids = rng.choice(hot, size=K, replace=False).astype(np.uint32)
        a = (ctypes.c_uint32 * K)(*eids.tolist())
        assert ref.c_layer_step_decode_ex(lid, a, K, 0) == lib.c_layer_step_decode_ex(lid, a, K, 0), step
        assert list(bref)[:K] == list(bour)[:K], step
        if step % 3 == 0:
            pred = rng.choice(hot, size=M, replace=False).astype(np.int32)
            p = (ctypes.c_int32 * M)(*pred.tolist())
            ref.c_layer_start_prefetch(lid, p, M, max_fetch)
            lib.c_layer_start_prefetch(lid, p, M, max_fetch)
        if step % 50 == 49:
            ref.c_layer_reset_cache(lid) if step % 100 == 99 else None
            lib.c_layer_reset_cache(lid) if step % 100 == 99 else None
    sr, so = (u64 * 18)(), (u64 * 18)()
    ref.c_layer_get_stats(lid, sr)
    lib.c_layer_get_stats(lid, so)
    assert list(sr) == list(so)
    er, sl_r, cr = (ctypes.c_int32 * 512)(), (ctypes.c_int32 * 512)(), ctypes.c_int(0)
    eo, sl_o, co = (ctypes.c_int32 * 512)(), (ctypes.c_int32 * 512)(), ctypes.c_int(0)
    ref.c_layer_get_lru_state(lid, er, sl_r, ctypes.byref(cr))
    lib.c_layer_get_lru_state(lid, eo, sl_o, ctypes.byref(co))
    assert cr.value == co.value and list(er)[:cr.value] == list(eo)[:co.value]
    assert list(sl_r)[:cr.value] == list(sl_o)[:co.value]


def test_fill_kernel_and_host_fill_copy_pool_rows(dev, lib):
    from moe_offload_b200._lib import call
    E, cap, K = 64, 16, 8
    rng = np.random.default_rng(7)
    rows = [4096, 1024, 528 * 16 // 16 * 16]
    pools = [torch.from_numpy(rng.integers(0, 255, size=(E, r), dtype=np.uint8)).pin_memory() for r in rows]
    for use_kernel in (True, False):
        slots = [torch.zeros((cap, r), dtype=torch.uint8, device=dev) for r in rows]
        src = (ctypes.c_void_p * 3)(*[p.data_ptr() for p in pools])
        dst = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in slots])
        rb = (ctypes.c_uint64 * 3)(*rows)
        state = torch.empty(int(call("moe_lru_state_bytes", E, cap)), dtype=torch.uint8, device=dev)
        s = torch.cuda.current_stream(dev).cuda_stream
        call("moe_lru_init", state.data_ptr(), E, cap, 1, s)
        resident = {}
        for step in range(20):
            eids = torch.from_numpy(rng.choice(E, size=K, replace=False).astype(np.int32)).to(dev)
            out_s = torch.zeros(K, dtype=torch.int32, device=dev)
            miss = torch.zeros(1 + 2 * K, dtype=torch.int32, device=dev)
            call("moe_lru_step", state.data_ptr(), E, cap, eids.data_ptr(), K, out_s.data_ptr(), miss.data_ptr(), s)
            if use_kernel:
                call("moe_fill_slots", miss.data_ptr(), K, E, cap, 3, src, dst, rb, 0, s)
            else:
                mh = miss.cpu().numpy().astype(np.int32)
                call("moe_fill_slots_host", mh.ctypes.data, K, E, cap, 3, src, dst, rb, s)
            torch.cuda.synchronize()
            for e, sl in zip(eids.cpu().tolist(), out_s.cpu().tolist()):
                resident[sl] = e
            for sl, e in resident.items():
                for p, t in zip(pools, slots):
                    assert torch.equal(t[sl].cpu(), p[e]), (use_kernel, step, sl, e)
    assert int(call("moe_device_error", 1)) == 0


def test_cached_layer_matches_resident_layer(dev):
    """CachedSwitchGLU (slots filled from the pinned pool) gives exactly the outputs of the
    same experts resident in HBM, through hits, misses and prefetches."""
    from moe_offload_b200 import ops
    from moe_offload_b200.offload import CachedSwitchGLU, HostExpertPool
    from moe_offload_b200.synthetic import (ExpertLayer, np_bf16_normal, np_qmatrix, np_to_bf16_tensor,
                                            to_device_qmatrix)
    rng = np.random.default_rng(11)
    E, H, I, K, cap = 64, 1024, 256, 8, 16
    g, u, d = np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, H, I)
    res = ExpertLayer(np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev), to_device_qmatrix(g, dev),
                      to_device_qmatrix(u, dev), to_device_qmatrix(d, dev))
    cache = CachedSwitchGLU(None, 1, cap, pool=HostExpertPool.from_layer(res), device=dev, top_k=K)
    hot = rng.permutation(E)[:24]
    for step in range(40):
        x = np_to_bf16_tensor(np_bf16_normal(rng, (1, 1, H)), dev)
        eids = torch.from_numpy(rng.choice(hot, size=K, replace=False).astype(np.int32)).to(dev).view(1, 1, K)
        y = cache(x, eids)
        act = ops.experts_gateup(x.view(1, H), eids.view(1, K), res.gate, res.up)
        _, yk = ops.experts_down(act, eids.view(1, K), res.down, None, want_yk=True)
        assert torch.equal(y.view(K, H), yk.view(K, H)), step
        if step % 4 == 3:
            pred = torch.from_numpy(rng.choice(hot, size=12, replace=False).astype(np.int32)).to(dev)
            cache.start_prefetch(pred, 3)
    st = cache.get_layer_stats()
    assert st["decode_requests"] == 40 * K
    assert st["decode_lru_hits"] + st["decode_prefetch_hits"] + st["decode_demand_misses"] == 40 * K
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


def test_offload_stack_graph_matches_eager_and_resident(dev):
    """OffloadStack (layer 0 pinned, cached layers behind the GPU LRU, prefetch on a side
    stream): the captured graph gives the eager results, and both equal the all-resident
    per-layer path with the same routing."""
    from moe_offload_b200 import ops
    from moe_offload_b200.offload import HostExpertPool, OffloadStack, _pow2_normalize_dev, zipf_routing
    from moe_offload_b200.synthetic import (ExpertLayer, np_bf16_normal, np_qmatrix, np_to_bf16_tensor,
                                            to_device_qmatrix)
    rng = np.random.default_rng(21)
    L, E, H, I, K, cap = 3, 64, 1024, 256, 8, 16
    layers = []
    for _ in range(L):
        layers.append(ExpertLayer(np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev),
                                  to_device_qmatrix(np_qmatrix(rng, E, I, H), dev),
                                  to_device_qmatrix(np_qmatrix(rng, E, I, H), dev),
                                  to_device_qmatrix(np_qmatrix(rng, E, H, I), dev)))
    pools = [HostExpertPool.from_layer(layers[l]) for l in range(1, L)]
    caps = {l: cap for l in range(1, L)}
    routing, bias = zipf_routing(seed=5, layers=L, tokens=24, E=E, K=K)
    inj = torch.from_numpy(routing).to(dev)
    hs = [np_to_bf16_tensor(np_bf16_normal(rng, (1, H)), dev) for _ in range(24)]

    def make():
        st = OffloadStack([ly.router for ly in layers], layers[0], pools, caps, K, dev)
        st.pred_bias = torch.from_numpy(bias).to(dev)
        return st

    eager, graphed = make(), make()
    graphed.capture()
    graphed.reset_caches()
    graphed.reset_stats()
    for t in range(24):
        ye = eager.decode_token(hs[t], inj[t]).clone()
        yg = graphed.decode_graph(hs[t], inj[t]).clone()
        # resident reference for the same token and routing
        x = hs[t]
        for l in range(L):
            xin = _pow2_normalize_dev(x)
            r = ops.router_topk(xin, layers[l].router, K)
            e = inj[t][l].view(1, K)
            act = ops.experts_gateup(xin, e, layers[l].gate, layers[l].up)
            x, _ = ops.experts_down(act, e, layers[l].down, r["scores"], resid=x)
        torch.cuda.synchronize()
        assert torch.equal(ye, yg), t
        assert torch.equal(ye, x), t
    te, tg = eager.decode_totals(), graphed.decode_totals()
    assert te == tg
    assert te["decode_requests"] == 24 * K * (L - 1)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0
