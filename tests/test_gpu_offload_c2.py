"""The offload decode path the c2 bench times (OffloadStack.decode_graph: one CUDA graph per
token, LRU steps, fills and prefetches on the device) against the reference's own LRU cache
(mlx-qwen38/expert_io.c, compiled unmodified into oracle/_ref) fed the same calls in the same
order, at BASELINE config 2's cache geometry: 28 layers, layer 0 pinned, 102 slots per cached
layer (20 % of 512 experts, compute_layer_capacities), top-10 routing injected from the
synthetic Zipf(1.1) + 30 % reuse stream (seed 2), top-12 ranked predictions of recall@10
83.6 % (the reference's measured predictor recall) prefetching at most 3 experts per layer,
256 tokens. Every step's miss count and slot ids, every layer's 18 counters and the final LRU
order must be identical. The hidden and intermediate sizes are reduced (H 256, I 128): the
cache's decisions depend only on the expert ids, and the small experts keep the pinned host
pools at ~370 MB."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libexpert_io_ref.so")
u64 = ctypes.c_uint64
EXPERT_BYTES_REF = 1_536_000      # the byte counters' unit in the reference (expert_io.c:18-23)


def _reference_run(routing, preds, L, cap, K, M, pcap):
    """The same call sequence through the reference library: per token, after layer 0 the
    prefetch of layer 1, then for every cached layer l its decode step and (l < L-1) the
    prefetch of layer l+1 (loader.py:950-977 order)."""
    ref = ctypes.CDLL(REF_LIB)
    zeros9 = (u64 * 9)()
    bufs = {l: (ctypes.c_uint32 * 16)() for l in range(1, L)}
    for l in range(1, L):
        ref.c_layer_init(l, -1, cap, zeros9, zeros9, zeros9, u64(ctypes.addressof(bufs[l])))
    T = routing.shape[0]
    n_miss = np.zeros((T, L - 1), dtype=np.int32)
    slots = np.zeros((T, L - 1, K), dtype=np.int32)
    for t in range(T):
        for l in range(L):
            if l >= 1:
                eids = (ctypes.c_uint32 * K)(*[int(v) for v in routing[t, l]])
                n_miss[t, l - 1] = ref.c_layer_step_decode_ex(l, eids, K, 1)
                slots[t, l - 1] = list(bufs[l])[:K]
            if l + 1 < L:
                p = (ctypes.c_int32 * M)(*[int(v) for v in preds[t, l]])
                ref.c_layer_start_prefetch(l + 1, p, M, pcap)
    stats, order = [], []
    for l in range(1, L):
        st = (u64 * 18)()
        ref.c_layer_get_stats(l, st)
        stats.append([int(v) for v in st])
        oe, os_, cnt = (ctypes.c_int32 * 512)(), (ctypes.c_int32 * 512)(), ctypes.c_int(0)
        ref.c_layer_get_lru_state(l, oe, os_, ctypes.byref(cnt))
        order.append((list(oe)[:cnt.value], list(os_)[:cnt.value]))
    return n_miss, slots, stats, order


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built (oracle/_ref)")
def test_offload_graph_matches_reference_cache_at_c2_geometry():
    import dataclasses

    from moe_offload_b200.offload import (HostExpertPool, OffloadStack, compute_layer_capacities,
                                          synthetic_predictions, zipf_routing)
    from moe_offload_b200.synthetic import C2, dev_bf16_normal, dev_stack
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    dev = torch.device("cuda:0")
    L, E, K, M, PCAP, T = C2.layers, C2.experts, C2.top_k, 12, 3, 256
    cfg = dataclasses.replace(C2, hidden=256, inter=128)
    caps = compute_layer_capacities(budget_pct=20, num_layers=L, num_experts=E, expert_bytes=C2.expert_bytes)
    assert set(caps.values()) == {102}
    layers = dev_stack(cfg, dev, layers=L)
    pools = [HostExpertPool.from_layer(layers[l]) for l in range(1, L)]
    st = OffloadStack([ly.router for ly in layers], layers[0], pools, caps, K, dev, prefetch=True,
                      prefetch_top_m=M, prefetch_cap=PCAP, expert_bytes=EXPERT_BYTES_REF)
    routing, bias = zipf_routing(seed=C2.seed, layers=L, tokens=T, E=E, K=K)
    preds = synthetic_predictions(routing, bias, recall=0.836, M=M, seed=C2.seed)
    inject = torch.from_numpy(routing).to(dev)
    pred_dev = torch.from_numpy(preds).to(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(C2.seed)
    h = dev_bf16_normal((T, 1, cfg.hidden), dev, gen)
    st.capture(pred_injected=True)          # its warm-up token runs through the caches: start clean
    st.reset_caches()
    st.reset_stats()
    torch.cuda.synchronize()
    n_miss = np.zeros((T, L - 1), dtype=np.int32)
    slots = np.zeros((T, L - 1, K), dtype=np.int32)
    for t in range(T):
        st.decode_graph(h[t], inject[t], pred_dev[t])
        sl = torch.stack([c._slot_inds_buf.view(-1) for c in st.layers[1:]]).cpu().numpy()
        nm = torch.stack([c._miss[0] for c in st.layers[1:]]).cpu().numpy()
        slots[t] = sl
        n_miss[t] = nm
    r_miss, r_slots, r_stats, r_order = _reference_run(routing, preds, L, 102, K, M, PCAP)
    bad = np.argwhere(n_miss != r_miss)
    assert bad.size == 0, f"miss counts differ first at (token, layer) {tuple(bad[0] + [0, 1])}"
    bad = np.argwhere((slots != r_slots).any(axis=2))
    assert bad.size == 0, f"slot ids differ first at (token, layer) {tuple(bad[0] + [0, 1])}"
    for l in range(1, L):
        c = st.layers[l]
        assert c.raw_stats() == r_stats[l - 1], f"layer {l} counters"
        assert c.get_lru_state() == tuple(list(v) for v in r_order[l - 1]), f"layer {l} LRU order"
    # the prefetches are exercised and the cache behaves like BASELINE c2 says (80-90 % hits)
    tot = st.decode_totals()
    req = tot["decode_requests"]
    assert req == T * (L - 1) * K
    assert tot["decode_prefetch_hits"] / req > 0.05
    assert (tot["decode_lru_hits"] + tot["decode_prefetch_hits"]) / req >= 0.80
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0
    st.close()
