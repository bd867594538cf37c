"""The offload engine surface (OffloadEngine, loader.py:1004-1343) and the cached-layer prefill
(CachedSwitchGLU.__call__ with L > 1, loader.py:566-699) on the GPU: a prompt run through the
caches in capacity-sized chunks gives the same bits as the all-resident prefill, the LRU is
rebuilt by the reference's rule, and generate_greedy / collect_stats return the reference's
keys."""
import dataclasses

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF_RESULT_KEYS = {"prompt_tokens", "prefill_seconds", "prefill_tok_per_s", "decode_tokens", "decode_seconds",
                   "decode_tok_per_s", "prompt_pure_lru_hit_rate", "prompt_effective_hit_rate", "prompt_mb_per_token",
                   "first_window_tokens", "first_window_pure_hit_rate", "first_window_effective_hit_rate",
                   "first_window_tok_per_s", "steady_window_tokens", "steady_window_pure_hit_rate",
                   "steady_window_effective_hit_rate", "steady_window_tok_per_s", "generated_ids", "generated_text",
                   "step_latencies_ms"}


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _small_cfg():
    from moe_offload_b200.synthetic import C2
    return dataclasses.replace(C2, name="engine_test", layers=3, hidden=512, experts=32, top_k=4, inter=128, seed=7)


def _rebuild(slot_to_eid, last, cap):
    order = [s for s in range(last, cap) if s in slot_to_eid] + [s for s in range(last) if s in slot_to_eid]
    return [slot_to_eid[s] for s in order], order


def test_cached_prefill_matches_resident_and_rebuilds_lru(dev):
    from moe_offload_b200 import _lib, ops
    from moe_offload_b200.offload import HostExpertPool, OffloadStack
    from moe_offload_b200.synthetic import dev_bf16_normal, dev_stack
    cfg = _small_cfg()
    layers = dev_stack(cfg, dev)
    pools = [HostExpertPool.from_layer(ly) for ly in layers[1:]]
    caps = {1: 16, 2: 16}
    st = OffloadStack([ly.router for ly in layers], layers[0], pools, caps, cfg.top_k, dev, prefetch=False)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    T = 40
    h = dev_bf16_normal((T, cfg.hidden), dev, gen)
    # resident reference: the same layers, every expert on the device
    x = h.clone()
    ref_inds = []
    for ly in layers:
        xn = torch.empty_like(x)
        _lib.call("moe_pow2_rows", x.data_ptr(), T, cfg.hidden, xn.data_ptr(), torch.cuda.current_stream().cuda_stream)
        r = ops.router_topk(xn, ly.router, cfg.top_k)
        ref_inds.append(r["inds"].cpu().numpy())
        x = ops.prefill_experts(xn, r["inds"], r["scores"], ly.gate, ly.up, ly.down, resid=x)
    y = st.prefill(h)
    torch.cuda.synchronize()
    assert torch.equal(y, x), "cached prefill differs from the resident prefill"
    # LRU rebuilt by the reference's rule from an empty cache: chunk c of the sorted unique
    # experts occupies slots 0..len-1 in turn; the last chunk is most recently used
    for l in (1, 2):
        uniq = np.unique(ref_inds[l])
        cap = caps[l]
        slot_to_eid = {}
        last = 0
        for u0 in range(0, len(uniq), cap):
            chunk = uniq[u0:u0 + cap]
            last = len(chunk)
            for i, e in enumerate(chunk.tolist()):
                slot_to_eid[i] = e
        want = _rebuild(slot_to_eid, last, cap)
        got = st.layers[l].get_lru_state()
        assert (list(got[0]), list(got[1])) == (want[0], want[1]), f"layer {l} LRU order"
        s = st.layers[l].get_layer_stats()
        assert s["prefill_requests"] == T * cfg.top_k
        assert s["prefill_demand_misses"] == len(uniq)
        assert s["prefill_lru_hits"] == T * cfg.top_k - len(uniq)
        assert s["prefill_demand_bytes"] == len(uniq) * cfg.expert_bytes
    assert int(_lib.call("moe_device_error", 1)) == 0
    st.close()


def test_engine_generate_and_collect_stats(dev):
    from moe_offload_b200 import _lib
    from moe_offload_b200.engine import OffloadEngine
    eng = OffloadEngine(budget_pct=50.0, config=_small_cfg(), device=dev)
    assert eng.capacities == {1: 16, 2: 16}
    assert eng.total_cached_slots == 32 and eng.cache_budget_bytes == 32 * eng.config.expert_bytes
    out = eng.generate_greedy("a synthetic prompt of some length", max_new_tokens=20, reset_stats_before=True)
    assert REF_RESULT_KEYS <= set(out)
    assert out["prompt_tokens"] == len("a synthetic prompt of some length".encode())
    assert len(out["step_latencies_ms"]) == 20 and out["first_window_tokens"] == 10
    for k in ("prompt_pure_lru_hit_rate", "prompt_effective_hit_rate", "first_window_pure_hit_rate",
              "steady_window_pure_hit_rate"):
        assert 0.0 <= out[k] <= 1.0, k
    st = eng.collect_stats(20, out["prompt_tokens"])
    assert set(st) == {"budget_summary", "decode_aggregate", "prefill_aggregate", "per_layer"}
    assert st["decode_aggregate"]["total_requests_layers_1_47"] == 20 * 2 * eng.config.top_k
    assert st["prefill_aggregate"]["total_requests_layers_1_47"] == out["prompt_tokens"] * 2 * eng.config.top_k
    assert len(st["per_layer"]) == 2
    eng.set_prefetch(False)
    out2 = eng.generate_greedy("x", max_new_tokens=4)
    assert out2["decode_tokens"] == 4
    assert int(_lib.call("moe_device_error", 1)) == 0
    eng.close()
