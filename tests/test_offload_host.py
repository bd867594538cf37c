"""Host logic of the offload path (no GPU): the per-layer capacity rule of the reference's
compute_layer_capacities (mlx-qwen38/loader.py:245-303) and the c2 synthetic routing."""
import numpy as np
import pytest

from moe_offload_b200.offload import compute_layer_capacities, zipf_routing


def test_capacity_pct_rule():
    caps = compute_layer_capacities(budget_pct=20)          # the reference default engine setting
    assert set(caps) == set(range(1, 48)) and set(caps.values()) == {102}
    assert set(compute_layer_capacities(budget_pct=0.2, num_layers=28).values()) == {102}
    assert set(compute_layer_capacities(budget_pct=1.5).values()) == {16}      # 1.5 % -> 8, clamped to 16
    assert set(compute_layer_capacities(budget_pct=1).values()) == {512}       # <= 1 is a fraction
    assert set(compute_layer_capacities(budget_pct=100).values()) == {512}


def test_capacity_budget_rule():
    caps = compute_layer_capacities(budget_gb=7.5)
    # round(7.5e9 / 1,536,000) = 4883 slots over 47 layers: 42 layers of 104, 5 of 103
    assert sum(caps.values()) == 4883
    assert [caps[l] for l in (1, 42, 43, 47)] == [104, 104, 103, 103]
    assert set(compute_layer_capacities(budget_gb=0.001).values()) == {16}     # floor of 16 per layer
    assert set(compute_layer_capacities(budget_gb=1e4).values()) == {512}


def test_capacity_proportional_rule():
    w = np.arange(1, 48, dtype=np.float64)
    caps = compute_layer_capacities(budget_pct=20, alloc_mode="proportional", weights=w)
    assert sum(caps.values()) == 47 * 102
    assert min(caps.values()) >= 16 and max(caps.values()) <= 512
    assert caps[47] > caps[1]
    # without weights the reference falls back to the even split
    assert compute_layer_capacities(budget_pct=20, alloc_mode="proportional") == compute_layer_capacities(budget_pct=20)
    with pytest.raises(ValueError):
        compute_layer_capacities(budget_pct=20, alloc_mode="proportional", weights=w[:3])


def test_zipf_routing_shape_reuse_and_popularity():
    r, bias = zipf_routing(seed=2, layers=3, tokens=200, E=512, K=10)
    assert r.shape == (200, 3, 10) and bias.shape == (3, 512)
    for t in range(200):
        for l in range(3):
            assert len(set(r[t, l].tolist())) == 10
    reuse = np.mean([len(set(r[t, 0]) & set(r[t - 1, 0])) / 10 for t in range(1, 200)])
    assert 0.3 < reuse < 0.9            # explicit reuse plus Zipf repeats
    r2, _ = zipf_routing(seed=2, layers=3, tokens=200, E=512, K=10)
    assert np.array_equal(r, r2)
    top = np.argsort(-bias[0])[:10]     # the popular experts dominate the draws
    assert np.isin(r[:, 0].ravel(), top).mean() > 0.2
