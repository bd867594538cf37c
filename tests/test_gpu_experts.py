"""Decode expert GEMVs on the GPU against the CPU oracle (and the reference's golden MLX
output on the fixture). Tolerance: per-token norm-relative error <= 1e-2 with the combine,
and 2e-3 on the unrounded-comparison of the SwiGLU activations."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2          # outputs vs oracle


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _rel(a_u16, b_u16):
    a = orc.bf16_to_f32(a_u16).astype(np.float64)
    b = orc.bf16_to_f32(b_u16).astype(np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _run(dev, x, slots, scores, g, u, d, sb_fp16, addend=None, resid=None):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_to_bf16_tensor, to_device_qmatrix
    G = to_device_qmatrix(g, dev, sb_fp16=sb_fp16)
    U = to_device_qmatrix(u, dev, sb_fp16=sb_fp16)
    D = to_device_qmatrix(d, dev, sb_fp16=sb_fp16)
    xt = np_to_bf16_tensor(x, dev)
    st = torch.from_numpy(np.ascontiguousarray(slots, dtype=np.uint32).view(np.int32)).to(dev)
    sc = np_to_bf16_tensor(scores, dev)
    act = ops.experts_gateup(xt, st, G, U)
    y, yk = ops.experts_down(act, st, D, sc, addend=None if addend is None else np_to_bf16_tensor(addend, dev),
                             resid=None if resid is None else np_to_bf16_tensor(resid, dev), want_yk=True)
    torch.cuda.synchronize()
    return bf16_tensor_to_np(act), bf16_tensor_to_np(y), bf16_tensor_to_np(yk)


def test_fixture_experts(moe_fixture, dev):
    fx = moe_fixture
    g = (fx["moe.switch_gate.weight"], fx["moe.switch_gate.scales"], fx["moe.switch_gate.biases"])
    u = (fx["moe.switch_up.weight"], fx["moe.switch_up.scales"], fx["moe.switch_up.biases"])
    d = (fx["moe.switch_down.weight"], fx["moe.switch_down.scales"], fx["moe.switch_down.biases"])
    for tag in ("dec", "pre"):
        x = fx[f"moe.x_{tag}"].reshape(-1, 256)
        inds = fx[f"moe.inds_{tag}"].reshape(-1, 4)
        sc = fx[f"moe.scores_{tag}"].reshape(-1, 4)
        sh = fx[f"moe.sh_{tag}"].reshape(-1, 256)
        act, y, yk = _run(dev, x, inds, sc, g, u, d, False, addend=sh)
        ref = orc.experts(x, inds, sc, g, u, d, sb_fp16=False, addend=sh, want_act=True, want_yk=True)
        assert _rel(act, ref["act"]) < 2e-3
        assert _rel(yk, ref["yk"]) < 5e-3
        assert _rel(y, ref["y"]) < REL_TOL
        # and against the reference's MLX output: within the north-star 1e-2 (MLX's own residual
        # against the exact arithmetic is 0.95 % decode / 0.48 % prefill, see the oracle tests)
        assert _rel(y, fx[f"moe.y_{tag}"].reshape(-1, 256)) < 1e-2


@pytest.mark.parametrize("T,H,I,E,K", [(1, 3072, 768, 24, 10), (2, 2048, 768, 16, 8), (1, 2688, 1856, 12, 9),
                                       (3, 256, 128, 16, 4)])
def test_experts_vs_oracle(dev, T, H, I, E, K):
    from moe_offload_b200.synthetic import np_bf16_normal, np_qmatrix
    rng = np.random.default_rng(E * 7 + H)
    g = np_qmatrix(rng, E, I, H)
    u = np_qmatrix(rng, E, I, H)
    d = np_qmatrix(rng, E, H, I)
    x = np_bf16_normal(rng, (T, H))
    slots = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.uint32)
    sc = orc.f32_to_bf16(rng.dirichlet(np.ones(K), size=T).astype(np.float32))
    resid = np_bf16_normal(rng, (T, H))
    act, y, yk = _run(dev, x, slots, sc, g, u, d, True, resid=resid)
    ref = orc.experts(x, slots, sc, g, u, d, sb_fp16=True, resid=resid, want_act=True, want_yk=True)
    for t in range(T):
        assert _rel(act[t], ref["act"][t]) < 2e-3, t
        assert _rel(yk[t], ref["yk"][t]) < 5e-3, t
        assert _rel(y[t], ref["y"][t]) < REL_TOL, t


def test_slot_path_equals_resident_path(dev):
    """The same expert read through a permuted slot buffer gives bit-identical output."""
    from moe_offload_b200.synthetic import np_bf16_normal, np_qmatrix
    rng = np.random.default_rng(5)
    E, H, I, K = 20, 3072, 768, 10
    g, u, d = np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, H, I)
    x = np_bf16_normal(rng, (1, H))
    eids = rng.permutation(E)[:K].astype(np.uint32)[None]
    sc = orc.f32_to_bf16(np.full((1, K), 1.0 / K, dtype=np.float32))
    perm = rng.permutation(E)
    slot_of = np.argsort(perm)               # expert e lives in slot slot_of[e]
    g2, u2, d2 = (tuple(a[perm] for a in m) for m in (g, u, d))
    _, y_res, _ = _run(dev, x, eids, sc, g, u, d, True)
    _, y_slot, _ = _run(dev, x, slot_of[eids].astype(np.uint32), sc, g2, u2, d2, True)
    assert np.array_equal(y_res, y_slot)


@pytest.mark.parametrize("H,I,E,K,M", [(2048, 768, 64, 8, 0), (3072, 768, 32, 10, 12), (2688, 1856, 24, 9, 0)])
def test_fused_decode_layer_vs_oracle(dev, H, I, E, K, M):
    """router -> gate/up -> down chained with records in the workspace (the stack's layer)."""
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import (bf16_tensor_to_np, np_bf16_normal, np_qmatrix, np_to_bf16_tensor,
                                            to_device_qmatrix)
    rng = np.random.default_rng(H + E)
    T = 2
    g, u, d = np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, H, I)
    wr = np_bf16_normal(rng, (E, H), 0.02)
    wn = np_bf16_normal(rng, (E, H), 0.02)
    x = np_bf16_normal(rng, (T, H))
    out = ops.decode_layer(np_to_bf16_tensor(x, dev), np_to_bf16_tensor(wr, dev), to_device_qmatrix(g, dev),
                           to_device_qmatrix(u, dev), to_device_qmatrix(d, dev), K,
                           router_next=np_to_bf16_tensor(wn, dev) if M else None, M=M,
                           resid=np_to_bf16_tensor(x, dev))
    torch.cuda.synchronize()
    _, inds, scores = orc.softmax_topk(orc.router_logits(x, wr, E), K)
    assert np.array_equal(out["inds"].cpu().numpy().astype(np.uint32), inds)
    assert np.array_equal(bf16_tensor_to_np(out["scores"]), scores)
    if M:
        assert np.array_equal(out["pred"].cpu().numpy().astype(np.uint32), orc.topm_sorted(orc.router_logits(x, wn, E), M))
    ref = orc.experts(x, inds, scores, g, u, d, sb_fp16=True, resid=x)
    y = bf16_tensor_to_np(out["y"])
    for t in range(T):
        # compare the MoE contribution (y - resid) so the residual does not mask errors
        a = orc.bf16_to_f32(y[t]).astype(np.float64) - orc.bf16_to_f32(x[t])
        b = orc.bf16_to_f32(ref["y"][t]).astype(np.float64) - orc.bf16_to_f32(x[t])
        assert np.linalg.norm(a - b) / np.linalg.norm(b) < REL_TOL
