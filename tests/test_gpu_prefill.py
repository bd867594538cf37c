"""Prefill experts (expert-grouped tcgen05 GEMMs) against the CPU oracle with the reference's
prefill tolerance rule (mlx-qwen38/test_prefill_qproj.py:80-81: per-row max |err| <= 0.02 *
max |ref|) and a norm-relative bound of 1e-2. Routing from the GPU router (bit-exact with the
oracle's, tested elsewhere). The per-row rule is checked against the fp64 dequantised
expert math (the reference test's own reference), the norm-relative bound against the CPU
oracle with MLX's bf16 roundings, on the output without the residual; the residual path is
checked for exactness separately."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _case(dev, rng, T, H, I, E, K, sb_fp16=True, sample=None):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import (bf16_tensor_to_np, np_bf16_normal, np_qmatrix, np_to_bf16_tensor,
                                            to_device_qmatrix)
    x = np_bf16_normal(rng, (T, H))
    wr = np_bf16_normal(rng, (E, H), 0.02)
    g = np_qmatrix(rng, E, I, H, sb_fp16=sb_fp16)
    u = np_qmatrix(rng, E, I, H, sb_fp16=sb_fp16)
    d = np_qmatrix(rng, E, H, I, sb_fp16=sb_fp16)
    xt = np_to_bf16_tensor(x, dev)
    r = ops.router_topk(xt, np_to_bf16_tensor(wr, dev), K)
    G = [to_device_qmatrix(m, dev, sb_fp16=sb_fp16) for m in (g, u, d)]
    y = ops.prefill_experts(xt, r["inds"], r["scores"], *G)
    yr = ops.prefill_experts(xt, r["inds"], r["scores"], *G, resid=xt)
    torch.cuda.synchronize()
    inds = r["inds"].cpu().numpy().astype(np.uint32)
    scores = bf16_tensor_to_np(r["scores"])
    Y = orc.bf16_to_f32(bf16_tensor_to_np(y)).astype(np.float64)
    # the residual is added once, exactly as bf16(x + moe)
    want = orc.f32_to_bf16((orc.bf16_to_f32(x) + orc.bf16_to_f32(bf16_tensor_to_np(y))).astype(np.float32))
    assert np.array_equal(bf16_tensor_to_np(yr), want), "residual path differs"
    rows = np.arange(T) if sample is None else np.sort(rng.choice(T, size=sample, replace=False))

    def sb(a):
        return a.view(np.float16).astype(np.float64) if sb_fp16 else orc.bf16_to_f32(a).astype(np.float64)

    def dense(m, e):
        w, sc, bi = m
        codes = ((w[e][..., None] >> (2 * np.arange(16, dtype=np.uint32))) & 3).reshape(w.shape[1], -1)
        return codes * np.repeat(sb(sc[e]), 64, axis=1) + np.repeat(sb(bi[e]), 64, axis=1)

    xf = orc.bf16_to_f32(x).astype(np.float64)
    sf = orc.bf16_to_f32(scores).astype(np.float64)
    cache = {}
    row_err = 0.0
    ref_rows = []
    for t in rows:
        acc = np.zeros(H)
        for k in range(K):
            e = int(inds[t, k])
            if e not in cache:
                cache[e] = (dense(g, e), dense(u, e), dense(d, e))
            Wg, Wu, Wd = cache[e]
            gg, uu = Wg @ xf[t], Wu @ xf[t]
            acc += sf[t, k] * (Wd @ (gg / (1.0 + np.exp(-gg)) * uu))
        row_err = max(row_err, np.abs(Y[t] - acc).max() / np.abs(acc).max())
        ref_rows.append(acc)
    # against the oracle (MLX's bf16 roundings)
    ref = orc.experts(x[rows], inds[rows], scores[rows], g, u, d, sb_fp16=sb_fp16)["y"]
    b = orc.bf16_to_f32(ref).astype(np.float64)
    rel = np.linalg.norm(Y[rows] - b) / np.linalg.norm(b)
    return row_err, rel


@pytest.mark.parametrize("T,H,I,E,K", [(64, 256, 128, 8, 2), (600, 256, 128, 2, 1), (48, 512, 256, 64, 4),
                                       (256, 1024, 256, 32, 8)])
def test_prefill_small_vs_oracle(dev, T, H, I, E, K):
    rng = np.random.default_rng(T + H + E)
    row_err, rel = _case(dev, rng, T, H, I, E, K)
    assert row_err <= 0.02, row_err
    assert rel <= 1e-2, rel
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


def test_prefill_bf16_scales(dev):
    rng = np.random.default_rng(5)
    row_err, rel = _case(dev, rng, 128, 512, 256, 16, 4, sb_fp16=False)
    assert row_err <= 0.02 and rel <= 1e-2, (row_err, rel)


def test_prefill_c3_qwen_shape_sampled(dev):
    """c3: 2048 tokens, 512 experts, top-10, H 3072, I 768; 24 tokens checked."""
    rng = np.random.default_rng(3)
    row_err, rel = _case(dev, rng, 2048, 3072, 768, 512, 10, sample=24)
    assert row_err <= 0.02 and rel <= 1e-2, (row_err, rel)


def test_prefill_c3_nemotron_shape_sampled(dev):
    """c3 variant: 1024 tokens, 240 experts, top-9, H 2688, I 1856; 16 tokens checked."""
    rng = np.random.default_rng(4)
    row_err, rel = _case(dev, rng, 1024, 2688, 1856, 240, 9, sample=16)
    assert row_err <= 0.02 and rel <= 1e-2, (row_err, rel)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


def test_prefill_layer_norm_router_and_residual(dev):
    """moe_prefill_layer = per-row power-of-two normalisation + router + experts + residual:
    indices bit-exact with the oracle's router on the normalised rows, output within the
    tolerance of the oracle's expert block on those rows plus the residual."""
    from moe_offload_b200 import ops
    from moe_offload_b200.ops import pow2_normalize
    from moe_offload_b200.synthetic import (bf16_tensor_to_np, np_bf16_normal, np_qmatrix, np_to_bf16_tensor,
                                            to_device_qmatrix)
    rng = np.random.default_rng(11)
    T, H, I, E, K = 96, 512, 256, 32, 4
    x = (orc.bf16_to_f32(np_bf16_normal(rng, (T, H))) * np.float32(3.0) ** rng.integers(-3, 4, size=(T, 1))
         ).astype(np.float32)
    x = orc.f32_to_bf16(x)
    wr = np_bf16_normal(rng, (E, H), 0.02)
    g, u, d = np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, H, I)
    xt = np_to_bf16_tensor(x, dev)
    o = ops.prefill_layer(xt, np_to_bf16_tensor(wr, dev), *[to_device_qmatrix(m, dev) for m in (g, u, d)], K,
                          norm=True, resid=xt)
    torch.cuda.synchronize()
    xn = np.stack([pow2_normalize(x[t]) for t in range(T)])
    _, ri, rs = orc.softmax_topk(orc.router_logits(xn, wr, E), K)
    assert np.array_equal(o["inds"].cpu().numpy().astype(np.uint32), ri), "prefill_layer indices differ"
    assert np.array_equal(bf16_tensor_to_np(o["scores"]), rs), "prefill_layer scores differ"
    ref = orc.experts(xn, ri, rs, g, u, d, sb_fp16=True, resid=x)["y"]
    a = orc.bf16_to_f32(bf16_tensor_to_np(o["y"])).astype(np.float64) - orc.bf16_to_f32(x)
    b = orc.bf16_to_f32(ref).astype(np.float64) - orc.bf16_to_f32(x)
    rel = np.linalg.norm(a - b) / np.linalg.norm(b)
    assert rel <= 1e-2, rel
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0
