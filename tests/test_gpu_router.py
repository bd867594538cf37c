"""Router parity on the GPU: indices and probabilities bit-exact against the CPU oracle
(and against the reference's golden MLX vectors on the fixture)."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _np(t):
    from moe_offload_b200.synthetic import bf16_tensor_to_np
    return bf16_tensor_to_np(t)


def test_fixture_router_8bit(moe_fixture, dev):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import np_to_bf16_tensor
    fx = moe_fixture
    sbd = torch.bfloat16
    wq = ops.QMatrix(torch.from_numpy(fx["moe.gate.weight"].view(np.int32)).to(dev),
                     torch.from_numpy(fx["moe.gate.scales"].view(np.int16)).to(dev).view(sbd),
                     torch.from_numpy(fx["moe.gate.biases"].view(np.int16)).to(dev).view(sbd), bits=8)
    for tag in ("dec", "pre"):
        x = fx[f"moe.x_{tag}"].reshape(-1, 256)
        out = ops.router_topk(np_to_bf16_tensor(x, dev), wq, 4, want_logits=True, want_probs=True)
        torch.cuda.synchronize()
        lg = orc.router_logits(x, fx["moe.gate.weight"], 16, rbits=8, scales=fx["moe.gate.scales"],
                               biases=fx["moe.gate.biases"], group_size=64, sb_fp16=False)
        probs, inds, scores = orc.softmax_topk(lg, 4)
        assert np.array_equal(_np(out["logits"]), lg)
        assert np.array_equal(_np(out["probs"]), probs)
        assert np.array_equal(out["inds"].cpu().numpy().astype(np.uint32), inds)
        assert np.array_equal(out["inds"].cpu().numpy().astype(np.uint32), fx[f"moe.inds_{tag}"].reshape(-1, 4))
        assert np.array_equal(_np(out["scores"]), scores)


@pytest.mark.parametrize("T,H,E,K,M", [(1, 3072, 512, 10, 12), (4, 2048, 64, 8, 0), (3, 2688, 240, 9, 12),
                                       (2, 256, 16, 4, 12),
                                       # batched path (T >= 256: tiled double-precision GEMM + per-token selection)
                                       (1024, 3072, 512, 10, 12), (1100, 2688, 240, 9, 0), (1030, 1000, 100, 6, 7),
                                       (512, 3072, 512, 10, 0), (256, 1024, 64, 4, 12)])
def test_router_bf16_bit_exact(dev, T, H, E, K, M):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(1000 + E)
    x = np_bf16_normal(rng, (T, H))
    w = np_bf16_normal(rng, (E, H), 0.02)
    wn = np_bf16_normal(rng, (E, H), 0.02)
    bias = rng.normal(0, 0.1, size=E).astype(np.float32) if M else None
    out = ops.router_topk(np_to_bf16_tensor(x, dev), np_to_bf16_tensor(w, dev), K,
                          w_next=np_to_bf16_tensor(wn, dev) if M else None, M=M,
                          pred_bias=torch.from_numpy(bias).to(dev) if M else None,
                          want_logits=True, want_probs=True)
    torch.cuda.synchronize()
    lg = orc.router_logits(x, w, E)
    probs, inds, scores = orc.softmax_topk(lg, K)
    assert np.array_equal(_np(out["logits"]), lg), "logits differ"
    assert np.array_equal(_np(out["probs"]), probs), "probs differ"
    assert np.array_equal(out["inds"].cpu().numpy().astype(np.uint32), inds), "indices differ"
    assert np.array_equal(_np(out["scores"]), scores), "scores differ"
    if M:
        plg = orc.router_logits(x, wn, E, bias_f32=bias)
        pred = orc.topm_sorted(plg, M)
        assert np.array_equal(out["pred"].cpu().numpy().astype(np.uint32), pred), "prediction differs"


def test_router_ties_resolved_like_mlx(dev):
    """Identical router rows force exact probability ties; the higher expert index wins."""
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(7)
    E, H, K = 64, 512, 8
    w = np_bf16_normal(rng, (E, H), 0.02)
    w[40:48] = w[3]           # 9 identical rows -> tied logits/probs
    x = np_bf16_normal(rng, (2, H))
    x[1] = x[0]
    out = ops.router_topk(np_to_bf16_tensor(x, dev), np_to_bf16_tensor(w, dev), K)
    torch.cuda.synchronize()
    _, inds, scores = orc.softmax_topk(orc.router_logits(x, w, E), K)
    assert np.array_equal(out["inds"].cpu().numpy().astype(np.uint32), inds)
    assert np.array_equal(_np(out["scores"]), scores)


def test_router_repeated_calls_rearm_workspace(dev):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(3)
    E, H, K = 512, 3072, 10
    w = np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev)
    xs = [np_bf16_normal(rng, (1, H)) for _ in range(5)]
    got = [ops.router_topk(np_to_bf16_tensor(x, dev), w, K)["inds"].clone() for x in xs]
    torch.cuda.synchronize()
    wn = orc.f32_to_bf16(orc.bf16_to_f32(_np(w)))
    for x, g in zip(xs, got):
        _, inds, _ = orc.softmax_topk(orc.router_logits(x, wn, E), K)
        assert np.array_equal(g.cpu().numpy().astype(np.uint32), inds)


@pytest.mark.parametrize("fmt,nfmt", [(16, 8), (8, 16), (8, 4)])
def test_router_prediction_with_other_format_next_router(dev, fmt, nfmt):
    """A next-layer router of another format than the layer's own (an 8-bit router after bf16
    ones, as in a checkpoint whose last layers keep their router at 8 bits): the prediction is
    the next router's top-M of its own logits, and the layer's routing is unchanged."""
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import np_bf16_normal, np_qmatrix, np_to_bf16_tensor, to_device_qmatrix
    rng = np.random.default_rng(50 + fmt + nfmt)
    T, H, E, K, M = 3, 1024, 64, 4, 12
    x = np_bf16_normal(rng, (T, H))

    def router(bits):
        if bits == 16:
            w = np_bf16_normal(rng, (E, H), 0.02)
            return np_to_bf16_tensor(w, dev), lambda xx: orc.router_logits(xx, w, E)
        wq = np_qmatrix(rng, 1, E, H, bits=bits, sb_fp16=False)
        d = to_device_qmatrix(wq, dev, bits=bits, sb_fp16=False)
        q = [a[0] for a in wq]
        return (ops.QMatrix(d.w[0], d.s[0], d.b[0], bits, 64),
                lambda xx: orc.router_logits(xx, q[0], E, rbits=bits, scales=q[1], biases=q[2], group_size=64))
    w, lg_w = router(fmt)
    wn, lg_wn = router(nfmt)
    out = ops.router_topk(np_to_bf16_tensor(x, dev), w, K, w_next=wn, M=M)
    torch.cuda.synchronize()
    probs, inds, scores = orc.softmax_topk(lg_w(x), K)
    assert np.array_equal(out["inds"].cpu().numpy().astype(np.uint32), inds)
    assert np.array_equal(_np(out["scores"]), scores)
    assert np.array_equal(out["pred"].cpu().numpy().astype(np.uint32), orc.topm_sorted(lg_wn(x), M))


def test_router_abi_refuses_affine_next_router_behind_bf16(dev):
    """The C entry point reads both routers in the layer router's format, so it refuses an
    affine next-layer router (scales and biases given) behind a bf16 one."""
    from moe_offload_b200 import _lib, ops
    T, H, E, K, M = 1, 256, 16, 4, 4
    x = torch.zeros((T, H), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((E, H), dtype=torch.bfloat16, device=dev)
    wn = torch.zeros((E, H // 4), dtype=torch.int32, device=dev)
    sb = torch.zeros((E, H // 64), dtype=torch.bfloat16, device=dev)
    inds = torch.zeros((T, K), dtype=torch.int32, device=dev)
    scores = torch.zeros((T, K), dtype=torch.bfloat16, device=dev)
    pred = torch.zeros((T, M), dtype=torch.int32, device=dev)
    ws = ops.router_workspace(dev, T, E, M)
    with pytest.raises(_lib.MoeError, match="format"):
        _lib.call("moe_router_topk", x.data_ptr(), T, H, E, K, w.data_ptr(), None, None, 16, 64, 0,
                  wn.data_ptr(), sb.data_ptr(), sb.data_ptr(), M, None, None, None, inds.data_ptr(),
                  scores.data_ptr(), pred.data_ptr(), ws.data_ptr(), ws.numel(),
                  torch.cuda.current_stream(dev).cuda_stream)
