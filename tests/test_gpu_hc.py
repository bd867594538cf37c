"""The hyper-connection mixer on the GPU (csrc/hc.cu, moe_hc_mix) against the CPU oracle and
the reference's golden MLX tensors (tests/golden/hc_fixture).

Tolerances: written is bit-exact. mixed and inj differ from the oracle only where CUDA's expf
and the host's round a sigmoid differently: >= 99 % of mixed and >= 96 % of inj bit-equal, mixed
within 1e-3 norm-relative. The next-layer top-12 prediction computed on the GPU's mixed input
is bit-exact with MLX's."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

HC, H, R = 4, 2560, 320


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _rel(a, b):
    a = orc.bf16_to_f32(a).astype(np.float64)
    b = orc.bf16_to_f32(b).astype(np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _q(fx, p):
    return fx[f"{p}.weight"], fx[f"{p}.scales"], fx[f"{p}.biases"]


def _dq(t, dev, bits=8, gs=64, sb_fp16=False):
    from moe_offload_b200.synthetic import to_device_qmatrix
    return to_device_qmatrix(t, dev, bits=bits, gs=gs, sb_fp16=sb_fp16)


def _gpu(dev, h, norm_w, down, up, inject, branch=None, gate=None, sb_fp16=False):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_to_bf16_tensor
    write = None
    if branch is not None:
        write = (np_to_bf16_tensor(branch, dev), np_to_bf16_tensor(gate, dev))
    mixed, written, inj = ops.hc_mix(np_to_bf16_tensor(h, dev), np_to_bf16_tensor(norm_w, dev),
                                     _dq(down, dev, sb_fp16=sb_fp16), _dq(up, dev, sb_fp16=sb_fp16),
                                     None if inject is None else _dq(inject, dev, sb_fp16=sb_fp16), write=write)
    torch.cuda.synchronize()
    return bf16_tensor_to_np(mixed), bf16_tensor_to_np(written), bf16_tensor_to_np(inj)


@pytest.mark.parametrize("tag,rows", [("r1", 1), ("r8", 8), ("r18", 18)])
@pytest.mark.parametrize("write", [False, True])
@pytest.mark.parametrize("combine", [True, False])
def test_hc_fixture(hc_fixture, dev, tag, rows, write, combine):
    fx = hc_fixture
    h = fx[f"hc.{tag}.h_in"].reshape(rows, -1)
    br = fx[f"hc.{tag}.br_in"].reshape(rows, -1) if write else None
    gt = fx[f"hc.{tag}.gt_in"].reshape(rows, -1) if write else None
    inject = _q(fx, "hc.inject") if combine else None
    mixed, written, inj = _gpu(dev, h, fx["hc.norm.weight"], _q(fx, "hc.down"), _q(fx, "hc.up"), inject, br, gt)
    ref = orc.hc_mix(h, fx["hc.norm.weight"], _q(fx, "hc.down"), _q(fx, "hc.up"), inject, branch=br, gate=gt)
    assert np.array_equal(written, ref["written"] if write else h)
    assert np.mean(mixed == ref["mixed"]) >= 0.99 and _rel(mixed, ref["mixed"]) <= 1e-3
    assert np.mean(inj == ref["inj"]) >= 0.96
    sfx = "write" if write else "nowrite"
    key = f"hc.{tag}.m_{sfx}" if combine or rows <= 16 else f"hc.{tag}.mix_write"
    if combine or write:
        bound = 3e-3 if rows <= 16 or combine else 6e-3
        assert _rel(mixed, fx[key].reshape(rows, -1)) <= bound
    if combine:
        assert np.mean(inj == fx[f"hc.{tag}.inj_{sfx}"].reshape(rows, -1)) >= 0.96


@pytest.mark.parametrize("write", [False, True])
def test_hc_next_layer_prediction(hc_fixture, dev, write):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import np_to_bf16_tensor
    fx = hc_fixture
    h = fx["hc.r1.h_in"].reshape(1, -1)
    br = fx["hc.r1.br_in"].reshape(1, -1) if write else None
    gt = fx["hc.r1.gt_in"].reshape(1, -1) if write else None
    mixed, _, _ = _gpu(dev, h, fx["hc.norm.weight"], _q(fx, "hc.down"), _q(fx, "hc.up"), _q(fx, "hc.inject"), br, gt)
    gate = _dq(_q(fx, "pred_next.gate"), dev)
    o = ops.router_topk(np_to_bf16_tensor(mixed, dev), gate, 4, w_next=gate, M=12)
    torch.cuda.synchronize()
    ref = fx["pred_next.top12_write" if write else "pred_next.top12_nowrite"].reshape(1, 12)
    assert np.array_equal(o["pred"].cpu().numpy().astype(np.uint32), ref)


@pytest.mark.parametrize("T,sb_fp16,bits,gs", [(3, False, 8, 64), (17, True, 8, 64), (5, False, 4, 32), (2, True, 2, 128)])
def test_hc_synthetic(dev, T, sb_fp16, bits, gs):
    rng = np.random.default_rng(T * 31 + bits)
    Hs, Rs = 512, 128

    def qm(N, K, scale):
        per = 32 // bits
        w = rng.integers(0, 2 ** 32, size=(N, K // per), dtype=np.uint64).astype(np.uint32)
        s = (rng.random((N, K // gs)) * scale + scale / 10).astype(np.float32)
        b = rng.normal(0, scale, (N, K // gs)).astype(np.float32)
        if sb_fp16:
            return w, s.astype(np.float16).view(np.uint16), b.astype(np.float16).view(np.uint16)
        return w, orc.f32_to_bf16(s), orc.f32_to_bf16(b)

    down, up, inject = qm(Rs, HC * Hs, 2e-3 * 4 / bits), qm(HC * Hs, Rs, 2e-3 * 4 / bits), qm(HC, HC * Hs, 2e-4)
    h = orc.f32_to_bf16(rng.normal(0, 0.3, (T, HC * Hs)).astype(np.float32))
    nw = orc.f32_to_bf16(rng.normal(0, 0.05, HC * Hs).astype(np.float32))
    br = orc.f32_to_bf16(rng.normal(0, 0.3, (T, Hs)).astype(np.float32))
    gt = orc.f32_to_bf16(rng.normal(0, 0.5, (T, HC)).astype(np.float32))
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_to_bf16_tensor
    mk = lambda t: _dq(t, dev, bits=bits, gs=gs, sb_fp16=sb_fp16)
    mixed, written, inj = ops.hc_mix(np_to_bf16_tensor(h, dev), np_to_bf16_tensor(nw, dev), mk(down), mk(up),
                                     mk(inject), write=(np_to_bf16_tensor(br, dev), np_to_bf16_tensor(gt, dev)))
    torch.cuda.synchronize()
    ref = orc.hc_mix(h, nw, down, up, inject, branch=br, gate=gt, bits=bits, group_size=gs, sb_fp16=sb_fp16)
    assert np.array_equal(bf16_tensor_to_np(written), ref["written"])
    assert np.mean(bf16_tensor_to_np(mixed) == ref["mixed"]) >= 0.99
    assert _rel(bf16_tensor_to_np(mixed), ref["mixed"]) <= 1e-3
    assert np.mean(bf16_tensor_to_np(inj) == ref["inj"]) >= 0.9


def test_hc_bad_arguments(dev):
    from moe_offload_b200._lib import MoeError, call
    h = torch.zeros((1, 4 * 64), dtype=torch.bfloat16, device=dev)
    with pytest.raises(MoeError):          # three streams: the quantised path has four
        call("moe_hc_mix", h.data_ptr(), 1, 3, 64, 32, None, None, h.data_ptr(), 1e-6, *([h.data_ptr()] * 3), 8, 64,
             *([h.data_ptr()] * 3), 8, 64, None, None, None, 8, 64, 0, None, h.data_ptr(), None, h.data_ptr(), 1 << 20, 0)
    with pytest.raises(MoeError):          # a write without an output for the written streams
        call("moe_hc_mix", h.data_ptr(), 1, 4, 64, 32, h.data_ptr(), h.data_ptr(), h.data_ptr(), 1e-6,
             *([h.data_ptr()] * 3), 8, 64, *([h.data_ptr()] * 3), 8, 64, None, None, None, 8, 64, 0, None,
             h.data_ptr(), None, h.data_ptr(), 1 << 20, 0)
