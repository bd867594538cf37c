"""Shared expert and affine-quantised linear layers on the GPU (csrc/shared.cu) against the CPU
oracle, and the whole MoE layer (routed experts + this shared expert as the combine addend)
against the reference's golden MLX output.

Tolerances: moe_affine_linear is bit-exact with orc_affine_linear (same sums in the same
order). The shared expert differs from the oracle only where CUDA's expf and the host's expf
round a sigmoid differently: norm-relative error <= 2e-3 with >= 99 % of outputs bit-equal.
Against MLX's output the bound is MLX's own residual (1.5e-2 decode, 1.0e-2 prefill)."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _rel(a_u16, b_u16):
    a = orc.bf16_to_f32(a_u16).astype(np.float64)
    b = orc.bf16_to_f32(b_u16).astype(np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _rand_q(rng, N, K, bits, gs, sb_fp16, scale=0.04):
    per = 32 // bits
    w = rng.integers(0, 2 ** 32, size=(N, K // per), dtype=np.uint64).astype(np.uint32)
    s = (rng.random((N, K // gs)) * scale + scale / 20).astype(np.float32)
    b = rng.normal(0, scale / 2, (N, K // gs)).astype(np.float32)
    if sb_fp16:
        return w, s.astype(np.float16).view(np.uint16), b.astype(np.float16).view(np.uint16)
    return w, orc.f32_to_bf16(s), orc.f32_to_bf16(b)


def _qdev(t, dev, bits, gs, sb_fp16):
    from moe_offload_b200.synthetic import to_device_qmatrix
    return to_device_qmatrix(t, dev, bits=bits, gs=gs, sb_fp16=sb_fp16)


@pytest.mark.parametrize("bits,gs,T,K,N,sb_fp16", [
    (4, 64, 1, 3072, 768, False),      # shared gate/up at the stack's H
    (4, 64, 1, 768, 3072, False),      # shared down
    (8, 64, 1, 3072, 1, False),        # the scalar shared-expert gate
    (4, 64, 20, 256, 128, False),      # fixture shape, prefill
    (2, 64, 5, 512, 33, True),
    (4, 32, 9, 384, 7, True),
    (8, 128, 2, 1024, 64, False),
    (2, 32, 1, 64, 1, False),
])
def test_affine_linear_bit_exact(dev, bits, gs, T, K, N, sb_fp16):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_to_bf16_tensor
    rng = np.random.default_rng(bits * 1000 + T * 10 + N)
    wq = _rand_q(rng, N, K, bits, gs, sb_fp16)
    x = orc.f32_to_bf16(rng.normal(0, 0.3, (T, K)).astype(np.float32))
    y = ops.affine_linear(np_to_bf16_tensor(x, dev), _qdev(wq, dev, bits, gs, sb_fp16))
    torch.cuda.synchronize()
    ref = orc.affine_linear(x, wq, bits, gs, sb_fp16=sb_fp16)
    assert np.array_equal(bf16_tensor_to_np(y), ref)


def _gpu_shared(dev, x, mats, sb_fp16=False, bits=4, gs=64, gbits=8, ggs=64):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_to_bf16_tensor
    g, u, d, e = mats
    y = ops.shared_expert(np_to_bf16_tensor(x, dev), _qdev(g, dev, bits, gs, sb_fp16), _qdev(u, dev, bits, gs, sb_fp16),
                          _qdev(d, dev, bits, gs, sb_fp16), _qdev(e, dev, gbits, ggs, sb_fp16))
    torch.cuda.synchronize()
    return bf16_tensor_to_np(y)


def test_shared_expert_fixture_and_full_layer(moe_fixture, dev):
    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_to_bf16_tensor
    fx = moe_fixture
    H, K = 256, 4
    q = lambda p: (fx[f"{p}.weight"], fx[f"{p}.scales"], fx[f"{p}.biases"])
    mats = [q("moe.shared_gate"), q("moe.shared_up"), q("moe.shared_down"), q("moe.shared_expert_gate")]
    sw = [q(f"moe.switch_{p}") for p in ("gate", "up", "down")]
    for tag, bound in (("dec", 1.5e-2), ("pre", 1.0e-2)):
        x = fx[f"moe.x_{tag}"].reshape(-1, H)
        sh = _gpu_shared(dev, x, mats)
        ref = orc.shared_expert(x, *mats, sb_fp16=False)["y"]
        assert _rel(sh, ref) < 2e-3 and np.mean(sh == ref) >= 0.99, tag
        assert _rel(sh, fx[f"moe.sh_{tag}"].reshape(-1, H)) < bound, tag
        # the whole layer: routed experts with this shared output as the combine addend
        inds = fx[f"moe.inds_{tag}"].reshape(-1, K)
        sc = fx[f"moe.scores_{tag}"].reshape(-1, K)
        st = torch.from_numpy(inds.astype(np.uint32).view(np.int32)).to(dev)
        G, U, D = (_qdev(t, dev, 2, 64, False) for t in sw)
        xt = np_to_bf16_tensor(x, dev)
        act = ops.experts_gateup(xt, st, G, U)
        y, _ = ops.experts_down(act, st, D, np_to_bf16_tensor(sc, dev), addend=np_to_bf16_tensor(sh, dev))
        torch.cuda.synchronize()
        y = bf16_tensor_to_np(y)
        yo = orc.experts(x, inds, sc, *sw, bits=2, group_size=64, sb_fp16=False, addend=ref)["y"]
        assert _rel(y, yo) < 1e-2, tag
        assert _rel(y, fx[f"moe.y_{tag}"].reshape(-1, H)) < bound, tag


@pytest.mark.parametrize("T,H,I,sb_fp16", [(1, 3072, 768, False), (7, 3072, 768, True), (3, 1024, 512, False)])
def test_shared_expert_synthetic(dev, T, H, I, sb_fp16):
    rng = np.random.default_rng(T * 7 + I)
    mats = [_rand_q(rng, I, H, 4, 64, sb_fp16, 0.01), _rand_q(rng, I, H, 4, 64, sb_fp16, 0.01),
            _rand_q(rng, H, I, 4, 64, sb_fp16, 0.02), _rand_q(rng, 1, H, 8, 64, sb_fp16, 0.001)]
    x = orc.f32_to_bf16(rng.normal(0, 0.5, (T, H)).astype(np.float32))
    sh = _gpu_shared(dev, x, mats, sb_fp16=sb_fp16)
    ref = orc.shared_expert(x, *mats, sb_fp16=sb_fp16)["y"]
    assert _rel(sh, ref) < 2e-3
    assert np.mean(sh == ref) >= 0.99


def test_shared_expert_bad_arguments(dev):
    from moe_offload_b200._lib import MoeError, call
    from moe_offload_b200.ops import QMatrix, affine_linear
    x = torch.zeros((1, 256), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((4, 256 * 4 // 32), dtype=torch.int32, device=dev)
    s = torch.zeros((4, 4), dtype=torch.bfloat16, device=dev)
    with pytest.raises(MoeError):                       # 3-bit codes are not a supported width
        call("moe_affine_linear", x.data_ptr(), 1, 256, 4, w.data_ptr(), s.data_ptr(), s.data_ptr(), 3, 64, 0,
             x.data_ptr(), 0)
    with pytest.raises(MoeError):                       # group does not tile the row
        call("moe_affine_linear", x.data_ptr(), 1, 256, 4, w.data_ptr(), s.data_ptr(), s.data_ptr(), 4, 96, 0,
             x.data_ptr(), 0)
    with pytest.raises(MoeError):                       # too small a workspace
        call("moe_shared_expert", x.data_ptr(), 1, 256, 4, *([w.data_ptr()] * 9), 4, 64, *([w.data_ptr()] * 3), 8, 64,
             0, x.data_ptr(), w.data_ptr(), 16, 0)
    with pytest.raises(ValueError):
        affine_linear(x, QMatrix(w.view(1, 4, 32), s.view(1, 4, 4), s.view(1, 4, 4), 4, 64))
