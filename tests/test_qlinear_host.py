"""Host-side argument checks of the quantised-linear, shared-expert and mixer entry points
(csrc/shared.cu, csrc/hc.cu): they run on a CPU-only host because every rejection happens
before any device call. The pointers below are never dereferenced."""
import pytest

from moe_offload_b200._lib import MoeError, call

P = 0x100000                                     # 16-byte aligned, never read


def _affine(bits=4, gs=64, T=1, K=256, N=8, x=P):
    return call("moe_affine_linear", x, T, K, N, P, P, P, bits, gs, 0, P, 0)


@pytest.mark.parametrize("kw,needle", [
    (dict(bits=3), "bits=3"),
    (dict(gs=48), "group_size=48"),
    (dict(K=320, gs=128), "does not divide"),
    (dict(K=64 * 400), "groups per row"),
    (dict(T=0), "bad sizes"),
    (dict(x=P + 2), "aligned"),
])
def test_affine_linear_rejects(kw, needle):
    with pytest.raises(MoeError) as e:
        _affine(**kw)
    assert needle in e.value.msg


def test_shared_expert_workspace_and_rejects():
    need = call("moe_shared_expert_workspace_bytes", 3, 3072, 768)
    assert need == 4608 + 256                   # act [3, 768] bf16 + the scalar gate per token
    assert call("moe_shared_expert_workspace_bytes", 0, 3072, 768) == 0
    args = [P, 3, 3072, 768] + [P] * 9 + [4, 64] + [P] * 3 + [8, 64, 0, P]
    with pytest.raises(MoeError) as e:
        call("moe_shared_expert", *args, P, need - 1, 0)
    assert "workspace" in e.value.msg
    with pytest.raises(MoeError) as e:           # 128-value groups: at most 128 per row for gate + up
        call("moe_shared_expert", P, 1, 128 * 200, 128, *([P] * 9), 4, 128, *([P] * 3), 8, 128, 0, P, P, 1 << 30, 0)
    assert "shared_expert: 200 groups per row" in e.value.msg


def test_hc_mix_workspace_and_rejects():
    # normed [T, 4H] bf16, down totals [T, R] f32, inject totals [T, 4] f32, each 256-aligned
    assert call("moe_hc_workspace_bytes", 1, 4, 2560, 320) == 20480 + 1280 + 256
    base = [P, 1, 4, 2560, 320, None, None, P, 1e-6] + [P] * 3 + [8, 64] + [P] * 3 + [8, 64] + [P] * 3 + \
        [8, 64, 0, None, P, P, P, 1 << 30, 0]
    bad_hc = list(base)
    bad_hc[2] = 3
    with pytest.raises(MoeError) as e:
        call("moe_hc_mix", *bad_hc)
    assert "streams" in e.value.msg
    half_write = list(base)
    half_write[5] = P                            # a branch without a gate
    with pytest.raises(MoeError) as e:
        call("moe_hc_mix", *half_write)
    assert "write" in e.value.msg
    small = list(base)
    small[-2] = 100
    with pytest.raises(MoeError) as e:
        call("moe_hc_mix", *small)
    assert "workspace" in e.value.msg
