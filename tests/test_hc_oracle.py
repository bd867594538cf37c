"""The hyper-connection mixer before the MoE block (run_hc, kernels.cpp:1363-1560): the CPU
oracle (orc_hc_mix) against the reference's golden MLX tensors (tests/golden/hc_fixture,
from cpp/tests/fixtures.safetensors `hc.*` / `pred_next.*`). CPU only.

Rows 1 and 8 take the reference's fused decode kernels, row count 18 its prefill path; the
oracle follows the matching rounding regime for each."""
import numpy as np
import pytest

from oracle import oracle as orc

HC, H, R = 4, 2560, 320


def _q(fx, p):
    return fx[f"{p}.weight"], fx[f"{p}.scales"], fx[f"{p}.biases"]


def _run(fx, tag, rows, write, combine=True):
    h = fx[f"hc.{tag}.h_in"].reshape(rows, -1)
    br = fx[f"hc.{tag}.br_in"].reshape(rows, -1) if write else None
    gt = fx[f"hc.{tag}.gt_in"].reshape(rows, -1) if write else None
    return orc.hc_mix(h, fx["hc.norm.weight"], _q(fx, "hc.down"), _q(fx, "hc.up"),
                      _q(fx, "hc.inject") if combine else None, branch=br, gate=gt)


def _rel(a, b):
    a = orc.bf16_to_f32(a).astype(np.float64)
    b = orc.bf16_to_f32(b).astype(np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b)


# (tag, rows, mixed bit-equal fraction at least, mixed norm-relative error at most)
CASES = [("r1", 1, 0.99, 2e-4), ("r8", 8, 0.99, 2e-4), ("r18", 18, 0.9, 3e-3)]


@pytest.mark.parametrize("tag,rows,eq_min,rel_max", CASES)
def test_written_bit_exact(hc_fixture, tag, rows, eq_min, rel_max):
    fx = hc_fixture
    out = _run(fx, tag, rows, write=True)
    assert np.array_equal(out["written"], fx[f"hc.{tag}.h_write"].reshape(rows, -1))


@pytest.mark.parametrize("tag,rows,eq_min,rel_max", CASES)
@pytest.mark.parametrize("write", [False, True])
def test_mixed_and_inject(hc_fixture, tag, rows, eq_min, rel_max, write):
    """mixed within MLX's residual (the decode regime is bit-equal on these rows but for a
    handful of values), inject weights bit-exact but for at most one value in 32."""
    fx = hc_fixture
    sfx = "write" if write else "nowrite"
    out = _run(fx, tag, rows, write)
    ref = fx[f"hc.{tag}.m_{sfx}"].reshape(rows, -1)
    assert np.mean(out["mixed"] == ref) >= eq_min
    assert _rel(out["mixed"], ref) <= rel_max
    iref = fx[f"hc.{tag}.inj_{sfx}"].reshape(rows, -1)
    assert np.mean(out["inj"] == iref) >= 0.96
    assert np.max(np.abs(orc.bf16_to_f32(out["inj"]) - orc.bf16_to_f32(iref))) <= 2.0 ** -7


@pytest.mark.parametrize("tag,rows,eq_min,rel_max", CASES)
def test_mixer_without_inject(hc_fixture, tag, rows, eq_min, rel_max):
    """use_combine=False (the final mixer): same mixed output, no inject weights."""
    fx = hc_fixture
    out = _run(fx, tag, rows, write=True, combine=False)
    ref = fx[f"hc.{tag}.mix_write"].reshape(rows, -1)
    assert np.mean(out["mixed"] == ref) >= eq_min - 0.5 * (rows > 16)
    assert _rel(out["mixed"], ref) <= max(rel_max, 6e-3 * (rows > 16))
    assert not out["inj"].any()


@pytest.mark.parametrize("write", [False, True])
def test_next_layer_prediction_top12(hc_fixture, write):
    """pred_next: the top-12 experts of an 8-bit 64-expert gate on the mixed input, sorted by
    logit (loader.py:237-242), bit-exact with MLX's (gen_fixtures.py:685-705)."""
    fx = hc_fixture
    out = _run(fx, "r1", 1, write)
    w, s, b = _q(fx, "pred_next.gate")
    lg = orc.router_logits(out["mixed"], w, 64, rbits=8, scales=s, biases=b, group_size=64, sb_fp16=False)
    pred = orc.topm_sorted(lg, 12)
    ref = fx["pred_next.top12_write" if write else "pred_next.top12_nowrite"].reshape(1, 12)
    assert np.array_equal(pred.astype(np.uint32), ref)
