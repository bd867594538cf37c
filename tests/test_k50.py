"""The K50 expert pack reader (csrc/k50.cpp through moe_offload_b200.k50; the reference's
ExpertPackCpp, mlx-qwen38/cpp/src/loader.cpp:1187-1470): layer directories written in the pack
format read back record for record; ternary rows unpack into the reference's digit order
(five base-3 digits per byte, least significant first; 16 digits per uint32 word, lowest
bits first; loader.cpp:1393-1420) with bias = -scale (1426-1431); bad packs are refused."""
import json

import numpy as np
import pytest

from moe_offload_b200 import k50
from moe_offload_b200._lib import MoeError

GS = 64


def _bf16_bits(rng, shape, lo=0.001, hi=0.05):
    f = rng.uniform(lo, hi, size=shape).astype(np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def _rec(rng, kind, rows, cols, with_bias=True):
    bits = 2 if kind in ("tern", "2t", "2") else int(kind)
    r = {"kind": kind, "unit": "hot" if kind == "2t" else "cold", "shape": (rows, cols),
         "scales": _bf16_bits(rng, (rows, cols // GS))}
    if kind == "tern":
        r["digits"] = rng.integers(0, 3, size=(rows, cols), dtype=np.uint8)
        return r
    words = cols * bits // 32
    if kind == "2t":      # ternary values as 2-bit codes
        d = rng.integers(0, 3, size=(rows, cols), dtype=np.uint32).reshape(rows, words, 16)
        r["codes"] = np.bitwise_or.reduce(d << (np.arange(16, dtype=np.uint32) * 2), axis=-1).astype(np.uint32)
    else:
        r["codes"] = rng.integers(0, 2 ** 32, size=(rows, words), dtype=np.uint64).astype(np.uint32)
    r["biases"] = _bf16_bits(rng, (rows, cols // GS), -0.02, 0.02) if with_bias else None
    return r


def test_roundtrip_every_kind(tmp_path):
    rng = np.random.default_rng(1)
    kinds = ["tern", "2t", "2", "3", "4", "6", "8"]
    experts = {"gate_proj": [_rec(rng, k, 16, 320) for k in kinds],
               "up_proj": [_rec(rng, k, 16, 320, with_bias=(i % 2 == 0)) for i, k in enumerate(kinds)],
               "down_proj": [_rec(rng, k, 64, 320) for k in ("tern", "2", "4", "2t", "3", "8", "6")]}
    dense = {"self_attn.q_proj": _rec(rng, "4", 64, 128), "shared_expert.gate_proj": _rec(rng, "2", 32, 128)}
    k50.write_k50_layer(tmp_path / "L03", experts, dense)
    with k50.K50Pack(tmp_path / "L03") as pk:
        assert pk.count("gate_proj") == 7 and pk.count("down_proj") == 7 and pk.count("dense") == 2
        assert sorted(pk.dense_names()) == sorted(dense)
        for proj, recs in experts.items():
            for e, r in enumerate(recs):
                g = pk.record(proj, e)
                rows, cols = r["shape"]
                bits = 2 if r["kind"] in ("tern", "2t", "2") else int(r["kind"])
                assert (g["bits"], g["rows"], g["cols"], g["kind"], g["unit"], g["group_size"]) == \
                    (bits, rows, cols, r["kind"], r["unit"], GS)
                assert g["words"] == cols * bits // 32 and g["groups"] == cols // GS
                w, s, b = pk.materialize(proj, e)
                assert np.array_equal(s, r["scales"])
                if r["kind"] == "tern":
                    assert np.array_equal(k50.codes_to_digits(w, cols), r["digits"])
                    assert np.array_equal(b, r["scales"] ^ 0x8000)
                else:
                    assert np.array_equal(w, r["codes"])
                    want_b = r["scales"] ^ 0x8000 if r["biases"] is None else r["biases"]
                    assert np.array_equal(b, want_b)
        w, s, b = pk.materialize("self_attn.q_proj")
        assert np.array_equal(w, dense["self_attn.q_proj"]["codes"])


def test_ternary_known_answer(tmp_path):
    """One 80-column row: byte 1 -> digits 1,0,0,0,0; 3 -> 0,1,0,0,0; 81 -> 0,0,0,0,1;
    242 -> 2,2,2,2,2; zeros after."""
    raw = np.zeros((1, 16), dtype=np.uint8)
    raw[0, :4] = [1, 3, 81, 242]
    d = np.zeros((1, 80), dtype=np.uint8)
    d[0, 0] = 1
    d[0, 6] = 1
    d[0, 14] = 1
    d[0, 15:20] = 2
    assert np.array_equal(k50.ternary_to_base3(d), raw)
    rec = {"kind": "tern", "shape": (1, 80), "digits": d, "scales": np.array([[0x3F80]], dtype=np.uint16)}
    k50.write_k50_layer(tmp_path / "L00", {"gate_proj": [rec]}, group_size=80)
    with k50.K50Pack(tmp_path / "L00") as pk:
        w, s, b = pk.materialize("gate_proj", 0)
    assert w[0, 0] == (1 | 1 << 12 | 1 << 28 | 2 << 30)
    assert w[0, 1] == 0b10101010             # digits 16..19 = 2
    assert list(w[0, 2:]) == [0, 0, 0]
    assert b[0, 0] == 0xBF80                 # -1.0


def test_bad_packs(tmp_path):
    rng = np.random.default_rng(2)
    with pytest.raises(MoeError):
        k50.K50Pack(tmp_path / "missing")
    k50.write_k50_layer(tmp_path / "L01", {"gate_proj": [_rec(rng, "2", 8, 128)]})
    idx = json.loads((tmp_path / "L01" / "index.json").read_text())
    idx["experts"]["gate_proj"][0]["code_nbytes"] += 4          # rows do not divide evenly
    (tmp_path / "L01" / "index.json").write_text(json.dumps(idx))
    with k50.K50Pack(tmp_path / "L01") as pk:
        with pytest.raises(MoeError):
            pk.record("gate_proj", 0)
        with pytest.raises(MoeError):
            pk.record("gate_proj", 1)                              # no such expert
    (tmp_path / "L01" / "index.json").write_text('{"experts": {"gate_proj": [{"expert": 0, "kind": }]}}')
    with pytest.raises(MoeError):
        k50.K50Pack(tmp_path / "L01")
    # a number beyond int64 is refused, not thrown through the C ABI
    (tmp_path / "L01" / "index.json").write_text('{"experts": {"gate_proj": [{"expert": 0, "code_off": 1' + '0' * 30 + '}]}}')
    with pytest.raises(MoeError):
        k50.K50Pack(tmp_path / "L01")


def test_pool_refuses_wider_codes(tmp_path):
    """The expert kernels run 2-bit codes: a layer with a 4-bit expert is refused (before any
    pinned allocation)."""
    rng = np.random.default_rng(3)
    experts = {p: [_rec(rng, "2", 32, 128), _rec(rng, "4" if p == "up_proj" else "2t", 32, 128)]
               for p in k50.PROJS}
    k50.write_k50_layer(tmp_path / "L02", experts)
    with pytest.raises(ValueError, match="kinds"):
        k50.load_k50_pool(tmp_path / "L02", 2)
