"""Host side of the token loop: the byte tokenizer, and the oracle's LM head and sampling rule
pinned against their definitions (plain double matmul; the reference's sort-based top-p mask,
server.py:93-110, on inputs without boundary ties; categorical frequencies)."""
import numpy as np
import pytest


def test_byte_tokenizer_round_trip():
    from moe_offload_b200.tokens import ByteTokenizer
    tok = ByteTokenizer(600)
    assert tok.eos_token_id == 599
    ids = tok.encode("héllo, wörld")
    assert all(0 <= i < 256 for i in ids)
    assert tok.decode(ids + [599, 300]) == "héllo, wörld"
    with pytest.raises(ValueError):
        ByteTokenizer(200)


def test_oracle_lm_head_is_the_rounded_double_product():
    from oracle import oracle as orc
    rng = np.random.default_rng(0)
    for V, H, T in ((300, 512, 2), (129, 1032, 1)):
        w = orc.f32_to_bf16(rng.normal(0, 0.02, (V, H)).astype(np.float32))
        x = orc.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
        ref = (orc.bf16_to_f32(x).astype(np.float64) @ orc.bf16_to_f32(w).astype(np.float64).T).astype(np.float32)
        assert np.array_equal(orc.lm_head_logits(w, x), ref)


def _reference_top_p_mask(scaled: np.ndarray, top_p: float) -> np.ndarray:
    """server.py:99-106: sort descending, softmax, cumsum, mask (cum - p) >= top_p."""
    order = np.argsort(-scaled, kind="stable")
    sl = scaled[order].astype(np.float64)
    p = np.exp(sl - sl.max())
    p /= p.sum()
    cum = np.cumsum(p)
    keep_sorted = (cum - p) < top_p
    keep = np.zeros(scaled.shape[0], dtype=bool)
    keep[order[keep_sorted]] = True
    return keep


def test_oracle_top_p_set_matches_reference_rule():
    from oracle import oracle as orc
    rng = np.random.default_rng(3)
    for trial in range(40):
        V = int(rng.integers(5, 400))
        lg = rng.normal(0, 2.5, (1, V)).astype(np.float32)
        temperature, top_p = float(rng.uniform(0.3, 1.5)), float(rng.uniform(0.05, 0.97))
        want = _reference_top_p_mask(lg[0] / np.float32(temperature), top_p)
        # every draw lands in the reference's candidate set, and over many draws covers it
        seen = set()
        for counter in range(300):
            i = int(orc.sample_tokens(lg, temperature, top_p, seed=trial, counter=counter)[0])
            assert want[i], (trial, i)
            seen.add(i)
        if want.sum() <= 3:
            assert seen == set(np.flatnonzero(want).tolist())


def test_oracle_sampling_frequencies_and_greedy():
    from oracle import oracle as orc
    base = np.array([[1.5, 0.2, -0.3, 0.9]], dtype=np.float32)
    assert orc.sample_tokens(base)[0] == 0
    assert orc.sample_tokens(np.array([[1.0, 3.0, 3.0, 2.0]], dtype=np.float32))[0] == 1   # first maximum
    n = 6000
    ids = np.array([orc.sample_tokens(base, 0.8, 1.0, seed=1, counter=c)[0] for c in range(n)])
    p = np.exp(base[0] / 0.8 - (base[0] / 0.8).max())
    p /= p.sum()
    freq = np.bincount(ids, minlength=4) / n
    assert np.all(np.abs(freq - p) <= 5 * np.sqrt(p * (1 - p) / n))
