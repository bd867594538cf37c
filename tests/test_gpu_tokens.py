"""The token loop around the stack (server.py:93-199, loader.py:1125-1244) on the GPU:
embedding rows bit-exact, LM-head logits bit-exact against the oracle's fixed-order double sums,
argmax = the first index of the maximum, sampled ids equal to the oracle's Gumbel-max draws and
distributed as softmax(logits / temperature) over the top-p set, and the decode loop feeding
each step's argmax id back (teacher-forced check of every step against the oracle)."""
import dataclasses

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _bf16(rng, shape, std):
    from oracle import oracle as orc
    return orc.f32_to_bf16(rng.normal(0.0, std, shape).astype(np.float32))


def _t(a, dev):
    from moe_offload_b200.synthetic import np_to_bf16_tensor
    return np_to_bf16_tensor(a, dev)


def test_embed_rows_exact_and_bad_id_flagged(dev):
    from moe_offload_b200 import _lib
    from moe_offload_b200.tokens import TokenHead
    rng = np.random.default_rng(1)
    V, H = 1000, 1024
    emb = _bf16(rng, (V, H), 1.0)
    head = TokenHead(_t(emb, dev))
    ids = np.array([0, V - 1, 17, 17, 512], dtype=np.int32)
    out = head.embed(torch.from_numpy(ids).to(dev)).cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(out, emb[ids])
    _lib.call("moe_device_error", 1)
    bad = head.embed(torch.tensor([3, V], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert int(_lib.call("moe_device_error", 1)) & 2
    assert torch.count_nonzero(bad[1]).item() == 0
    assert np.array_equal(bad[0].cpu().view(torch.int16).numpy().view(np.uint16), emb[3])


@pytest.mark.parametrize("V,H,T", [(3000, 3072, 1), (4097, 1032, 3), (777, 256, 4)])
def test_lm_head_bit_exact(dev, V, H, T):
    from oracle import oracle as orc
    from moe_offload_b200.tokens import TokenHead
    rng = np.random.default_rng(V + H + T)
    w = _bf16(rng, (V, H), 0.02)
    x = _bf16(rng, (T, H), 1.0)
    head = TokenHead(_t(_bf16(rng, (V, H), 1.0), dev), _t(w, dev))
    lg = head.logits(_t(x, dev)).cpu().numpy()
    ref = orc.lm_head_logits(w, x)
    assert np.array_equal(lg.view(np.uint32), ref.view(np.uint32))


def test_argmax_first_index_of_maximum(dev):
    from moe_offload_b200.tokens import TokenHead
    rng = np.random.default_rng(5)
    V = 248_320
    head = TokenHead(torch.zeros((V, 8), dtype=torch.bfloat16, device=dev))
    lg = rng.normal(0, 3, (4, V)).astype(np.float32)
    lg[1, [5, 200_000, 248_319]] = 100.0                   # ties: the first index wins
    lg[2, :] = -7.0                                        # all equal
    lg[3, V - 1] = 1e30
    ids = head.sample(torch.from_numpy(lg).to(dev)).cpu().numpy()
    assert ids.tolist() == [int(np.argmax(lg[0])), 5, 0, V - 1]


@pytest.mark.parametrize("V,H,T", [(100_003, 1024, 3), (5000, 3072, 1)])
def test_lm_head_argmax_fused(dev, V, H, T):
    """The fused head + argmax pass: the same logits as moe_lm_head_logits and, per row, the
    first index of their maximum (planted ties between identical head rows included), on two
    calls in a row (the workspace is left zeroed for the next call)."""
    from moe_offload_b200.tokens import TokenHead
    g = torch.Generator(device=dev)
    g.manual_seed(V)
    w = (torch.randn((V, H), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    ref = TokenHead(w).logits(x)
    top = ref.argmax(dim=1)
    w[V - 1] = w[top[0]]                      # a later row equal to row 0's winner
    w[min(7, V - 2)] = w[top[0]]              # an earlier one: it must win
    head = TokenHead(w)
    ref = head.logits(x).cpu().numpy()
    for _ in range(2):
        lg = torch.empty((T, V), dtype=torch.float32, device=dev)
        ids = head.argmax(x, logits=lg).cpu().numpy()
        assert np.array_equal(lg.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        assert ids.tolist() == [int(np.argmax(ref[t])) for t in range(T)]
    assert np.count_nonzero(ref[0] == ref[0].max()) >= 2          # the planted tie is there
    assert head.argmax(x).cpu().numpy().tolist() == ids.tolist()           # without the logits


@pytest.mark.parametrize("temperature,top_p", [(0.7, 1.0), (1.0, 0.9), (1.3, 0.5)])
def test_sampling_matches_oracle(dev, temperature, top_p):
    from oracle import oracle as orc
    from moe_offload_b200.tokens import TokenHead
    rng = np.random.default_rng(11)
    V, H, T = 1000, 512, 4
    w = _bf16(rng, (V, H), 0.05)
    head = TokenHead(_t(w, dev))
    lg = orc.lm_head_logits(w, _bf16(rng, (T, H), 1.0))
    lgd = torch.from_numpy(lg).to(dev)
    agree = total = 0
    for counter in range(50):
        got = head.sample(lgd, temperature, top_p, seed=99, counter=counter).cpu().numpy()
        ref = orc.sample_tokens(lg, temperature, top_p, seed=99, counter=counter)
        agree += int(np.sum(got == ref))
        total += T
    # the same rule and random stream; CUDA's expf / log and the host's may differ in the last
    # bit, which can move a near-tie, so 99 % agreement is required (all agree in practice)
    assert agree >= 0.99 * total, (agree, total)


def test_sampling_distribution_and_top_p_set(dev):
    from moe_offload_b200.tokens import TokenHead
    V, T = 6, 8000
    head = TokenHead(torch.zeros((V, 8), dtype=torch.bfloat16, device=dev))
    base = np.array([2.0, 1.0, 0.5, 0.0, -1.0, -3.0], dtype=np.float32)
    lg = torch.from_numpy(np.tile(base, (T, 1))).to(dev)
    ids = head.sample(lg, 1.0, 1.0, seed=3, counter=0).cpu().numpy()
    p = np.exp(base - base.max())
    p /= p.sum()
    freq = np.bincount(ids, minlength=V) / T
    sigma = np.sqrt(p * (1 - p) / T)
    assert np.all(np.abs(freq - p) <= 5 * sigma + 1e-4), (freq, p)
    # top_p = 0.8: the smallest set of the largest probabilities holding 80 % of the mass
    order = np.argsort(-p)
    k = int(np.searchsorted(np.cumsum(p[order]), 0.8) + 1)
    allowed = set(order[:k].tolist())
    ids = head.sample(lg, 1.0, 0.8, seed=4, counter=1).cpu().numpy()
    assert set(np.unique(ids).tolist()) == allowed
    q = p[order[:k]] / p[order[:k]].sum()
    freq = np.array([np.mean(ids == i) for i in order[:k]])
    assert np.all(np.abs(freq - q) <= 5 * np.sqrt(q * (1 - q) / T) + 1e-4), (freq, q)
    # the same (seed, counter) gives the same draws
    again = head.sample(lg, 1.0, 0.8, seed=4, counter=1).cpu().numpy()
    assert np.array_equal(ids, again)


def test_resident_token_loop_teacher_forced(dev):
    """Every step of the captured loop: the stack's input is the embedding row of the previous
    step's id, the stack matches the oracle layer by layer, and the next id is the oracle's
    argmax of the LM head on the stack's output."""
    from oracle import oracle as orc
    from moe_offload_b200.ops import pow2_normalize
    from moe_offload_b200.stack import PersistentStack
    from moe_offload_b200.synthetic import (ExpertLayer, bf16_tensor_to_np, np_bf16_normal, np_qmatrix,
                                            to_device_qmatrix)
    from moe_offload_b200.tokens import ResidentTokenLoop, TokenHead
    rng = np.random.default_rng(21)
    L, H, I, E, K, V = 2, 1024, 256, 32, 4, 2048
    nl = [dict(router=np_bf16_normal(rng, (E, H), 0.02), g=np_qmatrix(rng, E, I, H), u=np_qmatrix(rng, E, I, H),
               d=np_qmatrix(rng, E, H, I)) for _ in range(L)]
    layers = [ExpertLayer(_t(ly["router"], dev), to_device_qmatrix(ly["g"], dev), to_device_qmatrix(ly["u"], dev),
                          to_device_qmatrix(ly["d"], dev)) for ly in nl]
    st = PersistentStack(layers, K, dev, keep_layer_inputs=True)
    emb, hw = _bf16(rng, (V, H), 1.0), _bf16(rng, (V, H), 0.02)
    loop = ResidentTokenLoop(st, TokenHead(_t(emb, dev), _t(hw, dev)))
    tok = 65
    loop.start(tok)
    for _ in range(5):
        nxt = loop.step()
        hs = bf16_tensor_to_np(st.hs)
        assert np.array_equal(hs[0], emb[tok])
        for li, ly in enumerate(nl):
            xin = pow2_normalize(hs[li][None])
            _, ri, rs = orc.softmax_topk(orc.router_logits(xin, ly["router"], E), K)
            assert np.array_equal(st.inds[li].cpu().numpy().astype(np.uint32), ri[0])
            ref = orc.experts(xin, ri, rs, ly["g"], ly["u"], ly["d"], sb_fp16=True, resid=hs[li][None])["y"]
            a = orc.bf16_to_f32(hs[li + 1]).astype(np.float64) - orc.bf16_to_f32(hs[li])
            b = orc.bf16_to_f32(ref[0]).astype(np.float64) - orc.bf16_to_f32(hs[li])
            assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-2
        assert nxt == int(np.argmax(orc.lm_head_logits(hw, hs[L][None])[0]))
        tok = nxt


def test_engine_token_loop_greedy_and_stream(dev):
    """OffloadEngine with a token head: generate_greedy returns generated ids and text, and
    generate_stream's greedy ids from the same prompt on a reset cache are the same ids."""
    from moe_offload_b200.engine import OffloadEngine
    from moe_offload_b200.synthetic import C2
    cfg = dataclasses.replace(C2, name="tokens_test", layers=3, hidden=512, experts=32, top_k=4, inter=128, seed=7)
    eng = OffloadEngine(budget_pct=50, config=cfg, device=dev, vocab_size=512)
    r = eng.generate_greedy("hello world", max_new_tokens=8, reset_cache_before=True, reset_stats_before=True)
    assert r["prompt_tokens"] == len("hello world".encode())
    assert len(r["generated_ids"]) == 8 and all(0 <= i < 512 for i in r["generated_ids"])
    assert r["generated_text"] == eng.tokenizer.decode(r["generated_ids"])
    eng.reset_caches()
    got = list(eng.generate_stream(eng.tokenizer.encode("hello world"), 8, stop_ids=[]))
    eos = eng.tokenizer.eos_token_id
    want = r["generated_ids"][:r["generated_ids"].index(eos)] if eos in r["generated_ids"] else r["generated_ids"]
    assert got == want
    t = eng._last_timings
    assert set(t) == {"prefill_s", "decode_s", "decode_tok_per_s", "stopped_by_token"}
    # sampled: reproducible for a seed, and stops at max_tokens
    eng.reset_caches()
    s1 = list(eng.generate_stream([1, 2, 3], 6, temperature=0.8, top_p=0.9, seed=5))
    eng.reset_caches()
    s2 = list(eng.generate_stream([1, 2, 3], 6, temperature=0.8, top_p=0.9, seed=5))
    assert s1 == s2 and len(s1) <= 6
    eng.close()
