"""The hook surface (moe_offload_b200.hooks: install_offload_hooks / hooked_layer_call,
loader.py:827-1001) and CachedSwitchGLU built from a shard (loader.py:311).

A hooked model (layer 0 resident, layers 1.. behind LRU caches of a few slots, prefetch on)
gives the same bits as the same model fully resident and un-hooked, token after token, with
and without hyper-connection mixers and shared experts. Its cache calls, recorded as they are
made, replayed in the same order into the reference's own expert_io.c (oracle/_ref) give the
same slot ids, 18 counters and final LRU order."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libexpert_io_ref.so")
u64 = ctypes.c_uint64
L, E, H, I, K, CAP, HC, R, IS = 4, 64, 512, 256, 8, 16, 4, 64, 128


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _weights(seed, with_hc, with_shared):
    from moe_offload_b200.synthetic import np_bf16_normal, np_qmatrix
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(L):
        w = dict(router=np_bf16_normal(rng, (E, H), 0.02), g=np_qmatrix(rng, E, I, H), u=np_qmatrix(rng, E, I, H),
                 d=np_qmatrix(rng, E, H, I))
        if with_shared:
            w["sh"] = [np_qmatrix(rng, 1, IS, H, 4, 64, False), np_qmatrix(rng, 1, IS, H, 4, 64, False),
                       np_qmatrix(rng, 1, H, IS, 4, 64, False), np_qmatrix(rng, 1, 1, H, 8, 64, False)]
        if with_hc:
            w["hc"] = (np_bf16_normal(rng, (HC * H,), 0.1), np_qmatrix(rng, 1, R, HC * H, 8, 64, False),
                       np_qmatrix(rng, 1, HC * H, R, 8, 64, False), np_qmatrix(rng, 1, HC, HC * H, 8, 64, False))
        out.append(w)
    return out


def _model(ws, dev, cached, expert_bytes=1536000):
    from moe_offload_b200.hooks import HyperConnection, MoEBlock, MoEDecoderLayer, MoEModel, SharedExpert
    from moe_offload_b200.offload import CachedSwitchGLU, HostExpertPool
    from moe_offload_b200.synthetic import ExpertLayer, np_to_bf16_tensor, to_device_qmatrix

    def q2(t, bits=8):            # [1, rows, cols] numpy triple -> 2-D QMatrix (bf16 scales)
        return to_device_qmatrix(tuple(a[0] for a in t), dev, bits=bits, sb_fp16=False)

    layers = []
    ps = torch.cuda.Stream(device=dev)
    for l, w in enumerate(ws):
        res = ExpertLayer(np_to_bf16_tensor(w["router"], dev), to_device_qmatrix(w["g"], dev),
                          to_device_qmatrix(w["u"], dev), to_device_qmatrix(w["d"], dev))
        sw = res
        if cached and l > 0:
            sw = CachedSwitchGLU(None, l, CAP, pool=HostExpertPool.from_layer(res), device=dev, top_k=K,
                                 expert_bytes=expert_bytes, prefetch_stream=ps)
        sh = None
        if "sh" in w:
            sh = SharedExpert(q2(w["sh"][0], 4), q2(w["sh"][1], 4), q2(w["sh"][2], 4), q2(w["sh"][3]))
        hc = None
        if "hc" in w:
            n, dn, up, inj = w["hc"]
            hc = HyperConnection(np_to_bf16_tensor(n, dev), q2(dn), q2(up), q2(inj))
        layers.append(MoEDecoderLayer(MoEBlock(res.router, sw, K, sh), hc))
    return MoEModel(layers)


def _record(model):
    """Wraps every cache's step and start_prefetch to log (op, layer, device tensor copy)."""
    log = []
    for layer in model.layers[1:]:
        c = layer.mlp.switch_mlp
        step0, pref0 = c.step, c.start_prefetch

        def step(indices, c=c, step0=step0):
            slots = step0(indices)
            log.append(("step", c.layer_idx, indices.reshape(-1).clone(), slots.reshape(-1).clone()))
            return slots

        def pref(pred, max_fetch=3, c=c, pref0=pref0):
            log.append(("pref", c.layer_idx, pred.reshape(-1).clone(), max_fetch))
            return pref0(pred, max_fetch)

        c.step, c.start_prefetch = step, pref
    return log


@pytest.mark.parametrize("with_hc,with_shared", [(False, False), (False, True), (True, True)])
def test_hooked_decode_matches_resident_model(dev, with_hc, with_shared):
    from moe_offload_b200.hooks import install_offload_hooks
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    ws = _weights(5, with_hc, with_shared)
    hooked = _model(ws, dev, cached=True)
    plain = _model(ws, dev, cached=False)
    install_offload_hooks(hooked, prefetch_enabled=True, prefetch_top_m=12, prefetch_cap=3)
    log = _record(hooked)
    rng = np.random.default_rng(7)
    W = HC * H if with_hc else H
    for t in range(24):
        h = np_to_bf16_tensor(np_bf16_normal(rng, (1, W)), dev)
        ya = hooked(h)
        yb = plain(h)
        torch.cuda.synchronize()
        assert torch.equal(ya, yb), t
    # the order of the cache calls: per token prefetch(1) after layer 0, then for each cached
    # layer its step followed by the next layer's prefetch
    ops = [(op, l) for op, l, *_ in log[:2 * (L - 1)]]
    assert ops == [("pref", 1), ("step", 1), ("pref", 2), ("step", 2), ("pref", 3), ("step", 3)]
    # prefill rows through the hooked model: the plain path with the caches' prefill
    hp = np_to_bf16_tensor(np_bf16_normal(rng, (40, W)), dev)
    ya, yb = hooked(hp), plain(hp)
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


@pytest.mark.skipif(not os.path.exists(REF_LIB), reason="reference library not built (oracle/_ref)")
def test_hooked_cache_calls_replay_in_reference(dev):
    from moe_offload_b200.hooks import install_offload_hooks
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    ws = _weights(11, False, False)
    model = _model(ws, dev, cached=True)
    install_offload_hooks(model, prefetch_enabled=True, prefetch_top_m=12, prefetch_cap=3)
    log = _record(model)
    rng = np.random.default_rng(3)
    for t in range(64):
        model(np_to_bf16_tensor(np_bf16_normal(rng, (1, H)), dev))
        if t == 31:
            model._prefetch_enabled = False       # a stretch without prefetch
        if t == 47:
            model._prefetch_enabled = True
    torch.cuda.synchronize()
    ref = ctypes.CDLL(REF_LIB)
    zeros9 = (u64 * 9)()
    bufs = {l: (ctypes.c_uint32 * 16)() for l in range(1, L)}
    base = 20                                   # layer ids apart from other tests in the process
    for l in range(1, L):
        ref.c_layer_init(base + l, -1, CAP, zeros9, zeros9, zeros9, u64(ctypes.addressof(bufs[l])))
    n_pref = 0
    for op, l, a, b in log:
        v = a.cpu().numpy()
        if op == "step":
            arr = (ctypes.c_uint32 * K)(*v.astype(np.uint32).tolist())
            ref.c_layer_step_decode_ex(base + l, arr, K, 1)
            assert list(bufs[l])[:K] == b.cpu().numpy().tolist(), (l, "slot ids differ")
        else:
            n_pref += 1
            arr = (ctypes.c_int32 * len(v))(*v.astype(np.int32).tolist())
            ref.c_layer_start_prefetch(base + l, arr, len(v), b)
    assert n_pref > 0
    for l in range(1, L):
        c = model.layers[l].mlp.switch_mlp
        st = (u64 * 18)()
        ref.c_layer_get_stats(base + l, st)
        assert c.raw_stats() == list(st), (l, "counters differ")
        oe, os_, cnt = (ctypes.c_int32 * 512)(), (ctypes.c_int32 * 512)(), ctypes.c_int(0)
        ref.c_layer_get_lru_state(base + l, oe, os_, ctypes.byref(cnt))
        assert c.get_lru_state() == (list(oe)[:cnt.value], list(os_)[:cnt.value]), (l, "LRU order differs")


def test_cached_switch_glu_from_shard(dev, tmp_path):
    """CachedSwitchGLU(shard_path, layer_idx, capacity), the reference's constructor: the
    pool is read from the experts-XX.safetensors shard, and its outputs equal the same experts
    resident in HBM."""
    from moe_offload_b200 import checkpoint as ck
    from moe_offload_b200 import ops
    from moe_offload_b200.offload import CachedSwitchGLU
    from moe_offload_b200.synthetic import np_bf16_normal, np_qmatrix, np_to_bf16_tensor, to_device_qmatrix
    rng = np.random.default_rng(17)
    mats = [np_qmatrix(rng, E, I, H, sb_fp16=False), np_qmatrix(rng, E, I, H, sb_fp16=False),
            np_qmatrix(rng, E, H, I, sb_fp16=False)]
    tm = [tuple(torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a.view(np.int16)).view(
        torch.int32 if a.dtype == np.uint32 else torch.bfloat16) for a in m) for m in mats]
    path = tmp_path / ck.shard_name(2)
    ck.write_expert_shard(path, 2, tm)
    torch.cuda.set_device(dev)
    cache = CachedSwitchGLU(path, 2, 12)
    assert (cache.layer_idx, cache.capacity, cache.K, cache.shard_path) == (2, 12, 10, path)
    g, u, d = (to_device_qmatrix(m, dev, sb_fp16=False) for m in mats)
    for step in range(6):
        x = np_to_bf16_tensor(np_bf16_normal(rng, (1, 1, H)), dev)
        eids = torch.from_numpy(rng.choice(E, size=10, replace=False).astype(np.int32)).to(dev).view(1, 1, 10)
        y = cache(x, eids)
        act = ops.experts_gateup(x.view(1, H), eids.view(1, 10), g, u)
        _, yk = ops.experts_down(act, eids.view(1, 10), d, None, want_yk=True)
        assert torch.equal(y.view(10, H), yk.view(10, H)), step
    st = cache.get_layer_stats()
    assert st["decode_requests"] == 60 and st["layer"] == 2
