"""A cached layer whose pinned pool comes from a K50 pack (experts of kinds tern, 2t and 2)
decodes bit for bit like the same weights from an experts-XX.safetensors shard and like the
same experts resident in HBM."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
E, H, I, K, CAP, GS = 24, 640, 320, 6, 12, 64


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _bf16(rng, shape, lo, hi):
    f = rng.uniform(lo, hi, size=shape).astype(np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def test_k50_pool_decodes_like_safetensors(dev, tmp_path):
    from moe_offload_b200 import checkpoint as ck
    from moe_offload_b200 import k50, ops
    from moe_offload_b200.offload import CachedSwitchGLU
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor, to_device_qmatrix
    rng = np.random.default_rng(5)
    kinds = ["tern", "2t", "2"]
    recs = {p: [] for p in k50.PROJS}
    mlx = {p: [[], [], []] for p in k50.PROJS}       # materialised codes / scales / biases per expert
    for p, (rows, cols) in zip(k50.PROJS, ((I, H), (I, H), (H, I))):
        for e in range(E):
            kind = kinds[(e + len(p)) % 3]
            sc = _bf16(rng, (rows, cols // GS), 0.005, 0.03)
            d = rng.integers(0, 4 if kind == "2" else 3, size=(rows, cols), dtype=np.uint32)
            words = np.bitwise_or.reduce(d.reshape(rows, cols // 16, 16) << (np.arange(16, dtype=np.uint32) * 2),
                                         axis=-1).astype(np.uint32)
            if kind == "tern":
                rec = {"kind": kind, "shape": (rows, cols), "scales": sc, "digits": d.astype(np.uint8)}
                bias = sc ^ 0x8000
            elif kind == "2t":
                bias = sc ^ 0x8000
                rec = {"kind": kind, "shape": (rows, cols), "scales": sc, "codes": words, "biases": bias}
            else:
                bias = _bf16(rng, (rows, cols // GS), -0.02, 0.02)
                rec = {"kind": kind, "shape": (rows, cols), "scales": sc, "codes": words, "biases": bias}
            recs[p].append(rec)
            for j, a in enumerate((words, sc, bias)):
                mlx[p][j].append(a)
    k50.write_k50_layer(k50.layer_dir(tmp_path, 4), recs)
    mats = [tuple(np.stack(mlx[p][j]) for j in range(3)) for p in k50.PROJS]
    tm = [(torch.from_numpy(w.view(np.int32)), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
           torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)) for w, s, b in mats]
    shard = tmp_path / ck.shard_name(4)
    ck.write_expert_shard(shard, 4, tm)

    pool = k50.load_k50_pool(k50.layer_dir(tmp_path, 4), E)
    for a, b in zip(pool.t, [t for m in tm for t in m]):
        assert torch.equal(a.view(torch.int16) if a.dtype != torch.int32 else a,
                           b.view(torch.int16) if b.dtype != torch.int32 else b)
    a = CachedSwitchGLU(None, 4, CAP, pool=pool, device=dev, top_k=K)
    b = CachedSwitchGLU(shard, 4, CAP, device=dev, top_k=K)
    g, u, d = (to_device_qmatrix(m, dev, sb_fp16=False) for m in mats)
    for step in range(12):
        x = np_to_bf16_tensor(np_bf16_normal(rng, (1, 1, H)), dev)
        eids = torch.from_numpy(rng.choice(E, size=K, replace=False).astype(np.int32)).to(dev).view(1, 1, K)
        ya, yb = a(x, eids), b(x, eids)
        act = ops.experts_gateup(x.view(1, H), eids.view(1, K), g, u)
        _, yr = ops.experts_down(act, eids.view(1, K), d, None, want_yk=True)
        torch.cuda.synchronize()
        assert torch.equal(ya, yb), step
        assert torch.equal(ya.view(K, H), yr.view(K, H)), step
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0
