"""Expert shards in the reference's checkpoint layout (moe_offload_b200.checkpoint): write a
shard, read it back, cross-check with the safetensors package, locate expert rows the way the
reference's CachedSwitchGLU does (loader.py:329-366), and fill slots from the shard with the
P1 scheduler (file source, as the reference's engine does; the only test here that needs a GPU)."""
import os

import numpy as np
import pytest
import torch

from moe_offload_b200 import checkpoint as ck

E, H, I, BITS, GS = 8, 256, 128, 2, 64


def _mats(seed, sb=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    out = []
    for rows, cols in ((I, H), (I, H), (H, I)):
        w = torch.randint(-(2 ** 31), 2 ** 31 - 1, (E, rows, cols * BITS // 32), dtype=torch.int32, generator=g)
        s = (torch.rand((E, rows, cols // GS), generator=g) * 0.04 + 0.001).to(sb)
        b = (torch.randn((E, rows, cols // GS), generator=g) * 0.01).to(sb)
        out.append((w, s, b))
    return out


@pytest.fixture
def shard(tmp_path):
    mats = _mats(1)
    path = tmp_path / ck.shard_name(3)
    ck.write_expert_shard(path, 3, mats)
    return path, mats


def test_roundtrip_and_params(shard):
    path, mats = shard
    ts = ck.load_expert_tensors(path, 3, GS, pin=False)
    flat = [t for m in mats for t in m]
    assert len(ts) == 9
    for a, b in zip(ts, flat):
        assert a.dtype == b.dtype and a.shape == b.shape
        assert torch.equal(a.view(torch.int16) if a.dtype != torch.int32 else a,
                           b.view(torch.int16) if b.dtype != torch.int32 else b)
    q = ck.quant_params(path, 3, GS)
    assert (q["bits"], q["experts"], q["inter"], q["hidden"], q["down_rows"], q["sb_dtype"]) == (BITS, E, I, H, H, "BF16")


def test_safetensors_package_reads_the_shard(shard):
    safetensors = pytest.importorskip("safetensors")
    from safetensors import safe_open
    path, mats = shard
    flat = [t for m in mats for t in m]
    with safe_open(str(path), framework="pt") as f:
        for i, proj in enumerate(ck.PROJS):
            for j, part in enumerate(ck.PARTS):
                t = f.get_tensor(ck.NAME.format(layer=3, proj=proj, part=part))
                want = flat[3 * i + j]
                assert t.numel() == want.numel()
                assert np.array_equal(t.contiguous().view(torch.uint8).numpy(), want.view(torch.uint8).numpy())


def test_rows_at_reference_offsets(shard):
    """Expert e's row of tensor t is row_bytes[t] bytes at offsets[t] + e * row_bytes[t]
    (loader.py:341-344: abs_offset = 8 + header + data_offsets[0], row = bytes / shape[0])."""
    path, mats = shard
    offs, rb = ck.shard_rows(path, 3, GS)
    flat = [t for m in mats for t in m]
    fd = os.open(path, os.O_RDONLY)
    try:
        for t, (o, r) in enumerate(zip(offs, rb)):
            assert r == flat[t][0].numel() * flat[t].element_size()
            for e in (0, 5, E - 1):
                raw = os.pread(fd, r, o + e * r)
                assert raw == flat[t][e].contiguous().view(torch.uint8).numpy().tobytes()
    finally:
        os.close(fd)


@pytest.mark.gpu
def test_p1_scheduler_fills_slots_from_the_shard(shard):
    """Rows at the shard's offsets through the P1 scheduler (its state lives on the GPU)."""
    from moe_offload_b200.io_sched import P1IoScheduler
    path, mats = shard
    offs, rb = ck.shard_rows(path, 3, GS)
    flat = [t for m in mats for t in m]
    cap = 4
    bufs = [np.zeros(cap * r, dtype=np.uint8) for r in rb]
    inds = np.zeros(8, dtype=np.uint32)
    fd = os.open(path, os.O_RDONLY)
    s = P1IoScheduler()
    try:
        s.layer_init(3, fd, cap, 9, offs, rb, [b.ctypes.data for b in bufs], inds.ctypes.data)
        s.set_wait_reader_callback(lambda layer: s.unpin_layer_slots(layer))
        for eids in ([1, 6], [6, 2, 7], [0, 3], [5, 1]):
            n, slots = s.step_decode(3, eids)
            if n:
                s.wait_layer_urgent(3)
            for e, sl in zip(eids, slots):
                for t, r in enumerate(rb):
                    assert bufs[t][sl * r:(sl + 1) * r].tobytes() == flat[t][e].contiguous().view(torch.uint8).numpy().tobytes()
            s.unpin_layer_slots(3)
        assert s.get_layer_stats(3)["bytes"] > 0
    finally:
        s.close()
        os.close(fd)


def test_fp16_scales_and_bad_shards(tmp_path):
    mats = _mats(2, torch.float16)
    p = tmp_path / ck.shard_name(1)
    ck.write_expert_shard(p, 1, mats)
    assert ck.quant_params(p, 1)["sb_dtype"] == "F16"
    with pytest.raises(KeyError):
        ck.expert_tensors(p, 2)                      # no such layer in the shard
    bad = [list(m) for m in mats]
    bad[2][1] = bad[2][1].to(torch.bfloat16)          # down scales of another type
    q = tmp_path / "bad.safetensors"
    ck.write_expert_shard(q, 1, bad)
    with pytest.raises(ValueError):
        ck.expert_tensors(q, 1)
