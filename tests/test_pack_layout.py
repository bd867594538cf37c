"""The packed expert layout: the numpy restatement against the layout's definition (CPU),
and the CUDA packer against the restatement (GPU)."""
import numpy as np
import pytest

from packref import pack_experts_np


def _mats(rng, E, H, I):
    from moe_offload_b200.synthetic import np_qmatrix
    return np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, I, H), np_qmatrix(rng, E, H, I)


def test_pack_np_matches_definition():
    rng = np.random.default_rng(3)
    E, H, I = 3, 512, 256
    g, u, d = _mats(rng, E, H, I)
    pk = pack_experts_np(g, u, d, H, I)
    assert pk.shape == (E, (I // 64) * 60 * H)
    gb, ub = 60 * H, 5 * H
    for _ in range(200):
        e, G, uu = rng.integers(E), rng.integers(I // 64), rng.integers(8)
        gg, Gj = rng.integers(8), rng.integers(H // 64)
        j, t = Gj // 4, Gj % 4
        row = 64 * G + 8 * uu + gg
        ci = (j * 8 + gg) * 4 + t
        blk = pk[e, G * gb: (G + 1) * gb]
        gate = blk[uu * ub + ci * 16: uu * ub + ci * 16 + 16].view(np.uint32)
        up = blk[uu * ub + 2 * H + ci * 16: uu * ub + 2 * H + ci * 16 + 16].view(np.uint32)
        assert np.array_equal(gate, g[0][e, row, 4 * Gj: 4 * Gj + 4])
        assert np.array_equal(up, u[0][e, row, 4 * Gj: 4 * Gj + 4])
        rec = blk[uu * ub + 4 * H + ci * 8: uu * ub + 4 * H + ci * 8 + 8].view(np.uint16)
        assert list(rec) == [g[1][e, row, Gj], g[2][e, row, Gj], u[1][e, row, Gj], u[2][e, row, Gj]]
        r = rng.integers(H)
        assert np.array_equal(blk[40 * H + 16 * r: 40 * H + 16 * r + 16].view(np.uint32), d[0][e, r, 4 * G: 4 * G + 4])
        assert list(blk[56 * H + 4 * r: 56 * H + 4 * r + 4].view(np.uint16)) == [d[1][e, r, G], d[2][e, r, G]]


@pytest.mark.gpu
def test_cuda_pack_matches_np():
    import torch
    from moe_offload_b200.stack import pack_layer_experts
    from moe_offload_b200.synthetic import ExpertLayer, np_bf16_normal, np_to_bf16_tensor, to_device_qmatrix
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(4)
    for E, H, I in [(5, 1024, 256), (3, 3072, 768)]:
        g, u, d = _mats(rng, E, H, I)
        layer = ExpertLayer(np_to_bf16_tensor(np_bf16_normal(rng, (E, H)), dev), to_device_qmatrix(g, dev),
                            to_device_qmatrix(u, dev), to_device_qmatrix(d, dev))
        got = pack_layer_experts(layer, dev).cpu().numpy()
        assert np.array_equal(got, pack_experts_np(g, u, d, H, I))
