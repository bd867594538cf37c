"""Expert-parallel decode (moe_ep_decode_layer): on one GPU the single-rank form must equal the
single-GPU decode layer bit for bit (below 32 tokens; from 32 tokens up, the grouped-GEMM
path, the single-GPU prefill layer); on two GPUs (when present) every rank, holding half of
the experts, must produce the same bits as the single-GPU layer (tests/ep_worker.py)."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


@pytest.mark.parametrize("T", [1, 5, 31, 32, 40])
def test_ep_single_rank_equals_decode_layer(dev, T):
    from moe_offload_b200 import _lib, ops
    from moe_offload_b200.ep import ExchangeBuffers, ep_decode_layer
    from moe_offload_b200.synthetic import ExpertLayer, np_bf16_normal, np_qmatrix, np_to_bf16_tensor, to_device_qmatrix
    rng = np.random.default_rng(40 + T)
    E, H, I, K = 64, 2048, 768, 8
    ly = ExpertLayer(np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev),
                     to_device_qmatrix(np_qmatrix(rng, E, I, H), dev), to_device_qmatrix(np_qmatrix(rng, E, I, H), dev),
                     to_device_qmatrix(np_qmatrix(rng, E, H, I), dev))
    xbuf = ExchangeBuffers(T, K, H, dev)
    try:
        for rep in range(3):
            x = np_to_bf16_tensor(np_bf16_normal(rng, (T, H)), dev)
            o = ep_decode_layer(x, ly, E, 0, K, xbuf, norm=True, resid=x)
            if T < 32:
                r = ops.decode_layer(x, ly.router, ly.gate, ly.up, ly.down, K, norm=True, resid=x)
            else:
                r = ops.prefill_layer(x, ly.router, ly.gate, ly.up, ly.down, K, norm=True, resid=x)
            torch.cuda.synchronize()
            for key in ("inds", "scores", "y"):
                assert torch.equal(o[key], r[key]), f"call {rep}: {key} differs"
    finally:
        xbuf.close()
    assert int(_lib.call("moe_device_error", 1)) == 0


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_ranks_bit_exact_with_single_gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "ep_worker.py")]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    assert p.stdout.count('"bad": []') == 2, p.stdout[-3000:]
