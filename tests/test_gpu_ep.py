"""Expert parallelism (moe_ep_decode_layer: tokens replicated; moe_ep_a2a_layer: tokens sharded,
routed all-to-all): on one GPU the single-rank forms must equal the single-GPU decode layer bit
for bit (below 32 tokens; from 32 tokens up, the grouped-GEMM path, the single-GPU prefill
layer); a peer that never signals must make the bounded waits run out with an error status;
on two GPUs (when present) every rank, holding half of the experts, must produce the same bits
as the single-GPU layers (tests/ep_worker.py)."""
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


def _layer(rng, dev, E, H, I):
    from moe_offload_b200.synthetic import ExpertLayer, np_bf16_normal, np_qmatrix, np_to_bf16_tensor, to_device_qmatrix
    return ExpertLayer(np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev),
                       to_device_qmatrix(np_qmatrix(rng, E, I, H), dev), to_device_qmatrix(np_qmatrix(rng, E, I, H), dev),
                       to_device_qmatrix(np_qmatrix(rng, E, H, I), dev))


@pytest.mark.parametrize("T", [1, 8, 31, 32, 96])
def test_ep_a2a_single_rank_equals_single_gpu_layers(dev, T):
    """The token-sharded layer with one rank (every token and expert local, the same dispatch,
    expert and combine kernels as with N ranks) equals the single-GPU decode layer (T < 32) or
    prefill layer (T >= 32) bit for bit, three calls in a row (the epochs advance)."""
    from moe_offload_b200 import _lib, ops
    from moe_offload_b200.ep import ExchangeBuffers, ep_a2a_layer
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(70 + T)
    E, H, I, K = 64, 2048, 768, 8
    ly = _layer(rng, dev, E, H, I)
    xbuf = ExchangeBuffers(T, K, H, dev, a2a=True)
    try:
        for rep in range(3):
            x = np_to_bf16_tensor(np_bf16_normal(rng, (T, H)), dev)
            o = ep_a2a_layer(x, ly, E, [0, E], K, T, xbuf, norm=True, resid=x)
            ref = ops.decode_layer if T < 32 else ops.prefill_layer
            r = ref(x, ly.router, ly.gate, ly.up, ly.down, K, norm=True, resid=x)
            torch.cuda.synchronize()
            for key in ("inds", "scores", "y"):
                assert torch.equal(o[key], r[key]), f"call {rep}: {key} differs"
    finally:
        xbuf.close()
    assert int(_lib.call("moe_device_error", 1)) == 0


def test_ep_a2a_stack_graph_equals_layer_chain(dev):
    """EPA2AStack (one rank, the step captured as one CUDA graph) against a chain of
    single-GPU prefill layers, token after token."""
    from moe_offload_b200 import _lib, ops
    from moe_offload_b200.ep import EPA2AStack
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(5)
    L, T, E, H, I, K = 3, 48, 64, 1024, 256, 6
    layers = [_layer(rng, dev, E, H, I) for _ in range(L)]
    st = EPA2AStack(layers, E, [0, E], K, T, dev)
    try:
        for _ in range(3):
            x = np_to_bf16_tensor(np_bf16_normal(rng, (T, H)), dev)
            y = st.step_device(x).clone()
            h = x
            for ly in layers:
                h = ops.prefill_layer(h, ly.router, ly.gate, ly.up, ly.down, K, norm=True, resid=h)["y"]
            torch.cuda.synchronize()
            assert torch.equal(y, h)
    finally:
        st.close()
    assert int(_lib.call("moe_device_error", 1)) == 0


def _lone_rank_buffers(nbytes, dev):
    """This rank's exchange buffer and a second buffer standing in for rank 1, whose kernels
    never run: nothing ever signals rank 0, so every wait for rank 1 must run out."""
    import ctypes

    from moe_offload_b200._lib import call
    ptrs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        h = (ctypes.c_ubyte * 64)()
        call("moe_ep_buffer_alloc", nbytes, ctypes.byref(p), h)
        ptrs.append(p.value)
    return ptrs, torch.tensor(ptrs, dtype=torch.int64, device=dev)


@pytest.mark.parametrize("a2a", [False, True])
def test_ep_peer_that_never_signals_times_out(dev, a2a):
    """A peer rank that never runs its exchange: the bounded waits (2 s of %globaltimer) run
    out, the kernel records MOE_DEVERR_PEER_TIMEOUT in the device error word and returns, and
    the context stays usable (a later single-GPU layer still works)."""
    from moe_offload_b200 import _lib, ops
    from moe_offload_b200._lib import call
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(9)
    T, E, H, I, K = 8, 64, 1024, 256, 6
    ly = _layer(rng, dev, E, H, I)
    _lib.call("moe_device_error", 1)                     # start from a clear error word
    x = np_to_bf16_tensor(np_bf16_normal(rng, (T, H)), dev)
    inds = torch.empty((T, K), dtype=torch.int32, device=dev)
    scores = torch.empty((T, K), dtype=torch.bfloat16, device=dev)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    g, u, d = ly.gate, ly.up, ly.down
    s = torch.cuda.current_stream(dev).cuda_stream
    if a2a:
        nbytes = int(call("moe_ep_a2a_buffer_bytes", T, K, H, 2))
        ptrs, peers = _lone_rank_buffers(nbytes, dev)
        ws = torch.zeros(int(call("moe_ep_a2a_workspace_bytes", T, H, I, E, K, 2)), dtype=torch.uint8, device=dev)
        import ctypes
        ef = (ctypes.c_int * 3)(0, E // 2, E)
        from moe_offload_b200.ep import shard_layer
        loc = shard_layer(ly, 0, E // 2)
        n = T // 2                                       # rank 0 owns the first half of the batch
        call("moe_ep_a2a_layer", x.data_ptr(), T, H, I, E, K, ef, loc.router.data_ptr(), loc.gate.w.data_ptr(),
             loc.gate.s.data_ptr(), loc.gate.b.data_ptr(), loc.up.w.data_ptr(), loc.up.s.data_ptr(),
             loc.up.b.data_ptr(), loc.down.w.data_ptr(), loc.down.s.data_ptr(), loc.down.b.data_ptr(), 1, 1,
             x.data_ptr(), peers.data_ptr(), ptrs[0], 0, 2, inds.data_ptr(), scores.data_ptr(), y.data_ptr(),
             ws.data_ptr(), ws.numel(), s)
        assert n == 4
    else:
        nbytes = int(call("moe_ep_buffer_bytes", T, K, H))
        ptrs, peers = _lone_rank_buffers(nbytes, dev)
        ws = torch.zeros(int(call("moe_ep_workspace_bytes", T, H, I, E, K)), dtype=torch.uint8, device=dev)
        call("moe_ep_decode_layer", x.data_ptr(), T, H, I, E, K, 0, E, ly.router.data_ptr(), g.w.data_ptr(),
             g.s.data_ptr(), g.b.data_ptr(), u.w.data_ptr(), u.s.data_ptr(), u.b.data_ptr(), d.w.data_ptr(),
             d.s.data_ptr(), d.b.data_ptr(), 1, 1, x.data_ptr(), peers.data_ptr(), 0, 2, inds.data_ptr(),
             scores.data_ptr(), y.data_ptr(), ws.data_ptr(), ws.numel(), s)
    torch.cuda.synchronize()                             # returns: the waits are bounded
    err = int(_lib.call("moe_device_error", 1))
    assert err & 4, f"device error word {err}: no peer timeout recorded"
    for p in ptrs:
        call("moe_ep_buffer_free", p)
    r = ops.decode_layer(x, ly.router, g, u, d, K, norm=True)        # the context still works
    torch.cuda.synchronize()
    assert r["inds"].shape == (T, K)
    assert int(_lib.call("moe_device_error", 1)) == 0
