"""moe_router_topk_noalloc -- the router entry point for callers that cannot allocate device
memory (a C/FFI host holding only device pointers, or a process whose device memory is fully
taken by another allocator). It keeps its scratch in a fixed array inside the library image,
so this test calls it through the C ABI with nothing but input/output buffers and checks it
against the workspace entry point moe_router_topk on two calls in a row.

Collected last on purpose (file name) so a stop-at-first-failure run has already run the
rest; it also passes alone in a fresh process (the first call does the per-device set-up).
Tolerance: bit-exact, the same bar the router tests use (indices, scores, logits, pred)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc_call(lib, x, w, wn, T, H, E, K, M, inds, scores, pred, logits):
    P = ctypes.c_void_p
    fn = lib.moe_router_topk_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, P, P, P, ctypes.c_int, P, P, P, P, P, P, P]
    rc = fn(x.data_ptr(), T, H, E, K, w.data_ptr(), None, None, 16, 64, 0, wn.data_ptr(), None, None, M, None,
            None if logits is None else logits.data_ptr(), None, inds.data_ptr(), scores.data_ptr(),
            pred.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return rc


def test_noalloc_router_matches_workspace_router():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from moe_offload_b200 import _lib, ops
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor

    dev = torch.device("cuda:0")
    lib = ctypes.CDLL(_lib.LIB_PATH)
    rng = np.random.default_rng(2024)
    T, H, E, K, M = 2, 3072, 512, 10, 12
    w = np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev)
    wn = np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev)
    lib.moe_last_error.restype = ctypes.c_char_p
    for call in range(2):                       # two calls in a row reuse the shared scratch
        x = np_to_bf16_tensor(np_bf16_normal(rng, (T, H)), dev)
        ref = ops.router_topk(x, w, K, w_next=wn, M=M, want_logits=True)
        inds = torch.empty((T, K), dtype=torch.int32, device=dev)
        scores = torch.empty((T, K), dtype=torch.bfloat16, device=dev)
        pred = torch.empty((T, M), dtype=torch.int32, device=dev)
        # first call writes the logits to a caller buffer, second keeps them in the scratch
        logits = torch.empty((T, E), dtype=torch.bfloat16, device=dev) if call == 0 else None
        rc = _noalloc_call(lib, x, w, wn, T, H, E, K, M, inds, scores, pred, logits)
        assert rc == 0, lib.moe_last_error()
        torch.cuda.synchronize()
        assert torch.equal(inds, ref["inds"]), f"call {call}: indices differ"
        assert torch.equal(scores.view(torch.int16), ref["scores"].view(torch.int16)), f"call {call}: scores differ"
        assert torch.equal(pred, ref["pred"]), f"call {call}: prediction differs"
        if logits is not None:
            assert torch.equal(logits.view(torch.int16), ref["logits"].view(torch.int16)), "logits differ"


def test_noalloc_router_rejects_sizes_beyond_its_scratch():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    from moe_offload_b200 import _lib

    lib = ctypes.CDLL(_lib.LIB_PATH)
    lib.moe_last_error.restype = ctypes.c_char_p
    dev = torch.device("cuda:0")
    T, H, E, K, M = 257, 64, 16, 4, 0          # T above the 256-token limit
    x = torch.zeros((T, H), dtype=torch.bfloat16, device=dev)
    w = torch.zeros((E, H), dtype=torch.bfloat16, device=dev)
    inds = torch.empty((T, K), dtype=torch.int32, device=dev)
    scores = torch.empty((T, K), dtype=torch.bfloat16, device=dev)
    rc = _noalloc_call(lib, x, w, w, T, H, E, K, M, inds, scores, inds, x)
    assert rc == -22
    assert b"exceeds the static scratch" in lib.moe_last_error()
