"""ctypes binding of libmoe_b200.so (the C ABI declared in include/moe_b200.h).

The library is the only compute path: if it is missing or cannot be loaded, every op
raises; there is no CPU fallback."""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_b200.so")

P = ctypes.c_void_p
I = ctypes.c_int
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64

_lock = threading.Lock()
_lib = None


class MoeError(RuntimeError):
    """A libmoe_b200 entry point returned a negative status."""

    def __init__(self, fn: str, rc: int, msg: str):
        super().__init__(f"{fn} failed (status {rc}): {msg}")
        self.fn, self.rc, self.msg = fn, rc, msg


# name -> (restype, argtypes); mirrors include/moe_b200.h
SIGNATURES: dict[str, tuple] = {
    "moe_version": (I, []),
    "moe_last_error": (ctypes.c_char_p, []),
    "moe_router_workspace_bytes": (SZ, [I, I, I]),
    "moe_router_topk": (I, [P, I, I, I, I, P, P, P, I, I, I, P, P, P, I, P, P, P, P, P, P, P, SZ, P]),
    "moe_router_topk_noalloc": (I, [P, I, I, I, I, P, P, P, I, I, I, P, P, P, I, P, P, P, P, P, P, P]),
    "moe_experts_gateup": (I, [P, I, I, I, I, I, P, P, P, P, P, P, P, I, I, I, P, P]),
    "moe_experts_down": (I, [P, I, I, I, I, I, P, P, P, P, P, I, I, I, P, P, P, P, P]),
    "moe_device_error": (I, [I]),
    "moe_decode_workspace_bytes": (SZ, [I, I, I, I, I, I]),
    "moe_decode_layer": (I, [P, I, I, I, I, I, P, P, I, P] + [P] * 9 + [I, I, P, P, P, P, P, P, P, SZ, P]),
    "moe_packed_expert_bytes": (SZ, [I, I]),
    "moe_pack_experts": (I, [I, I, I, P, P, P, P, P, P, P, P, P, P, P]),
    "moe_stack_workspace_bytes": (SZ, [I, I, I, I]),
    "moe_stack_decode": (I, [P, I, I, I, I, I, I, I, P, P, P, P, P, P, SZ, I, P]),
}


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                    "(nvcc, sm_100a); the MoE ops have no fallback")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args) -> int:
    lib = load()
    rc = getattr(lib, name)(*args)
    if isinstance(rc, int) and rc < 0:
        raise MoeError(name, rc, (lib.moe_last_error() or b"").decode(errors="replace"))
    return rc
