"""ctypes binding of libmoe_b200.so (the C ABI declared in include/moe_b200.h).

The library is the only compute path: if it is missing or cannot be loaded, every op
raises; there is no CPU fallback."""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
# MOE_B200_LIB selects another build of the same library (the profiling build of build.py --trace)
LIB_PATH = os.environ.get("MOE_B200_LIB") or os.path.join(HERE, "libmoe_b200.so")

P = ctypes.c_void_p
I = ctypes.c_int
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64
U32 = ctypes.c_uint32
I32 = ctypes.c_int32
CP = ctypes.c_char_p

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
    "moe_embed_tokens": (I, [P, I, I, P, I, P, P]),
    "moe_lm_head_logits": (I, [P, I, I, P, I, P, P]),
    "moe_lm_head_argmax_workspace_bytes": (SZ, [I]),
    "moe_lm_head_argmax": (I, [P, I, I, P, I, P, P, P, SZ, P]),
    "moe_sample_workspace_bytes": (SZ, [I, I]),
    "moe_sample_tokens": (I, [P, I, I, ctypes.c_float, ctypes.c_float, U64, U64, P, P, SZ, P]),
    "moe_experts_gateup": (I, [P, I, I, I, I, I, P, P, P, P, P, P, P, I, I, I, P, P]),
    "moe_experts_down": (I, [P, I, I, I, I, I, P, P, P, P, P, I, I, I, P, P, P, P, P]),
    "moe_device_error": (I, [I]),
    "moe_decode_workspace_bytes": (SZ, [I, I, I, I, I, I]),
    "moe_decode_layer": (I, [P, I, I, I, I, I, P, P, I, P] + [P] * 9 + [I, I, P, P, P, P, P, P, P, SZ, P]),
    "moe_packed_expert_bytes": (SZ, [I, I]),
    "moe_pack_experts": (I, [I, I, I, P, P, P, P, P, P, P, P, P, P, P]),
    "moe_prefill_workspace_bytes": (SZ, [I, I, I, I, I]),
    "moe_prefill_experts": (I, [P, I, I, I, I, I, P, P, P, P, P, P, P, P, P, P, P, I, P, P, P, P, SZ, P]),
    "moe_prefill_layer_workspace_bytes": (SZ, [I, I, I, I, I]),
    "moe_prefill_layer": (I, [P, I, I, I, I, I, P] + [P] * 9 + [I, I, P, P, P, P, P, SZ, P]),
    "moe_prefill_experts_slots": (I, [P, I, I, I, I, I, P] + [P] * 9 + [I, P, P, SZ, P]),
    "moe_combine_rows": (I, [P, I, I, I, P, P, P, P]),
    "moe_pow2_rows": (I, [P, I, I, P, P]),
    "moe_affine_linear": (I, [P, I, I, I, P, P, P, I, I, I, P, P]),
    "moe_shared_expert_workspace_bytes": (SZ, [I, I, I]),
    "moe_shared_expert": (I, [P, I, I, I] + [P] * 9 + [I, I, P, P, P, I, I, I, P, P, SZ, P]),
    "moe_hc_workspace_bytes": (SZ, [I, I, I, I]),
    "moe_hc_mix": (I, [P, I, I, I, I, P, P, P, ctypes.c_float] + [P] * 3 + [I, I] + [P] * 3 + [I, I] + [P] * 3 +
                   [I, I, I, P, P, P, P, SZ, P]),
    "moe_ep_buffer_bytes": (SZ, [I, I, I]),
    "moe_ep_buffer_alloc": (I, [SZ, P, P]),
    "moe_ep_buffer_open": (I, [P, P]),
    "moe_ep_buffer_close": (I, [P]),
    "moe_ep_buffer_free": (I, [P]),
    "moe_ep_workspace_bytes": (SZ, [I, I, I, I, I]),
    "moe_ep_decode_layer": (I, [P, I, I, I, I, I, I, I, P] + [P] * 9 + [I, I, P, P, I, I, P, P, P, P, SZ, P]),
    "moe_ep_a2a_buffer_bytes": (SZ, [I, I, I, I]),
    "moe_ep_a2a_workspace_bytes": (SZ, [I, I, I, I, I, I]),
    "moe_ep_a2a_local_tokens": (I, [I, I, I, P]),
    "moe_ep_a2a_layer": (I, [P, I, I, I, I, I, P, P] + [P] * 9 + [I, I, P, P, P, I, I, P, P, P, P, SZ, P]),
    "moe_lru_state_bytes": (SZ, [I, I]),
    "moe_lru_init": (I, [P, I, I, U64, P]),
    "moe_lru_reset": (I, [P, I, I, I, P]),
    "moe_lru_step": (I, [P, I, I, P, I, P, P, P]),
    "moe_lru_prefetch": (I, [P, I, I, P, I, I, P, P]),
    "moe_lru_acct_bytes": (SZ, []),
    "moe_f3_stack_workspace_bytes": (SZ, [I, I, I]),
    "moe_f3_stack_decode": (I, [P, I, I, I, I, I, ctypes.c_float, P, P, P, P, P, P, P, P, SZ, I, P]),
    "moe_f3moe_stack_workspace_bytes": (SZ, [I, I, I, I, I, I]),
    "moe_f3moe_stack_decode": (I, [P] + [I] * 9 + [ctypes.c_float] + [P] * 11 + [SZ, I, P]),
    "moe_k50_open": (P, [CP]),
    "moe_k50_close": (None, [P]),
    "moe_k50_count": (I, [P, CP]),
    "moe_k50_dense_name": (I, [P, I, P, SZ]),
    "moe_k50_record": (I, [P, CP, I, P]),
    "moe_k50_materialize": (I, [P, CP, I, P, P, P]),
    "moe_lru_step_ex": (I, [P, I, I, P, I, P, P, P, I, P]),
    "moe_lru_prefetch_ex": (I, [P, I, I, P, I, I, P, P, I, P]),
    "moe_lru_get_state": (I, [P, I, I, P, P]),
    "moe_lru_set_state": (I, [P, I, I, P, P, I, U64, U64, U64, P]),
    "moe_lru_get_stats": (I, [P, I, I, P, P]),
    "moe_lru_add_stat": (I, [P, I, I, I, U64, P]),
    "moe_fill_slots": (I, [P, I, I, I, I, P, P, P, I, P]),
    "moe_fill_slots_host": (I, [P, I, I, I, I, P, P, P, P]),
    # the reference's expert cache C ABI (void functions: restype None)
    "c_io_init": (None, [I]),
    "c_layer_init": (None, [I, I, I, P, P, P, U64]),
    "c_layer_init_ex": (I, [I, I, I, U64, I, P, P, P, U64]),
    "c_layer_set_host_pool": (None, [I, P]),
    "c_layer_reset_cache": (None, [I]),
    "c_layer_reset_stats": (None, [I]),
    "c_layer_wait_prefetch": (None, [I]),
    "c_layer_wait_demand": (None, [I]),
    "c_layer_start_prefetch": (None, [I, P, I, I]),
    "c_layer_start_prefetch10": (None, [I, I] + [I32] * 10),
    "c_layer_start_prefetch12": (None, [I, I] + [I32] * 12),
    "c_layer_step_decode_ex": (I, [I, P, I, I]),
    "c_layer_step_decode": (I, [I, P, I]),
    "c_layer_step_decode10": (I, [I] + [U32] * 10),
    "c_layer_step_decode10_async": (I, [I] + [U32] * 10),
    "c_layer_load_sync": (None, [I, P, P, I, I]),
    "c_layer_get_lru_state": (None, [I, P, P, P]),
    "c_layer_set_lru_state": (None, [I, P, P, I, U64, U64, U64]),
    "c_layer_get_stats": (None, [I, P]),
    "c_get_decode_totals": (None, [I, P]),
    "c_set_io_accounting": (None, [I]),
    "c_begin_decode_token": (None, [I]),
    "c_end_decode_token": (None, [P]),
    "c_get_native_buffer_bytes": (U64, []),
    "c_layer_get_split_inds": (None, [I, P, P, P]),
    "c_layer_decode_step_sched": (I, [I, P, I, P, I, I, I, I]),
    "moe_stack_workspace_bytes": (SZ, [I, I, I, I]),
    "moe_stack_decode": (I, [P, I, I, I, I, I, I, I, P, P, P, P, P, P, SZ, I, P]),
}


# the P1 I/O scheduler (moe_p1_<method>): method -> (restype, argtypes); io_sched.P1IoScheduler
# binds the same table to any library exporting these functions under a prefix
P1_READER_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int)
P1_SIGNATURES: dict[str, tuple] = {
    "create": (P, []),
    "destroy": (None, [P]),
    "init": (I, [P, I]),
    "shutdown": (I, [P]),
    "num_threads": (I, [P]),
    "set_wait_reader_callback": (I, [P, P1_READER_FN, P]),
    "layer_init": (I, [P, I, I, I, I, P, P, P, U64]),
    "layer_init_pool": (I, [P, I, I, I, I, P, P, P, U64, I, I]),
    "resize_layer": (I, [P, I, I, P, U64, P, P, I]),
    "reset_cache": (I, [P, I]),
    "reset_stats": (I, [P, I]),
    "start_prefetch": (I, [P, I, P, I, I]),
    "step_decode": (I, [P, I, P, I, P]),
    "wait_layer_urgent": (I, [P, I]),
    "wait_layer_all": (I, [P, I]),
    "wait_all": (I, [P]),
    "unpin_layer_slots": (I, [P, I]),
    "pin_slots": (I, [P, I, P, I]),
    "unpin_slots": (I, [P, I, P, I]),
    "get_slot_pin_count": (I, [P, I, I]),
    "seed": (I, [P, U64]),
    "force_invalidate": (I, [P, I, ctypes.c_double]),
    "load_sync": (I, [P, I, P, P, I, I]),
    "get_lru_state": (I, [P, I, P, P, P]),
    "set_lru_state": (I, [P, I, P, P, I, U64, U64, U64]),
    "get_layer_stats": (I, [P, I, P]),
    "get_total_stats": (I, [P, I, P]),
    "copy_errors": (U64, [P]),
    "launches": (U64, [P]),
}
SIGNATURES.update({"moe_p1_" + k: v for k, v in P1_SIGNATURES.items()})


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
