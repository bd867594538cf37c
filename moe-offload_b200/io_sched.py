"""P1 I/O scheduler: the reference's qwen38::P1IoScheduler (mlx-qwen38/cpp/src/io_sched.h:46-245)
with the same methods, backed by libmoe_b200's moe_p1_* functions (csrc/p1_device.cu).

The scheduler's state -- every layer's LRU slot cache, pin counts and in-flight reads, the
URGENT and PREFETCH read queues -- lives in device memory, and each method runs as one control
kernel on it: prefetch cancel / promote, pins held for a GPU reader (step_decode pins the k
slots it returns; unpin_layer_slots releases them once the reader is done) and the reader-wait
callback when only pinned slots could be evicted (the call stops, the callback runs on the
host, the call resumes). Rows come from a file (layer_init: the reference's form) or from a
pool of experts (layer_init_pool, pinned host or device memory) and land in host or device
slot buffers; pool rows bound for device slots are copied by a copy kernel.

The class takes any library exporting the moe_p1_* signatures under a prefix, so the parity
tests run the same calls against a build of the reference scheduler."""
from __future__ import annotations

import ctypes
from typing import Callable, Optional, Sequence

from . import _lib

READER_FN = _lib.P1_READER_FN

STAT_FIELDS = ("decode_requests", "lru_hits", "urgent_reads", "prefetch_issued", "prefetch_cancelled",
               "prefetch_promoted", "prefetch_used", "prefetch_wasted", "pin_waits", "bytes", "io_wait_ns",
               "forced_invalidations", "prefill_requests", "prefill_lru_hits", "prefill_demand_misses",
               "prefill_demand_bytes")

SIGNATURES = _lib.P1_SIGNATURES

MAX_EXPERTS = 512


def _u64s(vals: Sequence[int]):
    return (ctypes.c_uint64 * len(vals))(*[int(v) for v in vals])


def _i32s(vals: Sequence[int]):
    return (ctypes.c_int32 * max(1, len(vals)))(*[int(v) for v in vals])


def _u32s(vals: Sequence[int]):
    return (ctypes.c_uint32 * max(1, len(vals)))(*[int(v) for v in vals])


class P1IoScheduler:
    """Same methods and argument meaning as qwen38::P1IoScheduler; pointers are integers
    (host addresses, or device addresses for layer_init_pool(on_device=True))."""

    def __init__(self, lib: Optional[ctypes.CDLL] = None, prefix: str = "moe_p1_"):
        self._own = lib is None
        self._lib = lib if lib is not None else _lib.load()
        self._fn = {}
        for name, (res, args) in SIGNATURES.items():
            f = getattr(self._lib, prefix + name, None)
            if f is None:
                continue                       # optional entry points (pool source, copy errors)
            f.restype = res
            f.argtypes = args
            self._fn[name] = f
        self._h = self._fn["create"]()
        if not self._h:
            raise MemoryError("P1IoScheduler: create failed")
        self._cb = None

    # ---- plumbing
    def _call(self, name: str, *args) -> int:
        rc = self._fn[name](self._h, *args)
        if self._own and isinstance(rc, int) and rc < 0:
            lib = _lib.load()
            raise _lib.MoeError("moe_p1_" + name, rc, (lib.moe_last_error() or b"").decode(errors="replace"))
        return rc

    def close(self) -> None:
        if self._h:
            self._fn["shutdown"](self._h)
            self._fn["destroy"](self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- reference methods
    def init(self, num_threads: int = 6) -> None:
        self._call("init", num_threads)

    def shutdown(self) -> None:
        self._call("shutdown")

    def num_threads(self) -> int:
        return self._fn["num_threads"](self._h)

    def set_wait_reader_callback(self, cb: Optional[Callable[[int], None]]) -> None:
        if cb is None:
            self._cb = None
            self._call("set_wait_reader_callback", READER_FN(), None)
            return
        self._cb = READER_FN(lambda _user, layer: cb(layer))
        self._call("set_wait_reader_callback", self._cb, None)

    def layer_init(self, layer_idx: int, fd: int, capacity: int, num_tensors: int, base_offsets: Sequence[int],
                   row_bytes: Sequence[int], base_ptrs: Sequence[int], slot_inds_ptr: int = 0) -> None:
        self._call("layer_init", layer_idx, fd, capacity, num_tensors, _u64s(base_offsets), _u64s(row_bytes),
                   _u64s(base_ptrs), slot_inds_ptr)

    def layer_init_pool(self, layer_idx: int, capacity: int, src_ptrs: Sequence[int], row_bytes: Sequence[int],
                        slot_ptrs: Sequence[int], slot_inds_ptr: int = 0, on_device: bool = False,
                        device: int = 0, *, num_experts: int) -> None:
        """Rows from a pool of `num_experts` experts (src_ptrs: expert 0 of every tensor, in
        pinned host or device memory) into slot buffers (device memory with on_device)."""
        self._call("layer_init_pool", layer_idx, capacity, len(row_bytes), num_experts, _u64s(src_ptrs),
                   _u64s(row_bytes), _u64s(slot_ptrs), slot_inds_ptr, int(on_device), device)

    def resize_layer(self, layer_idx: int, new_capacity: int, new_base_ptrs: Sequence[int], slot_inds_ptr: int,
                     ordered_eids: Sequence[int], ordered_slots: Sequence[int]) -> None:
        self._call("resize_layer", layer_idx, new_capacity, _u64s(new_base_ptrs), slot_inds_ptr,
                   _i32s(ordered_eids), _i32s(ordered_slots), len(ordered_eids))

    def reset_cache(self, layer_idx: int) -> None:
        self._call("reset_cache", layer_idx)

    def reset_stats(self, layer_idx: int) -> None:
        self._call("reset_stats", layer_idx)

    def start_prefetch(self, layer_idx: int, pred_eids: Sequence[int], max_fetch: int) -> None:
        self._call("start_prefetch", layer_idx, _i32s(pred_eids), len(pred_eids), max_fetch)

    def step_decode(self, layer_idx: int, eids: Sequence[int]) -> tuple[int, list[int]]:
        """Returns (number of the k slots still loading, the k slot ids)."""
        out = (ctypes.c_uint32 * max(1, len(eids)))()
        n = self._call("step_decode", layer_idx, _u32s(eids), len(eids), out)
        return n, list(out)[:len(eids)]

    def wait_layer_urgent(self, layer_idx: int) -> None:
        self._call("wait_layer_urgent", layer_idx)

    def wait_layer_all(self, layer_idx: int) -> None:
        self._call("wait_layer_all", layer_idx)

    def wait_all(self) -> None:
        self._call("wait_all")

    def unpin_layer_slots(self, layer_idx: int) -> None:
        self._call("unpin_layer_slots", layer_idx)

    def pin_slots(self, layer_idx: int, slots: Sequence[int]) -> None:
        self._call("pin_slots", layer_idx, _u32s(slots), len(slots))

    def unpin_slots(self, layer_idx: int, slots: Sequence[int]) -> None:
        self._call("unpin_slots", layer_idx, _u32s(slots), len(slots))

    def get_slot_pin_count(self, layer_idx: int, slot: int) -> int:
        return self._fn["get_slot_pin_count"](self._h, layer_idx, slot)

    def seed(self, seed: int) -> None:
        """Seeds the std::mt19937_64 that force_invalidate draws from."""
        self._call("seed", seed)

    def force_invalidate(self, layer_idx: int, rate: float) -> int:
        return self._call("force_invalidate", layer_idx, float(rate))

    def load_sync(self, layer_idx: int, eids: Sequence[int], slots: Sequence[int], is_prefill: bool) -> None:
        self._call("load_sync", layer_idx, _i32s(eids), _i32s(slots), len(eids), int(is_prefill))

    def get_lru_state(self, layer_idx: int) -> tuple[list[int], list[int]]:
        """(eids, slots) from least to most recently used."""
        e = (ctypes.c_int32 * MAX_EXPERTS)()
        s = (ctypes.c_int32 * MAX_EXPERTS)()
        n = ctypes.c_int(0)
        self._call("get_lru_state", layer_idx, e, s, ctypes.byref(n))
        return list(e)[:n.value], list(s)[:n.value]

    def set_lru_state(self, layer_idx: int, ordered_eids: Sequence[int], ordered_slots: Sequence[int],
                      add_prefill_requests: int = 0, add_prefill_hits: int = 0, add_prefill_misses: int = 0) -> None:
        self._call("set_lru_state", layer_idx, _i32s(ordered_eids), _i32s(ordered_slots), len(ordered_eids),
                   add_prefill_requests, add_prefill_hits, add_prefill_misses)

    def get_layer_stats(self, layer_idx: int) -> dict:
        out = (ctypes.c_uint64 * len(STAT_FIELDS))()
        self._call("get_layer_stats", layer_idx, out)
        return dict(zip(STAT_FIELDS, list(out)))

    def get_total_stats(self, num_layers: int = 48) -> dict:
        """Sums layers 1..num_layers-1 (layer 0 is the pinned layer of the reference's engine)."""
        out = (ctypes.c_uint64 * len(STAT_FIELDS))()
        self._call("get_total_stats", num_layers, out)
        return dict(zip(STAT_FIELDS, list(out)))

    def copy_errors(self) -> int:
        f = self._fn.get("copy_errors")
        return int(f(self._h)) if f else 0

    def launches(self) -> int:
        """Kernels launched so far (control and row-copy kernels; 0 for the reference)."""
        f = self._fn.get("launches")
        return int(f(self._h)) if f else 0
