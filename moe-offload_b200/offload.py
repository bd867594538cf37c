"""Offload path: per-layer LRU expert-slot caches on the GPU filled from a pinned host pool
The reference's surface, B200-native underneath:

  compute_layer_capacities  mlx-qwen38/loader.py:245-303 (same rule, parametrised sizes)
  CachedSwitchGLU           loader.py:306-748: slot buffers in HBM, the LRU state on the GPU
                            (moe_lru_*), demand fills by a kernel reading the miss list where
                            the LRU kernel wrote it (moe_fill_slots), prefetches on a side
                            stream; __call__ returns the unweighted [B, L, K, H] expert outputs
  OffloadStack              the decode loop of OffloadEngine.generate_greedy
                            (loader.py:1125-1244) over the synthetic stack: layer 0 pinned,
                            layers 1.. cached, router-driven next-layer prefetch

No step reads anything back to the host: router -> LRU step -> fill -> experts -> prefetch
is stream-ordered on the device (the reference synchronises on the router's indices every
layer, loader.py:958).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import ops
from ._lib import call
from .ops import QMatrix
from .synthetic import ExpertLayer

# the reference's compile-time model constants (expert_io.c:18-23, loader.py:77-84)
NUM_LAYERS_REF = 48
NUM_EXPERTS_REF = 512
EXPERT_BYTES_REF = 1_536_000

STAT_NAMES = ["decode_requests", "decode_lru_hits", "decode_prefetch_hits", "decode_demand_misses",
              "decode_demand_bytes", "decode_prefetch_bytes", "prefill_requests", "prefill_lru_hits",
              "prefill_demand_misses", "prefill_demand_bytes", "pred_top16_hits", "pred_top16_total_actual",
              "pred_top16_total_pred", "miss_pref_hits", "miss_pref_total_actual_misses",
              "miss_pref_total_fetched", "uncoalesced_tensor_reads", "coalesced_preadv_calls"]


def compute_layer_capacities(budget_gb: float | None = None, budget_pct: float | None = None,
                             alloc_mode: str = "even", *, num_layers: int = NUM_LAYERS_REF,
                             num_experts: int = NUM_EXPERTS_REF, expert_bytes: int = EXPERT_BYTES_REF,
                             weights=None) -> dict[int, int]:
    """Slots per cached layer 1..num_layers-1 (layer 0 is pinned), as loader.py:245-303.

    budget_pct (a percentage, or a fraction <= 1) of num_experts per layer, else budget_gb
    (decimal GB, default 7.5) over all cached layers; 'even' splits the total equally (the
    first layers get the remainder), 'proportional' by `weights` (the reference reads the
    per-layer active-expert counts of its analysis_summary.json; without weights it falls
    back to 'even', as the reference does when that file is absent). Clamped to [16, E]."""
    n = num_layers - 1
    if budget_pct is not None:
        frac = budget_pct / 100.0 if budget_pct > 1.0 else budget_pct
        per_layer = max(16, min(num_experts, round(frac * num_experts)))
        total = n * per_layer
    else:
        if budget_gb is None:
            budget_gb = 7.5
        total = int(round((budget_gb * 1e9) / expert_bytes))
        total = max(n * 16, min(n * num_experts, total))
    if alloc_mode == "proportional" and weights is not None:
        w = np.asarray(weights, dtype=np.float64)
        if w.shape != (n,):
            raise ValueError(f"weights must have {n} entries (layers 1..{num_layers - 1})")
        raw = w / w.sum() * total
        caps = np.clip(np.floor(raw).astype(int), 16, num_experts)
        rem = total - int(caps.sum())
        fr = raw - np.floor(raw)
        if rem > 0:
            for i in np.argsort(-fr):
                if rem == 0:
                    break
                if caps[i] < num_experts:
                    caps[i] += 1
                    rem -= 1
        elif rem < 0:
            for i in np.argsort(fr):
                if rem == 0:
                    break
                if caps[i] > 16:
                    caps[i] -= 1
                    rem += 1
        return {il: int(caps[il - 1]) for il in range(1, num_layers)}
    base, rem = divmod(total, n)
    return {il: min(num_experts, max(16, base + (1 if (il - 1) < rem else 0))) for il in range(1, num_layers)}


class HostExpertPool:
    """One layer's E experts in pinned host memory, MLX layout: the nine per-expert row arrays
    (gate/up/down codes, scales, biases). Replaces the reference's experts-XX.safetensors
    shard read with pread (loader.py:318-366)."""

    NAMES = ("gate.w", "gate.s", "gate.b", "up.w", "up.s", "up.b", "down.w", "down.s", "down.b")

    def __init__(self, tensors: list[torch.Tensor], bits: int = 2, group_size: int = 64):
        if len(tensors) != 9:
            raise ValueError("nine tensors expected")
        self.t = [t if t.is_pinned() else t.pin_memory() for t in tensors]
        self.E = self.t[0].shape[0]
        self.bits, self.group_size = bits, group_size
        self.row_bytes = [t[0].numel() * t.element_size() for t in self.t]
        self.expert_bytes = sum(self.row_bytes)

    @classmethod
    def from_layer(cls, layer: ExpertLayer) -> "HostExpertPool":
        """Copies a layer's experts (device or host tensors) into freshly pinned host memory."""
        ts = []
        for q in (layer.gate, layer.up, layer.down):
            for t in (q.w, q.s, q.b):
                h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                h.copy_(t)
                ts.append(h)
        return cls(ts, layer.gate.bits, layer.gate.group_size)

    def empty_slots(self, cap: int, device) -> list[torch.Tensor]:
        return [torch.empty((cap,) + tuple(t.shape[1:]), dtype=t.dtype, device=device) for t in self.t]


class CachedSwitchGLU:
    """LRU-cached routed experts of one layer (reference CachedSwitchGLU, loader.py:306-748).

    CachedSwitchGLU(shard_path, layer_idx, capacity) as in the reference (loader.py:311): the
    layer's nine expert tensors are read from the experts-XX.safetensors shard at shard_path
    into a pinned host pool (checkpoint.load_expert_pool) and `capacity` slots are allocated
    in HBM. Keywords: pool (an already loaded HostExpertPool; shard_path may then be None),
    device (default: the current CUDA device), top_k (default 10, the reference's TOP_K),
    group_size, expert_bytes (the byte-counter unit; default the pool's expert size) and
    prefetch_stream."""

    def __init__(self, shard_path, layer_idx: int, capacity: int, *, pool: HostExpertPool | None = None,
                 device=None, top_k: int = 10, group_size: int = 64, expert_bytes: int | None = None,
                 prefetch_stream: torch.cuda.Stream | None = None):
        if pool is None:
            if shard_path is None:
                raise ValueError("CachedSwitchGLU needs a shard path or a pool")
            from . import checkpoint
            pool = checkpoint.load_expert_pool(shard_path, layer_idx, group_size)
        self.shard_path = shard_path
        self.layer_idx = layer_idx
        self.capacity = int(capacity)
        self.pool = pool
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.E = pool.E
        self.K = top_k
        if not (0 < top_k <= self.capacity <= self.E):
            raise ValueError(f"need 0 < K={top_k} <= capacity={capacity} <= E={self.E}")
        self.expert_bytes = int(expert_bytes or pool.expert_bytes)
        sl = pool.empty_slots(self.capacity, self.device)
        self.slots = sl
        self.gate = QMatrix(sl[0], sl[1], sl[2], pool.bits, pool.group_size)
        self.up = QMatrix(sl[3], sl[4], sl[5], pool.bits, pool.group_size)
        self.down = QMatrix(sl[6], sl[7], sl[8], pool.bits, pool.group_size)
        nbytes = int(call("moe_lru_state_bytes", self.E, self.capacity))
        self.state = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self._slot_inds_buf = torch.zeros((1, 1, top_k), dtype=torch.int32, device=self.device)
        self._miss = torch.zeros(1 + 2 * top_k, dtype=torch.int32, device=self.device)
        self._pref = torch.zeros(1 + 2 * 32, dtype=torch.int32, device=self.device)
        import ctypes
        self._src = (ctypes.c_void_p * 9)(*[t.data_ptr() for t in pool.t])
        self._dst = (ctypes.c_void_p * 9)(*[t.data_ptr() for t in sl])
        self._rows = (ctypes.c_uint64 * 9)(*pool.row_bytes)
        self.pstream = prefetch_stream or torch.cuda.Stream(device=self.device)
        self._pevent = torch.cuda.Event()
        self._pevent_lru = torch.cuda.Event()
        self._pending = False
        self._pending_lru = False
        # CTAs of the prefetch fill kernel (0: one per SM). A few dozen keep the host link
        # saturated and leave the SMs to the expert kernels the fill overlaps.
        self.prefetch_ctas = 0
        self._act = torch.empty((1, top_k, self.gate.w.shape[1]), dtype=torch.bfloat16, device=self.device)
        call("moe_lru_init", self.state.data_ptr(), self.E, self.capacity, self.expert_bytes, self._cs())

    def _cs(self, stream=None) -> int:
        return (stream or torch.cuda.current_stream(self.device)).cuda_stream

    # ---------------------------------------------------------------- cache management
    def reset_cache(self) -> None:
        self.wait_prefetch()
        call("moe_lru_reset", self.state.data_ptr(), self.E, self.capacity, 0, self._cs())

    def reset_stats(self) -> None:
        self.wait_prefetch()
        call("moe_lru_reset", self.state.data_ptr(), self.E, self.capacity, 1, self._cs())

    def get_lru_state(self) -> tuple[list[int], list[int]]:
        """(eids, slots) from least to most recently used (c_layer_get_lru_state)."""
        self.wait_prefetch()
        out = torch.empty(1 + 2 * self.capacity, dtype=torch.int32, device=self.device)
        call("moe_lru_get_state", self.state.data_ptr(), self.E, self.capacity, out.data_ptr(), self._cs())
        o = out.cpu().tolist()
        n = o[0]
        return o[1:1 + n], o[1 + self.capacity:1 + self.capacity + n]

    def set_lru_state(self, eids, slots, add_requests: int = 0, add_hits: int = 0, add_misses: int = 0) -> None:
        self.wait_prefetch()
        e = torch.tensor(list(eids), dtype=torch.int32).to(self.device)
        s = torch.tensor(list(slots), dtype=torch.int32).to(self.device)
        call("moe_lru_set_state", self.state.data_ptr(), self.E, self.capacity, e.data_ptr(), s.data_ptr(),
             len(e), add_requests, add_hits, add_misses, self._cs())
        torch.cuda.current_stream(self.device).synchronize()

    def raw_stats(self) -> list[int]:
        self.wait_prefetch()
        out = torch.empty(18, dtype=torch.int64, device=self.device)
        call("moe_lru_get_stats", self.state.data_ptr(), self.E, self.capacity, out.data_ptr(), self._cs())
        return [int(v) for v in out.cpu().tolist()]

    def sync_stats_from_c(self) -> None:
        for name, v in zip(STAT_NAMES, self.raw_stats()):
            setattr(self, name, v)

    def get_layer_stats(self) -> dict:
        """The reference's per-layer stats dict (loader.py:701-739)."""
        self.sync_stats_from_c()
        dr = max(1, self.decode_requests)
        pr = max(1, self.prefill_requests)
        return {
            "layer": self.layer_idx, "capacity_experts": self.capacity,
            "capacity_mb": round(self.capacity * self.expert_bytes / 1e6, 3),
            "decode_requests": self.decode_requests, "decode_lru_hits": self.decode_lru_hits,
            "decode_prefetch_hits": self.decode_prefetch_hits, "decode_demand_misses": self.decode_demand_misses,
            "decode_pure_hit_rate": round(self.decode_lru_hits / dr, 5),
            "decode_effective_hit_rate": round((self.decode_lru_hits + self.decode_prefetch_hits) / dr, 5),
            "decode_demand_bytes": self.decode_demand_bytes, "decode_prefetch_bytes": self.decode_prefetch_bytes,
            "decode_total_bytes": self.decode_demand_bytes + self.decode_prefetch_bytes,
            "prefill_requests": self.prefill_requests, "prefill_lru_hits": self.prefill_lru_hits,
            "prefill_demand_misses": self.prefill_demand_misses,
            "prefill_hit_rate": round(self.prefill_lru_hits / pr, 5),
            "prefill_demand_bytes": self.prefill_demand_bytes,
            "top16_router_recall": round(self.pred_top16_hits / max(1, self.pred_top16_total_actual), 5),
            "top16_router_precision": round(self.pred_top16_hits / max(1, self.pred_top16_total_pred), 5),
            "miss_prefetch_recall": round(self.miss_pref_hits / max(1, self.miss_pref_total_actual_misses), 5),
            "miss_prefetch_precision": round(self.miss_pref_hits / max(1, self.miss_pref_total_fetched), 5),
            "uncoalesced_tensor_reads": self.uncoalesced_tensor_reads,
            "coalesced_preadv_calls": self.coalesced_preadv_calls,
        }

    # ---------------------------------------------------------------- prefetch
    def start_prefetch(self, pred: torch.Tensor, max_fetch: int = 3) -> None:
        """Router-driven prefetch (c_layer_start_prefetch): pred = device int32 [M] ranked
        predictions. The LRU insertion and the fills run on the prefetch stream, after the
        work that produced `pred` on the current stream. Two events mark its halves: the LRU
        update (what this layer's next LRU step needs) and the fills (what its next demand
        fill, which may overwrite a slot being filled, and its expert kernels need)."""
        self.wait_prefetch()
        n = int(pred.numel())
        self.pstream.wait_stream(torch.cuda.current_stream(self.device))
        ps = self.pstream.cuda_stream
        call("moe_lru_prefetch", self.state.data_ptr(), self.E, self.capacity, pred.data_ptr(), n, max_fetch,
             self._pref.data_ptr(), ps)
        self._pevent_lru.record(self.pstream)
        call("moe_fill_slots", self._pref.data_ptr(), max_fetch, self.E, self.capacity, 9, self._src, self._dst,
             self._rows, self.prefetch_ctas, ps)
        self._pevent.record(self.pstream)
        self._pending = True
        self._pending_lru = True

    def wait_prefetch(self) -> None:
        """The current stream waits for the whole pending prefetch (LRU update and fills)."""
        if self._pending:
            torch.cuda.current_stream(self.device).wait_event(self._pevent)
            self._pending = False
            self._pending_lru = False

    # ---------------------------------------------------------------- decode
    def step(self, indices: torch.Tensor) -> torch.Tensor:
        """LRU step + demand fill for device int32 indices [.., K]: the slot ids ([1, 1, K])."""
        slots = self.step_lru(indices)
        self.fill_demand()
        return slots

    def step_lru(self, indices: torch.Tensor) -> torch.Tensor:
        """The LRU step alone (after the pending prefetch's LRU update, not its fills): slot ids
        into the slot buffer, the miss list for fill_demand."""
        if self._pending_lru:
            torch.cuda.current_stream(self.device).wait_event(self._pevent_lru)
            self._pending_lru = False
        call("moe_lru_step", self.state.data_ptr(), self.E, self.capacity, indices.data_ptr(), self.K,
             self._slot_inds_buf.data_ptr(), self._miss.data_ptr(), self._cs())
        return self._slot_inds_buf

    def fill_demand(self) -> None:
        """The fills of the last step_lru's misses, after the pending prefetch's fills (a miss
        may take a slot a prefetch is still filling; the later write must win)."""
        self.wait_prefetch()
        call("moe_fill_slots", self._miss.data_ptr(), self.K, self.E, self.capacity, 9, self._src, self._dst,
             self._rows, 0, self._cs())

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """x [1, 1, H] bf16, indices [1, 1, K] int32 (device) -> unweighted expert outputs
        [1, 1, K, H] bf16 (the reference returns them unweighted; the caller applies scores)."""
        B, L, K = indices.shape
        if B != 1 or L != 1 or K != self.K:
            raise ValueError("decode path: indices [1, 1, K]")
        slots = self.step(indices)
        act = ops.experts_gateup(x.reshape(1, -1), slots.view(1, K), self.gate, self.up, act=self._act)
        _, yk = ops.experts_down(act, slots.view(1, K), self.down, None, want_yk=True)
        return yk.view(1, 1, K, -1)

    def forward_combined(self, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor, *,
                         addend=None, resid=None, y=None) -> torch.Tensor:
        """The hook's fused form: sum_k scores_k * expert_k(x) (+ addend, e.g. the shared
        expert's output) (+ resid), x [1, H]."""
        return self.combine_slots(x, self.step(indices), scores, addend=addend, resid=resid, y=y)

    def combine_slots(self, x: torch.Tensor, slots: torch.Tensor, scores: torch.Tensor, *,
                      addend=None, resid=None, y=None) -> torch.Tensor:
        """forward_combined after its LRU step: the experts on the given slot ids."""
        K = self.K
        act = ops.experts_gateup(x, slots.view(1, K), self.gate, self.up, act=self._act)
        out, _ = ops.experts_down(act, slots.view(1, K), self.down, scores.view(1, K), addend=addend, resid=resid,
                                  y=y)
        return out

    # ---------------------------------------------------------------- prefill
    def _load_sync(self, eids: list[int], slots: list[int]) -> None:
        """Synchronous fill of (eid -> slot) with the reference's prefill accounting
        (c_layer_load_sync, expert_io.c:710-724: prefill bytes; 9 reads per expert and 9 per
        run of consecutive expert ids)."""
        import ctypes
        n = len(eids)
        lst = (ctypes.c_int32 * (1 + 2 * n))(n, *eids, *slots)
        cs = self._cs()
        call("moe_fill_slots_host", lst, n, self.E, self.capacity, 9, self._src, self._dst, self._rows, cs)
        se = sorted(eids)
        runs = 1 + sum(1 for a, b in zip(se, se[1:]) if b != a + 1)
        for idx, v in ((9, n * self.expert_bytes), (16, 9 * n), (17, 9 * runs)):
            call("moe_lru_add_stat", self.state.data_ptr(), self.E, self.capacity, idx, v, cs)

    def prefill(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """The L > 1 branch of the reference's __call__ (loader.py:566-699): x [T, H] bf16
        (the layer's normalised input), indices [T, K] int32 (device) -> unweighted expert
        outputs [T, K, H] bf16. The prompt's unique experts (ascending id) are run in chunks of
        `capacity`: the chunk's i-th expert goes to slot i (a synchronous fill unless it is
        there already), the chunk's assignments run as grouped tensor-core GEMMs on the slot
        buffers (moe_prefill_experts_slots), and afterwards the LRU is rebuilt from the final
        slot contents with the last chunk most recently used, together with the prompt's
        hit / miss counts (c_layer_set_lru_state)."""
        self.wait_prefetch()
        T, K = indices.shape
        H = x.shape[1]
        I = self.gate.w.shape[1]
        eids0, slots0 = self.get_lru_state()
        lru = dict(zip(eids0, slots0))
        slot_to_eid = {sl: e for e, sl in lru.items()}
        eid_to_slot = dict(lru)
        idx = indices.reshape(-1).cpu().numpy().astype(np.int64)
        uniq, counts = np.unique(idx, return_counts=True)
        prior = set(lru)
        add_req, add_hits, add_misses = int(idx.size), 0, 0
        for e, c in zip(uniq.tolist(), counts.tolist()):
            if e in prior:
                add_hits += c
            else:
                add_misses += 1
                add_hits += c - 1
        yk = torch.empty((T * K, H), dtype=torch.bfloat16, device=self.device)
        nb = int(call("moe_prefill_workspace_bytes", T, H, I, self.capacity, K))
        ws = torch.empty(nb, dtype=torch.uint8, device=self.device)
        g, u, d = self.gate, self.up, self.down
        last = 0
        for u0 in range(0, len(uniq), self.capacity):
            chunk = uniq[u0:u0 + self.capacity]
            last = len(chunk)
            load_e, load_s = [], []
            for s_idx, e in enumerate(chunk.tolist()):
                if slot_to_eid.get(s_idx) != e:
                    old = slot_to_eid.get(s_idx)
                    if old is not None and eid_to_slot.get(old) == s_idx:
                        del eid_to_slot[old]
                    prev = eid_to_slot.get(e)
                    if prev is not None and prev != s_idx:
                        slot_to_eid.pop(prev, None)
                    slot_to_eid[s_idx] = e
                    eid_to_slot[e] = s_idx
                    load_e.append(e)
                    load_s.append(s_idx)
            if load_e:
                self._load_sync(load_e, load_s)
            pos = np.searchsorted(chunk, idx)
            inside = (pos < len(chunk)) & (chunk[np.minimum(pos, len(chunk) - 1)] == idx)
            sl = np.where(inside, pos, self.capacity).astype(np.int32)
            sl_dev = torch.from_numpy(sl).to(self.device)
            call("moe_prefill_experts_slots", x.data_ptr(), T, H, I, self.capacity, K, sl_dev.data_ptr(),
                 g.w.data_ptr(), g.s.data_ptr(), g.b.data_ptr(), u.w.data_ptr(), u.s.data_ptr(), u.b.data_ptr(),
                 d.w.data_ptr(), d.s.data_ptr(), d.b.data_ptr(), g.sb_fp16, yk.data_ptr(), ws.data_ptr(), ws.numel(),
                 self._cs())
        # rebuild the LRU: slots last.. in slot order, then the last chunk's slots (MRU end)
        order = [s_ for s_ in range(last, self.capacity) if s_ in slot_to_eid] + \
                [s_ for s_ in range(last) if s_ in slot_to_eid]
        self.set_lru_state([slot_to_eid[s_] for s_ in order], order, add_req, add_hits, add_misses)
        return yk.view(T, K, H)

    def close(self) -> None:
        self.wait_prefetch()


class OffloadStack:
    """Decode over a stack with layer 0 pinned in HBM and layers 1.. behind CachedSwitchGLU
    caches (the OffloadEngine decode loop, loader.py:1125-1244 with hooked_layer_call
    855-992): per layer the router (with the next layer's top-M prediction), the LRU step and
    fills, the experts and combine, then the prefetch of the next layer's predicted experts.

    routers: bf16 [E, H] per layer (device); layer0: the pinned layer's experts (device);
    pools: HostExpertPool per layer 1..L-1. `inject` (optional) replaces the routed experts by
    given eids (BASELINE c2 drives the cache with a synthetic Zipf routing; the router still
    runs). pred_bias: optional float32 [L, E] added to the next layer's logits before top-M."""

    def __init__(self, routers: list[torch.Tensor], layer0: ExpertLayer, pools: list[HostExpertPool],
                 capacities: dict[int, int], top_k: int, device, prefetch: bool = True, prefetch_top_m: int = 12,
                 prefetch_cap: int = 3, norm: bool = True, expert_bytes: int | None = None):
        self.device = torch.device(device)
        self.routers = routers
        self.layer0 = layer0
        self.L = len(routers)
        self.K = top_k
        self.M = prefetch_top_m
        self.prefetch = prefetch
        self.prefetch_cap = prefetch_cap
        self.norm = norm
        self.H = routers[0].shape[1]
        self.E = routers[0].shape[0]
        ps = torch.cuda.Stream(device=self.device)
        self.layers = [None] + [CachedSwitchGLU(None, l, capacities[l], pool=pools[l - 1], device=self.device,
                                                top_k=top_k, expert_bytes=expert_bytes, prefetch_stream=ps)
                                for l in range(1, self.L)]
        self.capacities = capacities
        self.hs = [torch.empty((1, self.H), dtype=torch.bfloat16, device=self.device) for _ in range(self.L + 1)]
        self.xn = [torch.empty((1, self.H), dtype=torch.bfloat16, device=self.device) for _ in range(self.L)]
        self.r_out = [{} for _ in range(self.L)]
        self.pred_bias = None

    def reset_caches(self) -> None:
        for c in self.layers[1:]:
            c.reset_cache()

    def reset_stats(self) -> None:
        for c in self.layers[1:]:
            c.reset_stats()

    def decode_token(self, h: torch.Tensor, inject: torch.Tensor | None = None,
                     pred_inject: torch.Tensor | None = None) -> torch.Tensor:
        """h [1, H] bf16 (device) -> output of the last layer; inject: device int32 [L, K]
        routed experts; pred_inject: device int32 [L, M], row l the ranked prediction of layer
        l+1's experts that drives its prefetch (the router's own prediction is still computed,
        as in the reference, but not used)."""
        self.hs[0].copy_(h)
        for l in range(self.L):
            x = self.hs[l]
            xin = x
            if self.norm:                              # one kernel (moe_pow2_rows), graph-safe buffer
                xin = self.xn[l]
                call("moe_pow2_rows", x.data_ptr(), 1, self.H, xin.data_ptr(),
                     torch.cuda.current_stream(self.device).cuda_stream)
            nxt = self.routers[l + 1] if (self.prefetch and l + 1 < self.L) else None
            pb = self.pred_bias[l + 1] if (nxt is not None and self.pred_bias is not None) else None
            r = ops.router_topk(xin, self.routers[l], self.K, w_next=nxt, M=self.M if nxt is not None else 0,
                                pred_bias=pb, out=self.r_out[l])
            eids = inject[l].view(1, self.K) if inject is not None else r["inds"]
            # The cache calls keep the reference's order (layer l's step, then layer l+1's
            # prefetch). Layer l+1's prefetch is issued between layer l's LRU step and its
            # demand fill, so the prefetch's LRU update runs beside the demand fill and its fill
            # crosses the host link while layer l's expert kernels run; the LRU step itself
            # waits only for the prefetch's LRU update, the demand fill for its fills. The two
            # calls touch different layers' caches, so every LRU state sequence is the
            # reference's.
            slots = eids if l == 0 else self.layers[l].step_lru(eids)
            if nxt is not None:
                pred = pred_inject[l] if pred_inject is not None else r["pred"].view(-1)
                self.layers[l + 1].start_prefetch(pred, self.prefetch_cap)
            if l > 0:
                self.layers[l].fill_demand()
            if l == 0:
                act = ops.experts_gateup(xin, eids, self.layer0.gate, self.layer0.up)
                ops.experts_down(act, eids, self.layer0.down, r["scores"], resid=x, y=self.hs[l + 1])
            else:
                self.layers[l].combine_slots(xin, slots, r["scores"], resid=x, y=self.hs[l + 1])
        return self.hs[self.L]

    def prefill(self, h: torch.Tensor) -> torch.Tensor:
        """The prompt's rows h [T, H] bf16 through every layer (the prefill of
        OffloadEngine.generate_greedy, loader.py:1150-1156): layer 0 (pinned) with the resident
        grouped GEMMs, layers 1.. through their caches' prefill (CachedSwitchGLU.prefill) and
        the MLX-order combine with the residual. Returns the last layer's output [T, H]."""
        x = h.contiguous()
        T = x.shape[0]
        for l in range(self.L):
            xin = x
            if self.norm:
                xin = torch.empty_like(x)
                call("moe_pow2_rows", x.data_ptr(), T, self.H, xin.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
            r = ops.router_topk(xin, self.routers[l], self.K)
            if l == 0:
                x = ops.prefill_experts(xin, r["inds"], r["scores"], self.layer0.gate, self.layer0.up,
                                        self.layer0.down, resid=x)
                continue
            yk = self.layers[l].prefill(xin, r["inds"])
            y = torch.empty_like(x)
            call("moe_combine_rows", yk.data_ptr(), T, self.K, self.H, r["scores"].data_ptr(), x.data_ptr(),
                 y.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
            x = y
        return x

    def capture(self, pred_injected: bool = False) -> None:
        """Records one decode_token as a CUDA graph over static input buffers (the token's
        hidden state, injected experts and, with pred_injected, injected predictions);
        decode_graph() then replays it. Every step of the token is device-side, so the graph
        needs no host decisions."""
        self.h_static = torch.zeros((1, self.H), dtype=torch.bfloat16, device=self.device)
        self.inj_static = torch.zeros((self.L, self.K), dtype=torch.int32, device=self.device)
        self.pred_static = torch.full((self.L, self.M), -1, dtype=torch.int32, device=self.device) \
            if pred_injected else None
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.decode_token(self.h_static, self.inj_static, self.pred_static)   # warm: workspaces, attributes
        s.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self.decode_token(self.h_static, self.inj_static, self.pred_static)
        torch.cuda.current_stream(self.device).wait_stream(s)

    def decode_graph(self, h: torch.Tensor, inject: torch.Tensor | None,
                     pred: torch.Tensor | None = None) -> torch.Tensor:
        """Replays the captured token: h [1, H], inject [L, K] routed experts and (when the
        graph was captured with pred_injected) pred [L, M] predictions, all device tensors."""
        self.h_static.copy_(h)
        if inject is not None:
            self.inj_static.copy_(inject)
        if pred is not None:
            if self.pred_static is None:
                raise ValueError("capture(pred_injected=True) first")
            self.pred_static.copy_(pred)
        self.graph.replay()
        return self.hs[self.L]

    def layer_stats(self) -> list[dict]:
        return [c.get_layer_stats() for c in self.layers[1:]]

    def decode_totals(self) -> dict:
        """c_get_decode_totals over the cached layers."""
        keys = ("decode_lru_hits", "decode_prefetch_hits", "decode_demand_misses", "decode_requests",
                "decode_demand_bytes", "decode_prefetch_bytes")
        tot = dict.fromkeys(keys, 0)
        for c in self.layers[1:]:
            s = dict(zip(STAT_NAMES, c.raw_stats()))
            for k in keys:
                tot[k] += s[k]
        return tot

    def close(self) -> None:
        for c in self.layers[1:]:
            c.close()


def _pow2_normalize_dev(h: torch.Tensor) -> torch.Tensor:
    """Power-of-two RMS normalisation on the device (same rule as ops.pow2_normalize): the
    exponent comes from the float64 sum of squares; the product is exact in bf16."""
    ss = h.double().pow(2).sum()
    n = h.numel()
    m, e = torch.frexp(ss / n)
    k = torch.where(e >= 0, torch.div(e, 2, rounding_mode="floor"), -torch.div(1 - e, 2, rounding_mode="floor"))
    k = torch.where(ss > 0, k, torch.zeros_like(k))
    return (h.double() * torch.pow(2.0, -k.double())).to(torch.bfloat16)


def zipf_routing(seed: int, layers: int, tokens: int, E: int, K: int, s: float = 1.1, reuse: float = 0.3):
    """BASELINE c2 synthetic routing: per layer a fixed random permutation of the experts with
    Zipf(s) popularity; per token K distinct draws, each reusing one of the previous token's
    experts with probability `reuse`. Returns int32 [tokens, layers, K] and the per-layer
    popularity (log) used as the prediction bias, float32 [layers, E]."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, E + 1, dtype=np.float64)
    pop = ranks ** -s
    pop /= pop.sum()
    perms = [rng.permutation(E) for _ in range(layers)]
    out = np.zeros((tokens, layers, K), dtype=np.int32)
    prev = [None] * layers
    for t in range(tokens):
        for l in range(layers):
            chosen: list[int] = []
            while len(chosen) < K:
                if prev[l] is not None and rng.random() < reuse:
                    e = int(prev[l][rng.integers(0, K)])
                else:
                    e = int(perms[l][rng.choice(E, p=pop)])
                if e not in chosen:
                    chosen.append(e)
            prev[l] = chosen
            out[t, l] = chosen
    bias = np.zeros((layers, E), dtype=np.float32)
    for l in range(layers):
        bias[l, perms[l]] = np.log(pop).astype(np.float32) - math.log(pop[-1])
    return out, bias


def synthetic_predictions(routing: np.ndarray, bias: np.ndarray, recall: float = 0.836, M: int = 12,
                          seed: int = 0) -> np.ndarray:
    """A next-layer predictor of stated recall for the synthetic c2 routing (the reference
    measured recall@10 = 83.6 % for its router-based predictor, README.md:35). For token t and
    layer l < L-1, row [t, l] ranks M candidates for layer l+1's experts routing[t, l+1]: each
    of the K routed experts is kept with probability `recall`, each dropped one is replaced by
    a distinct non-routed expert drawn from the layer's Zipf popularity (exp(bias)); the K
    kept-or-replacement entries come first in random order, then M-K more distinct popular
    non-routed experts. Row [t, L-1] is -1 (nothing to predict). int32 [tokens, layers, M]."""
    rng = np.random.default_rng(seed)
    T, L, K = routing.shape
    E = bias.shape[1]
    pop = np.exp(bias.astype(np.float64))
    pop /= pop.sum(axis=1, keepdims=True)
    out = np.full((T, L, M), -1, dtype=np.int32)
    for t in range(T):
        for l in range(L - 1):
            true = [int(e) for e in routing[t, l + 1]]
            taken = set(true)
            head = []
            for e in true:
                if rng.random() < recall:
                    head.append(e)
                else:
                    head.append(-1)

            def draw() -> int:
                while True:
                    c = int(rng.choice(E, p=pop[l + 1]))
                    if c not in taken:
                        taken.add(c)
                        return c
            head = [e if e >= 0 else draw() for e in head]
            rng.shuffle(head)
            tail = [draw() for _ in range(M - K)]
            out[t, l] = head + tail
    return out
