"""OffloadEngine: the reference's engine surface (mlx-qwen38/loader.py:1004-1343) over a synthetic
stack on the GPU.

The reference loads a Qwen3.8 checkpoint, its tokenizer and MLX modules; none of them exist
here, so the engine is built over a seeded synthetic stack with a BASELINE configuration's
shapes (`synthetic.StackConfig`, default c2: 28 layers x 512 experts x top-10) and keeps the
parts of the surface that belong to the MoE path: the per-layer capacities
(`compute_layer_capacities`), layer 0 pinned in HBM and layers 1.. behind LRU slot caches
filled from a pinned host pool, router-driven next-layer prefetch, `generate_greedy` with
the reference's result keys (prefill of the prompt's rows through every layer, then greedy
decode steps; windowed hit rates from the decode totals) and `collect_stats` with the
reference's layout. A prompt is `prompt_tokens` rows of seeded N(0, 1) hidden states (from
`user_content`: one row per UTF-8 byte when no count is given); a decode step feeds a fresh
N(0, 1) row, and `generated_ids` / `generated_text` stay empty. With `vocab_size` the engine
also carries the token loop (`tokens.py`): a seeded embedding table and LM head of that many
ids and a byte tokenizer, so the prompt is its UTF-8 byte ids, each decode step feeds the
previous step's argmax id, and `generate_stream` yields ids as the reference's server loop does.
"""
from __future__ import annotations

import hashlib
import time
from pathlib import Path
from typing import Any

import torch

from . import checkpoint
from .offload import HostExpertPool, OffloadStack, compute_layer_capacities
from .synthetic import C2, StackConfig, dev_bf16_normal, dev_stack
from .tokens import ByteTokenizer, TokenHead
from .tokens import generate_stream as _generate_stream


class OffloadEngine:
    """loader.py:1004-1343: OffloadEngine(model_path, budget_gb, budget_pct, alloc_mode, prefetch,
    prefetch_top_m, prefetch_cap). When model_path is a directory in the reference's layout
    (experts-XX.safetensors per layer, routers in base-*.safetensors, checkpoint.load_model_dir)
    the stack is loaded from it (top_k from its config.json or the top_k argument); otherwise
    the stack comes from `config` (synthetic weights, seed config.seed)."""

    def __init__(self, model_path=None, budget_gb: float | None = None, budget_pct: float | None = 20.0,
                 alloc_mode: str = "even", prefetch: bool = True, prefetch_top_m: int = 12, prefetch_cap: int = 3,
                 *, config: StackConfig = C2, device="cuda:0", top_k: int | None = None,
                 vocab_size: int | None = None):
        t0 = time.perf_counter()
        self.model_path = model_path
        self.device = torch.device(device)
        loaded = None
        if model_path is not None and (Path(model_path) / checkpoint.shard_name(0)).exists():
            loaded = checkpoint.load_model_dir(model_path, self.device, top_k=top_k)
            config = loaded["config"]
        self.config = config
        self.alloc_mode = alloc_mode
        self.prefetch = prefetch
        self.prefetch_top_m = prefetch_top_m
        self.prefetch_cap = prefetch_cap
        L, E = config.layers, config.experts
        self.num_layers, self.num_experts = L, E
        self.capacities = compute_layer_capacities(budget_gb=budget_gb, budget_pct=budget_pct, alloc_mode=alloc_mode,
                                                   num_layers=L, num_experts=E, expert_bytes=config.expert_bytes)
        self.total_cached_slots = sum(self.capacities.values())
        self.cache_budget_bytes = self.total_cached_slots * config.expert_bytes
        self.layer0_pinned_bytes = E * config.expert_bytes
        if loaded is not None:
            routers, layer0, pools = loaded["routers"], loaded["layer0"], loaded["pools"]
        else:
            layers = dev_stack(config, self.device)
            routers = [ly.router for ly in layers]
            pools = [HostExpertPool.from_layer(layers[l]) for l in range(1, L)]
            layer0 = layers[0]
            for l in range(1, L):
                layers[l] = None
            torch.cuda.empty_cache()
        self.stack = OffloadStack(routers, layer0, pools, self.capacities, config.top_k, self.device,
                                  prefetch=prefetch, prefetch_top_m=prefetch_top_m, prefetch_cap=prefetch_cap,
                                  expert_bytes=config.expert_bytes)
        self.cached_modules = {l: self.stack.layers[l] for l in range(1, L)}
        # token loop (server.py:113-199): a seeded embedding / LM head of vocab_size ids and the
        # byte tokenizer, when asked for; without it the loop feeds seeded hidden rows
        self.token_head = self.tokenizer = None
        if vocab_size is not None:
            self.token_head = TokenHead.synthetic(vocab_size, config.hidden, self.device, seed=config.seed + 101)
            self.tokenizer = ByteTokenizer(vocab_size)
        self._last_timings: dict[str, Any] = {}
        torch.cuda.synchronize(self.device)
        self.load_seconds = time.perf_counter() - t0

    # ------------------------------------------------------------------ settings
    def set_prefetch(self, enabled: bool, top_m: int | None = None, cap: int | None = None) -> None:
        self.prefetch = enabled
        self.stack.prefetch = enabled
        if top_m is not None:
            self.prefetch_top_m = top_m
            self.stack.M = top_m
        if cap is not None:
            self.prefetch_cap = cap
            self.stack.prefetch_cap = cap

    def reset_caches(self) -> None:
        self.stack.reset_caches()

    def reset_stats(self) -> None:
        self.stack.reset_stats()

    def _snapshot_decode_totals(self) -> tuple[int, int, int, int, int, int]:
        t = self.stack.decode_totals()
        return (t["decode_lru_hits"], t["decode_prefetch_hits"], t["decode_demand_misses"], t["decode_requests"],
                t["decode_demand_bytes"], t["decode_prefetch_bytes"])

    def _rows(self, n: int, seed: int) -> torch.Tensor:
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        return dev_bf16_normal((n, self.config.hidden), self.device, gen)

    # ------------------------------------------------------------------ generation
    def generate_stream(self, prompt_ids: list[int], max_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
                        stop_ids=None, seed: int = 0):
        """server.py:113-199 `_generate_stream_impl`: token ids of the continuation of prompt_ids,
        one per decode step (greedy when temperature <= 0, else sampled with top_p), stopping at
        the tokenizer's eos id, any of stop_ids, or max_tokens. Timings land in _last_timings."""
        if self.token_head is None:
            raise RuntimeError("this engine has no token head: construct it with vocab_size=...")
        stops = {self.tokenizer.eos_token_id} | (set(int(x) for x in stop_ids) if stop_ids is not None else set())
        self._last_timings = {}
        return _generate_stream(self.stack, self.token_head, list(prompt_ids), max_tokens, temperature, top_p,
                                stops, seed, self._last_timings)

    def generate_greedy(self, user_content: str = "", max_new_tokens: int = 128, reset_cache_before: bool = False,
                        reset_stats_before: bool = False, *, prompt_tokens: int | None = None) -> dict[str, Any]:
        """loader.py:1125-1244 with the same result keys."""
        if reset_cache_before:
            self.reset_caches()
        if reset_stats_before:
            self.reset_stats()
        seed = int.from_bytes(hashlib.sha256(user_content.encode()).digest()[:4], "little")
        dev = self.device
        head = self.token_head
        if head is not None:
            # token loop: the prompt's byte ids (or prompt_tokens seeded byte ids), each decode step
            # feeding the previous step's argmax id (loader.py:1150-1190)
            if prompt_tokens is not None:
                g = torch.Generator().manual_seed(seed)
                prompt_ids = torch.randint(0, 256, (prompt_tokens,), generator=g).tolist()
            else:
                prompt_ids = self.tokenizer.encode(user_content) or [0]
            n_prefill = len(prompt_ids)
            ids_dev = torch.tensor(prompt_ids, dtype=torch.int32).to(dev)
            prompt = head.embed(ids_dev)
        else:
            n_prefill = prompt_tokens if prompt_tokens is not None else max(1, len(user_content.encode()))
            prompt = self._rows(n_prefill, seed)
            dec_rows = self._rows(max(1, max_new_tokens), seed + 1)
        generated_ids: list[int] = []

        # 1. prefill
        torch.cuda.synchronize(dev)
        t_pre0 = time.perf_counter()
        out = self.stack.prefill(prompt)
        if head is not None:
            cur = head.argmax(out[-1:].contiguous())
        torch.cuda.synchronize(dev)
        prefill_sec = time.perf_counter() - t_pre0

        # 2. greedy decode
        s_start = self._snapshot_decode_totals()
        s_mid = s_start
        mid_tok = min(32, max_new_tokens // 2) if max_new_tokens >= 16 else max_new_tokens // 2
        step_latencies_ms: list[float] = []
        t_dec0 = time.perf_counter()
        for d_idx in range(max_new_tokens):
            if head is not None:
                generated_ids.append(int(cur.item()))
            t_step0 = time.perf_counter()
            if head is not None:
                head.argmax(self.stack.decode_token(head.embed(cur)), out=cur)
            else:
                self.stack.decode_token(dec_rows[d_idx:d_idx + 1])
            torch.cuda.synchronize(dev)
            step_latencies_ms.append(round((time.perf_counter() - t_step0) * 1000.0, 3))
            if (d_idx + 1) == mid_tok:
                s_mid = self._snapshot_decode_totals()
        decode_sec = time.perf_counter() - t_dec0
        s_end = self._snapshot_decode_totals()

        tot_req = max(1, s_end[3] - s_start[3])
        tot_lru, tot_pref = s_end[0] - s_start[0], s_end[1] - s_start[1]
        tot_dem_b, tot_pref_b = s_end[4] - s_start[4], s_end[5] - s_start[5]
        w1_req = max(1, s_mid[3] - s_start[3])
        w1_lru, w1_pref = s_mid[0] - s_start[0], s_mid[1] - s_start[1]
        w2_req = max(1, s_end[3] - s_mid[3])
        w2_lru, w2_pref = s_end[0] - s_mid[0], s_end[1] - s_mid[1]
        w1_sec = sum(step_latencies_ms[:mid_tok]) / 1000.0 if mid_tok > 0 else 0.0
        w2_sec = sum(step_latencies_ms[mid_tok:]) / 1000.0 if max_new_tokens > mid_tok else 0.0
        return {
            "prompt_tokens": n_prefill,
            "prefill_seconds": round(prefill_sec, 4),
            "prefill_tok_per_s": round(n_prefill / max(1e-9, prefill_sec), 3),
            "decode_tokens": max_new_tokens,
            "decode_seconds": round(decode_sec, 4),
            "decode_tok_per_s": round(max_new_tokens / max(1e-9, decode_sec), 3),
            "prompt_pure_lru_hit_rate": round(tot_lru / tot_req, 5),
            "prompt_effective_hit_rate": round((tot_lru + tot_pref) / tot_req, 5),
            "prompt_mb_per_token": round((tot_dem_b + tot_pref_b) / max(1, max_new_tokens) / 1e6, 3),
            "first_window_tokens": mid_tok,
            "first_window_pure_hit_rate": round(w1_lru / w1_req, 5),
            "first_window_effective_hit_rate": round((w1_lru + w1_pref) / w1_req, 5),
            "first_window_tok_per_s": round(mid_tok / max(1e-6, w1_sec), 3),
            "steady_window_tokens": max_new_tokens - mid_tok,
            "steady_window_pure_hit_rate": round(w2_lru / w2_req, 5),
            "steady_window_effective_hit_rate": round((w2_lru + w2_pref) / w2_req, 5),
            "steady_window_tok_per_s": round((max_new_tokens - mid_tok) / max(1e-6, w2_sec), 3),
            "generated_ids": generated_ids,
            "generated_text": self.tokenizer.decode(generated_ids) if head is not None else "",
            "step_latencies_ms": step_latencies_ms,
        }

    def collect_stats(self, total_decode_tokens: int, total_prefill_tokens: int) -> dict[str, Any]:
        """loader.py:1246-1338, same layout."""
        L = self.num_layers
        per_layer = [self.cached_modules[il].get_layer_stats() for il in range(1, L)]

        def tot(key):
            return sum(d[key] for d in per_layer)

        mods = list(self.cached_modules.values())

        def mtot(attr):
            return sum(getattr(c, attr) for c in mods)

        dec_req, dec_lru, dec_pref = tot("decode_requests"), tot("decode_lru_hits"), tot("decode_prefetch_hits")
        dec_dem_b, dec_pref_b = tot("decode_demand_bytes"), tot("decode_prefetch_bytes")
        dec_b = dec_dem_b + dec_pref_b
        pre_req, pre_hits, pre_miss = tot("prefill_requests"), tot("prefill_lru_hits"), tot("prefill_demand_misses")
        pre_b = tot("prefill_demand_bytes")
        uncoal, coal = tot("uncoalesced_tensor_reads"), tot("coalesced_preadv_calls")
        dec_tok, pre_tok = max(1, total_decode_tokens), max(1, total_prefill_tokens)
        return {
            "budget_summary": {
                "alloc_mode": self.alloc_mode,
                "prefetch_enabled": self.prefetch,
                "prefetch_top_m": self.prefetch_top_m if self.prefetch else 0,
                "prefetch_cap": self.prefetch_cap if self.prefetch else 0,
                "layer0_pinned_experts": self.num_experts,
                "layer0_pinned_bytes": self.layer0_pinned_bytes,
                "layer0_pinned_mib": round(self.layer0_pinned_bytes / (1024 ** 2), 2),
                "layer0_pinned_gb": round(self.layer0_pinned_bytes / 1e9, 4),
                "cached_layers_count": L - 1,
                "total_cached_slots": self.total_cached_slots,
                "mean_slots_per_cached_layer": round(self.total_cached_slots / max(1, L - 1), 2),
                "cache_budget_bytes": self.cache_budget_bytes,
                "cache_budget_gib": round(self.cache_budget_bytes / (1024 ** 3), 3),
                "cache_budget_gb": round(self.cache_budget_bytes / 1e9, 3),
                "total_routed_expert_resident_gb": round((self.cache_budget_bytes + self.layer0_pinned_bytes) / 1e9, 3),
            },
            "decode_aggregate": {
                "total_decode_tokens": total_decode_tokens,
                "total_requests_layers_1_47": dec_req,
                "lru_hits": dec_lru,
                "prefetch_hits": dec_pref,
                "demand_misses": tot("decode_demand_misses"),
                "pure_lru_hit_rate": round(dec_lru / max(1, dec_req), 5),
                "effective_hit_rate": round((dec_lru + dec_pref) / max(1, dec_req), 5),
                "top16_router_recall": round(mtot("pred_top16_hits") / max(1, mtot("pred_top16_total_actual")), 5),
                "top16_router_precision": round(mtot("pred_top16_hits") / max(1, mtot("pred_top16_total_pred")), 5),
                "miss_prefetch_recall": round(mtot("miss_pref_hits") / max(1, mtot("miss_pref_total_actual_misses")), 5),
                "miss_prefetch_precision": round(mtot("miss_pref_hits") / max(1, mtot("miss_pref_total_fetched")), 5),
                "demand_bytes_read": dec_dem_b,
                "prefetch_bytes_read": dec_pref_b,
                "total_bytes_read": dec_b,
                "demand_mb_per_token": round(dec_dem_b / dec_tok / 1e6, 3),
                "prefetch_mb_per_token": round(dec_pref_b / dec_tok / 1e6, 3),
                "total_mb_per_token": round(dec_b / dec_tok / 1e6, 3),
                "total_mib_per_token": round(dec_b / dec_tok / (1024 ** 2), 3),
                "uncoalesced_tensor_reads": uncoal,
                "coalesced_preadv_calls": coal,
                "coalesce_reduction_ratio": round(uncoal / max(1, coal), 4),
            },
            "prefill_aggregate": {
                "total_prefill_tokens": total_prefill_tokens,
                "total_requests_layers_1_47": pre_req,
                "lru_hits": pre_hits,
                "demand_misses": pre_miss,
                "hit_rate": round(pre_hits / max(1, pre_req), 5),
                "demand_bytes_read": pre_b,
                "mb_per_token": round(pre_b / pre_tok / 1e6, 3),
            },
            "per_layer": per_layer,
        }

    def close(self) -> None:
        self.stack.close()
