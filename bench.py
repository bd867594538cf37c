#!/usr/bin/env python3
"""MoE decode throughput on the 28-layer, 512-expert, top-10 resident stack.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token through all 28 layers (router -> 2-bit gate/up + SwiGLU -> 2-bit
down + combine, h_{l+1} = h_l + MoE_l(h_l)) with a fresh N(0,1) hidden state per step
(seed 1), expert weights random-init with the BASELINE distributions (synthetic: the
reference's checkpoints are not available). For N > 1 (torchrun) the run is BASELINE config 4,
expert parallelism: the experts of every layer split across the N GPUs (512/N each), a batch
of 8 tokens per GPU (B = 8N) owned in blocks by the ranks, every layer a routed all-to-all over
NVLink (each token's row to the ranks holding its experts, each output row back to its owner,
MLX-order combine) -- per-GPU work fixed: weak scaling. `--replicas` runs N independent copies
of the c1 stack instead (one token stream per GPU, no exchange).

The step is ONE launch of the persistent kernel (moe_stack_decode: all 28 layers inside,
experts in the packed layout). Prints one JSON line (rank 0). `value` is whole-job tokens/s
from CUDA events around the timed steps (max over ranks); `e2e` is the same metric through
PersistentStack.decode() with the hidden state copied from pinned host memory and the
result copied back every step; `roofline` is that kernel's algorithmic bytes per launch over
its live launch time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE decode tok/s (28-layer expert stack); expert GEMV HBM GB/s vs B200 peak"
UNIT = "tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c3n", "c4", "p1", "f3", "f3moe", "f4"], default="c1",
                    help="c1: resident stack (the headline); c2: offload stack with the LRU slot caches; "
                         "c3: 2048-token prefill through the resident 28-layer stack; c3n: the Nemotron-shaped "
                         "prefill layer (240 experts, top-9, 1024 tokens); c4: expert-parallel decode (experts "
                         "split across the ranks); p1: the P1 I/O scheduler filling c2-shaped expert slots; f3: the "
                         "hyper-connection mixer + shared expert in front of each of the 28 MoE blocks, decode; "
                         "f3moe: the mixer, the routed block and the shared expert of all 28 layers in one launch; "
                         "f4: the greedy token loop (embedding, the c1 stack, a 248,320-id LM head, argmax)")
    ap.add_argument("--batch", type=int, default=0, help="c4: tokens per step (default: 8 per GPU; 4096 = c4's prefill)")
    ap.add_argument("--replicas", action="store_true",
                    help="--gpus N > 1: N independent replicas of the c1 stack instead of expert parallelism")
    ap.add_argument("--no-check", action="store_true", help="c4: skip the bit-exact check of layer 0")
    ap.add_argument("--ep-mode", choices=["auto", "sharded", "replicated"], default="auto",
                    help="c4: tokens sharded (routed all-to-all) or replicated on every rank; auto: sharded "
                         "from 4 tokens per GPU")
    ap.add_argument("--prefetch-ctas", type=int, default=32,
                    help="c2: CTAs of each prefetch fill kernel (0 = one per SM)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling aid: run only the first N layers of the stack (0 = all 28)")
    return ap.parse_args()


def peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------- CPU legs

class CpuLayer:
    """The oracle port (C restatement, OpenMP on all host cores) of one layer of the c1 shape:
    512-expert bf16 router + softmax/top-10, then 10 routed 2-bit experts and the combine.
    64 experts are materialised on the host and the routing is taken modulo 64 (the
    per-token work is identical: 10 experts' weights are read either way)."""

    def __init__(self):
        import numpy as np

        from moe_offload_b200.synthetic import C1, np_bf16_normal, np_qmatrix
        from oracle import oracle as orc

        self.np, self.orc, self.cfg = np, orc, C1
        self.rng = np.random.default_rng(C1.seed)
        E, H, I = C1.experts, C1.hidden, C1.inter
        self.nres = 64
        self.g = np_qmatrix(self.rng, self.nres, I, H)
        self.u = np_qmatrix(self.rng, self.nres, I, H)
        self.d = np_qmatrix(self.rng, self.nres, H, I)
        self.wr = np_bf16_normal(self.rng, (E, H), 0.02)
        self.rand = lambda: np_bf16_normal(self.rng, (1, H))
        orc.set_threads(os.cpu_count() or 1)
        self.cores = orc.num_threads()
        # algorithmic bytes of one token-layer (10 experts + the router), for the effective GB/s
        self.layer_bytes = C1.top_k * C1.expert_bytes + C1.router_bytes

    def token_layer(self) -> float:
        x = self.rand()
        t0 = time.perf_counter()
        lg = self.orc.router_logits(x, self.wr, self.cfg.experts)
        _, inds, sc = self.orc.softmax_topk(lg, self.cfg.top_k)
        self.orc.experts(x, inds % self.nres, sc, self.g, self.u, self.d, sb_fp16=True, resid=x)
        return time.perf_counter() - t0


def cpu_layer_sample(seconds: float = 12.0) -> dict:
    """Bounded CPU baseline: as many token-layers as fit in `seconds`, extrapolated to the
    28-layer stack."""
    cl = CpuLayer()
    cl.token_layer()
    ts = []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        ts.append(cl.token_layer())
    per_layer = statistics.mean(ts)
    return {"value": round(1.0 / (cl.cfg.layers * per_layer), 4), "unit": UNIT, "cores": cl.cores,
            "kind": "port", "effective_gbs": round(cl.layer_bytes / per_layer / 1e9, 2),
            "sample": f"{len(ts)} token-layers of the c1 shape (1 of 28 layers: 512-expert router, top-10 "
                      f"2-bit experts, combine) in {seconds:.0f}s, extrapolated x28 layers; C restatement "
                      f"(MLX is not installable here)"}


def cpu_token_sample(vocab: int, hidden: int, seconds: float = 12.0, head_rows: int = 32768) -> dict:
    """Bounded CPU baseline of the f4 token step: the c1 stack's token-layers (as
    cpu_layer_sample) plus the LM head as the reference's CPU path would run it, one fp32 BLAS
    matrix-vector product (numpy, all BLAS threads) over `head_rows` rows of the head, scaled to
    the vocabulary, and its argmax; the embedding lookup is negligible."""
    import numpy as np

    stack = cpu_layer_sample(seconds)
    rng = np.random.default_rng(5)
    w = rng.normal(0.0, 0.02, (head_rows, hidden)).astype(np.float32)
    x = rng.normal(0.0, 1.0, (hidden,)).astype(np.float32)
    int(np.argmax(w @ x))                                   # warm-up
    reps = 5
    t0 = time.perf_counter()
    for _ in range(reps):
        int(np.argmax(w @ x))
    head_s = (time.perf_counter() - t0) / reps * vocab / head_rows
    token_s = 1.0 / stack["value"] + head_s
    return {"value": round(1.0 / token_s, 4), "unit": "tok/s", "cores": stack["cores"], "kind": "port",
            "head_s_per_token": round(head_s, 5), "stack_tok_s": stack["value"],
            "sample": stack["sample"] + f"; the LM head as an fp32 BLAS matvec over {head_rows} of {vocab} "
                      f"rows (numpy), scaled to the vocabulary"}


def c1_config(cfg, world: int) -> dict:
    """The workload description both arms print for the c1 stack (same dict, same keys)."""
    return {"workload": cfg.name, "layers": cfg.layers, "hidden": cfg.hidden, "experts": cfg.experts,
            "top_k": cfg.top_k, "inter": cfg.inter, "batch": 1, "group_size": cfg.group_size,
            "scales": "fp16", "router": "bf16", "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2: 707 MB of weights per step, 31.7 GB resident"}


def c4_config(cfg, world: int, B: int, sharded: bool, L: int | None = None) -> dict:
    """The workload description both arms print for the expert-parallel run (--gpus N > 1)."""
    return {"workload": f"{cfg.name}_batch{B}", "layers": L or cfg.layers, "hidden": cfg.hidden,
            "experts": cfg.experts, "top_k": cfg.top_k, "inter": cfg.inter, "batch": B,
            "group_size": cfg.group_size, "scales": "fp16", "router": "bf16 (replicated)",
            "parallelism": f"ep{world} (experts {cfg.experts}/{world} per GPU" +
                           (f", tokens {B}/{world} per GPU)" if sharded else ", tokens replicated)"),
            "exchange": ("routed all-to-all: peer stores over NVLink (dispatch once per token and rank, each "
                         "output row returned once) + epoch flags, no library collective") if sharded else
                        "every output row stored in every rank over NVLink + epoch flags",
            "l2": "inputs larger than L2"}


def run_reference(args, rank: int, world: int) -> None:
    """--impl reference: the reference computes this path with MLX, which is not installable
    here; its CPU restatement (oracle port) runs on all host cores on rank 0 only. One step
    = one token through one layer of the c1 shape, reported as 28-layer tok/s."""
    if rank != 0:
        return
    cl = CpuLayer()
    for _ in range(args.warmup):
        cl.token_layer()
    ts = [cl.token_layer() for _ in range(args.steps)]
    per_layer = statistics.mean(ts)
    v = 1.0 / (cl.cfg.layers * per_layer)
    cfg = cl.cfg
    cpu = {"value": round(v, 4), "unit": UNIT, "cores": cl.cores, "kind": "port",
           "effective_gbs": round(cl.layer_bytes / per_layer / 1e9, 2),
           "sample": f"{args.steps} token-layers (1 of 28 layers each), extrapolated x28; C restatement"}
    line = {"metric": METRIC, "value": round(v, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000.0 * per_layer * cfg.layers, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u2 codes x bf16 -> f32",
            "data": "synthetic", "impl": "reference",
            "config": c1_config(cfg, args.gpus) if (world == 1 or args.replicas) else
                      c4_config(cfg, world, args.batch or 8 * world, (args.batch or 8 * world) >= 4 * world),
            "cpu_baseline": cpu,
            "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------- GPU leg

STACK_KERNEL = "stack_kernel (persistent: router + top-10 + 2-bit gate/up/down + combine, 28 layers)"


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from moe_offload_b200.stack import PersistentStack
    from moe_offload_b200.synthetic import C1, dev_bf16_normal, dev_stack

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = C1
    if args.layers:
        import dataclasses
        cfg = dataclasses.replace(cfg, name=f"{cfg.name}_first{args.layers}", layers=args.layers)
    layers = dev_stack(cfg, dev)
    stack = PersistentStack(layers, cfg.top_k, dev, release_unpacked=True)
    del layers
    torch.cuda.empty_cache()
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed + 1000 * rank)
    n_in = args.warmup + args.steps
    h0 = dev_bf16_normal((n_in, 1, cfg.hidden), dev, gen)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        stack.step_device(h0[i])
    torch.cuda.synchronize()
    barrier()
    clk = ClockSampler(local_rank)
    clk.start()
    torch.cuda.synchronize()
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        stack.step_device(h0[args.warmup + i])
    e.record()
    torch.cuda.synchronize()
    barrier()
    clocks = clk.stop()
    t_ms = s.elapsed_time(e)
    if world > 1:
        tt = torch.tensor([t_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms = float(tt.item())
    value = world * args.steps / (t_ms / 1000.0)
    from moe_offload_b200 import _lib
    dev_err = int(_lib.call("moe_device_error", 1))

    e2e = None
    if not args.no_e2e:
        hh = h0.cpu().pin_memory()
        out_host = torch.empty((1, cfg.hidden), dtype=torch.bfloat16, pin_memory=True)
        for i in range(min(args.warmup, 4)):
            stack.decode(hh[i], out_host)
        barrier()
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(args.steps):
            stack.decode(hh[args.warmup + i], out_host)
        e2.record()
        torch.cuda.synchronize()
        barrier()
        t2 = s2.elapsed_time(e2)
        if world > 1:
            tt = torch.tensor([t2], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t2 = float(tt.item())
        e2e = {"value": round(world * args.steps / (t2 / 1000.0), 2), "unit": UNIT,
               "h2d_bytes_per_step": cfg.hidden * 2, "d2h_bytes_per_step": cfg.hidden * 2,
               "api": "moe_offload_b200.stack.PersistentStack.decode (pinned host in/out, sync per step)"}

    # roofline of the one kernel of the step: algorithmic bytes of a token (every routed
    # expert's packed bytes + every router, 28 layers) over the step's device time (the
    # kernel plus the 24 KB workspace clear before it)
    peak, peak_kind = peaks()
    step_bytes = cfg.layers * (cfg.top_k * cfg.expert_bytes + cfg.router_bytes)
    launch_s = t_ms / 1000.0 / args.steps
    achieved = step_bytes / launch_s / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get("stack_kernel_bytes_per_launch")
        except Exception:
            traffic = None
    roof = {"kernel": STACK_KERNEL, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic, "algorithmic_bytes_per_launch": step_bytes,
            "launch_us": round(launch_s * 1e6, 2), "peak_source": peak_kind}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_layer_sample()

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u2 codes x bf16 -> f32", "data": "synthetic",
                "config": c1_config(cfg, world),
                "roofline": roof, "clocks": clocks, "gpu_launches": stack.launches_per_step * args.steps,
                "device_error": dev_err, "e2e": e2e, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)


def h2d_peak_gbs(dev, nbytes: int = 1 << 28) -> float:
    """Pinned host -> device copy-engine bandwidth (cudaMemcpyAsync), measured here."""
    import torch

    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(4):
        dst.copy_(src, non_blocking=True)
    e.record()
    torch.cuda.synchronize()
    return 4 * nbytes / (s.elapsed_time(e) / 1000.0) / 1e9


def run_p1(args, rank: int, world: int, local_rank: int) -> None:
    """The P1 I/O scheduler (moe_offload_b200.io_sched) filling c2-shaped expert slots: one
    layer, 512 experts of 2,211,840 bytes (the nine MLX tensors of a c1 expert) in a pinned
    host pool, 102 slots in HBM, the scheduler's state on the GPU. A step is one decode step of
    10 random experts (step_decode -> coalesced URGENT rows -> wait_layer_urgent) followed by a
    3-expert prefetch that the next step uses or wastes. `value` = rows moved per second (the
    scheduler's byte counter: demand and prefetch) over the timed steps; the pinned
    cudaMemcpyAsync peak of this GPU is reported beside it."""
    import random

    import torch

    from moe_offload_b200.io_sched import P1IoScheduler

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    E, cap, K = 512, 102, 10
    rows = [589824, 73728, 73728] * 3
    ebytes = sum(rows)
    gen = torch.Generator().manual_seed(2)
    pool = [torch.randint(0, 256, (E, rb), dtype=torch.uint8, generator=gen).pin_memory() for rb in rows]
    slots = [torch.empty(cap * rb, dtype=torch.uint8, device=dev) for rb in rows]
    s = P1IoScheduler()
    s.init(8)
    s.layer_init_pool(1, cap, [p.data_ptr() for p in pool], rows, [b.data_ptr() for b in slots], 0, True,
                      local_rank, num_experts=E)
    s.set_wait_reader_callback(lambda layer: s.unpin_layer_slots(layer))
    rng = random.Random(2)

    def step():
        s.unpin_layer_slots(1)
        eids = rng.sample(range(E), K)
        n, _ = s.step_decode(1, eids)
        if n:
            s.wait_layer_urgent(1)
        s.start_prefetch(1, rng.sample(range(E), 12), 3)

    for _ in range(args.warmup):
        step()
    s.wait_all()
    s.reset_stats(1)
    l0 = s.launches()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    s.wait_all()
    dt = time.perf_counter() - t0
    launches = s.launches() - l0
    st = s.get_layer_stats(1)
    urgent_bytes = st["urgent_reads"] * ebytes
    value = st["bytes"] / dt / 1e9
    peak = h2d_peak_gbs(dev)
    line = {"metric": "P1 scheduler fill GB/s (c2 expert rows, demand + prefetch, pinned host pool -> HBM slots)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1000 / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8 rows", "data": "synthetic",
            "config": {"workload": "p1_c2_rows_cap102_k10", "experts": E, "slots": cap, "top_k": K,
                       "expert_bytes": ebytes, "tensors": 9,
                       "workers": "init(8): the copy kernel takes every queued row at the end of each call",
                       "prefetch": "top-12 random predictions, cap 3"},
            "demand_gbs": round(urgent_bytes / dt / 1e9, 2),
            "roofline": {"bound": "h2d link", "achieved": round(value, 2), "peak": round(peak, 2), "unit": "GB/s",
                         "frac": round(value / peak, 4), "traffic": None,
                         "peak_source": "pinned cudaMemcpyAsync measured in this run"},
            "stats": {k: v for k, v in st.items() if k != "io_wait_ns"}, "io_wait_ms": round(st["io_wait_ns"] / 1e6, 2),
            "copy_errors": s.copy_errors(), "gpu_launches": launches, "e2e": None, "cpu_baseline": None}
    s.close()
    print(json.dumps(line), flush=True)


def f3_mix_layers(dev, g, L, HC, H, R, I):
    """Synthetic mixer + shared-expert weights of L layers (8-bit g64 mixer down / up / inject,
    4-bit g64 shared gate / up / down, an 8-bit scalar gate; bf16 scales and biases)."""
    import torch

    from moe_offload_b200.ops import QMatrix

    def qm(N, K, bits, scale):
        w = torch.randint(-(2 ** 31), 2 ** 31 - 1, (N, K * bits // 32), dtype=torch.int32, device=dev, generator=g)
        sc = (torch.rand((N, K // 64), device=dev, generator=g) * scale + scale / 10).to(torch.bfloat16)
        b = (torch.randn((N, K // 64), device=dev, generator=g) * scale * 4).to(torch.bfloat16)
        return QMatrix(w, sc, b, bits, 64)

    return [{"nw": (torch.randn(HC * H, device=dev, generator=g) * 0.05).to(torch.bfloat16),
             "down": qm(R, HC * H, 8, 2e-4), "up": qm(HC * H, R, 8, 2e-3), "inj": qm(HC, HC * H, 8, 2e-4),
             "sg": qm(I, H, 4, 2e-3), "su": qm(I, H, 4, 2e-3), "sd": qm(H, I, 4, 2e-3), "se": qm(1, H, 8, 2e-4)}
            for _ in range(L)]


def run_f3(args, rank: int, world: int, local_rank: int) -> None:
    """The step in front of every MoE block, decode (one token): the hyper-connection mixer
    (run_hc with a write: 4 streams of H = 3072, rank 320, 8-bit g64 down / up / inject) and the
    shared expert on its output (gate / up / down 4-bit g64 with I = 768, an 8-bit scalar gate),
    for 28 chained layers with their own weights (347 MB, beyond L2): each layer's mixer writes
    the previous layer's block output (here the shared expert's) into the streams. The step is
    ONE launch of moe_f3_stack_decode (all layers, four grid barriers per layer); the same chain
    as five launches per layer (moe_hc_mix + moe_shared_expert, one CUDA graph) is timed beside
    it and must give the same bits. `value` = tokens/s through the 28 layers; roofline =
    algorithmic weight bytes per token / step time against the HBM peak; e2e adds the pinned
    host -> device copy of the token's streams and the read-back of the last block output."""
    import numpy as np
    import torch

    from moe_offload_b200 import ops
    from moe_offload_b200.hooks import hc_write
    from moe_offload_b200.ops import QMatrix

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L, HC, H, R, I = 28, 4, 3072, 320, 768
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    layers = f3_mix_layers(dev, g, L, HC, H, R, I)
    wbytes = sum(m.w.numel() * 4 + m.s.numel() * 4 for lay in layers for m in lay.values() if isinstance(m, QMatrix))
    h = (torch.randn(HC * H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    br = (torch.randn(H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    gt = (torch.randn(HC, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    st = torch.cuda.Stream(dev)
    stack = ops.F3Stack(layers, dev)
    out = {}
    chain_out = {}

    def step():
        stack.decode(h, br, gt, out=out, stream=st)

    def step_chain():
        state, write = h.view(1, -1), (br.view(1, -1), gt.view(1, -1))
        for lay in layers:
            mixed, written, inj = ops.hc_mix(state, lay["nw"], lay["down"], lay["up"], lay["inj"], write=write,
                                             stream=st)
            sh = ops.shared_expert(mixed, lay["sg"], lay["su"], lay["sd"], lay["se"], stream=st)
            state, write = written, (sh, inj)
        chain_out["state"] = hc_write(state, write[0], write[1])
        chain_out["branch"] = write[0]

    def timed(graph, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(n):
            graph.replay()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    with torch.cuda.stream(st):
        step()
        step_chain()
        torch.cuda.synchronize()
        gchain = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gchain, stream=st):
            step_chain()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            step()
        for _ in range(args.warmup):
            gchain.replay()
            graph.replay()
        torch.cuda.synchronize()
        same = bool(torch.equal(out["state"], chain_out["state"].view(-1)) and
                    torch.equal(out["branch"], chain_out["branch"].view(-1)))
        chain_ms = timed(gchain, args.steps)
        clk = ClockSampler(local_rank)
        clk.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(args.steps):
            graph.replay()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        e2e = None
        if not args.no_e2e:
            hp = torch.empty(HC * H, dtype=torch.bfloat16).pin_memory()
            hp.copy_(h.cpu())
            op = torch.empty(H, dtype=torch.bfloat16).pin_memory()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                h.copy_(hp, non_blocking=True)
                graph.replay()
                op.copy_(out["branch"], non_blocking=True)
                st.synchronize()
            dt = time.perf_counter() - t0
            e2e = {"value": round(args.steps / dt, 2), "unit": "tok/s", "h2d_bytes_per_step": hp.numel() * 2,
                   "d2h_bytes_per_step": op.numel() * 2}
        clocks = clk.stop()
    peak, src = peaks()
    achieved = wbytes / (ms / 1000.0) / 1e9
    cpu = None
    if not args.no_cpu:
        from oracle import oracle as orc
        rng = np.random.default_rng(4)
        lay = layers[0]
        tonp = lambda m: (m.w.cpu().numpy().view(np.uint32), m.s.view(torch.int16).cpu().numpy().view(np.uint16),
                          m.b.view(torch.int16).cpu().numpy().view(np.uint16))
        nw = lay["nw"].view(torch.int16).cpu().numpy().view(np.uint16)
        mats = {k: tonp(lay[k]) for k in ("down", "up", "inj", "sg", "su", "sd", "se")}
        hx = h.view(1, -1).view(torch.int16).cpu().numpy().view(np.uint16)
        bx = br.view(1, -1).view(torch.int16).cpu().numpy().view(np.uint16)
        gx = gt.view(1, -1).view(torch.int16).cpu().numpy().view(np.uint16)
        orc.set_threads(os.cpu_count() or 1)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 8.0:
            o = orc.hc_mix(hx, nw, mats["down"], mats["up"], mats["inj"], branch=bx, gate=gx)
            orc.shared_expert(o["mixed"], mats["sg"], mats["su"], mats["sd"], mats["se"])
            n += 1
        per = (time.perf_counter() - t0) / n
        cpu = {"value": round(1.0 / (L * per), 3), "unit": "tok/s", "cores": orc.num_threads(), "kind": "port",
               "sample": f"{n} token-layers (mixer + shared expert of one layer) in 8 s, extrapolated x{L}; "
                         "C restatement"}
    line = {"metric": "MoE-block front (hyper-connection mixer + shared expert) decode tok/s, 28 layers",
            "value": round(1000.0 / ms, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8/u4 codes x bf16 -> f32/f64", "data": "synthetic",
            "config": {"workload": "f3_hc4x3072_r320_shared768_28layers", "layers": L, "streams": HC, "hidden": H,
                       "rank": R, "shared_inter": I, "tokens": 1, "l2": "weights of 28 layers (347 MB) > L2",
                       "chained": "each layer's mixer writes the previous layer's shared-expert output"},
            "per_layer_launches": {"ms_per_step": round(chain_ms, 4), "value": round(1000.0 / chain_ms, 2),
                                   "launches_per_step": 5 * L, "same_bits": same},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "algorithmic_bytes_per_step": wbytes, "peak_source": src},
            "clocks": clocks, "gpu_launches": args.steps, "e2e": e2e, "cpu_baseline": cpu}
    del graph, gchain
    print(json.dumps(line), flush=True)


def run_f3moe(args, rank: int, world: int, local_rank: int) -> None:
    """The whole MoE half of every decoder layer at decode (one token), fused: the f3 step
    (hyper-connection mixer with the previous block's write, 4 streams of H = 3072, rank 320,
    8-bit; shared expert I = 768 4-bit with an 8-bit scalar gate) and the c1 routed block (512
    experts top-10, I = 768, 2-bit g64 fp16 scales, bf16 router) on the mixer output, combined
    as moe_experts_down with the shared output as its addend, for 28 chained layers. The step is
    ONE launch of moe_f3moe_stack_decode (five grid barriers per layer); the same chain as
    per-layer launches (moe_hc_mix, moe_router_topk, moe_shared_expert, moe_experts_gateup,
    moe_experts_down: 8 kernels per layer, one CUDA graph) is timed beside it. roofline =
    algorithmic bytes per token (mixer + shared weights, the router and the 10 routed experts'
    bytes of every layer) / step time against the HBM peak; e2e adds the pinned host copies of
    the token's streams in and the last block output out."""
    import numpy as np
    import torch

    from moe_offload_b200 import ops
    from moe_offload_b200._lib import call
    from moe_offload_b200.ops import QMatrix
    from moe_offload_b200.synthetic import C1, dev_stack

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L = args.layers or C1.layers
    HC, H, R, Is, K = 4, C1.hidden, 320, 768, C1.top_k
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    mix = f3_mix_layers(dev, g, L, HC, H, R, Is)
    routed = dev_stack(C1, dev, layers=L)
    E, I = C1.experts, C1.inter
    mix_bytes = sum(m.w.numel() * 4 + m.s.numel() * 4 for lay in mix for m in lay.values() if isinstance(m, QMatrix))
    routed_bytes = L * (K * int(call("moe_packed_expert_bytes", H, I)) + E * H * 2)
    wbytes = mix_bytes + routed_bytes
    resident_gb = (mix_bytes + L * E * int(call("moe_packed_expert_bytes", H, I))) / 1e9
    h = (torch.randn(HC * H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    br = (torch.randn(H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    gt = (torch.randn(HC, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    st = torch.cuda.Stream(dev)
    stack = ops.F3MoeStack(mix, routed, K, dev)
    out, chain_out = {}, {}
    r_out = [{} for _ in range(L)]

    def step():
        stack.decode(h, br, gt, out=out, stream=st)

    def step_chain():
        state, write = h.view(1, -1), (br.view(1, -1), gt.view(1, -1))
        inds = []
        for lay, rl, ro in zip(mix, routed, r_out):
            mixed, written, inj = ops.hc_mix(state, lay["nw"], lay["down"], lay["up"], lay["inj"], write=write,
                                             stream=st)
            r = ops.router_topk(mixed, rl.router, K, out=ro, stream=st)
            sh = ops.shared_expert(mixed, lay["sg"], lay["su"], lay["sd"], lay["se"], stream=st)
            act = ops.experts_gateup(mixed, r["inds"], rl.gate, rl.up, stream=st)
            y, _ = ops.experts_down(act, r["inds"], rl.down, r["scores"], addend=sh, stream=st)
            inds.append(r["inds"])
            state, write = written, (y, inj)
        chain_out["branch"] = write[0]
        chain_out["inds"] = inds

    def timed(graph, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(n):
            graph.replay()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    with torch.cuda.stream(st):
        step()
        step_chain()
        torch.cuda.synchronize()
        gchain = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gchain, stream=st):
            step_chain()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            step()
        for _ in range(args.warmup):
            gchain.replay()
            graph.replay()
        torch.cuda.synchronize()
        ci = torch.stack([x.view(-1) for x in chain_out["inds"]])
        layers_same = int((ci == out["inds"]).all(dim=1).sum())
        rel = float((out["branch"].float() - chain_out["branch"].view(-1).float()).norm() /
                    chain_out["branch"].float().norm())
        chain_ms = timed(gchain, args.steps)
        clk = ClockSampler(local_rank)
        clk.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(args.steps):
            graph.replay()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        dev_err = int(call("moe_device_error", 1))
        e2e = None
        if not args.no_e2e:
            hp = torch.empty(HC * H, dtype=torch.bfloat16).pin_memory()
            hp.copy_(h.cpu())
            op = torch.empty(H, dtype=torch.bfloat16).pin_memory()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                h.copy_(hp, non_blocking=True)
                graph.replay()
                op.copy_(out["branch"], non_blocking=True)
                st.synchronize()
            dt = time.perf_counter() - t0
            e2e = {"value": round(args.steps / dt, 2), "unit": "tok/s", "h2d_bytes_per_step": hp.numel() * 2,
                   "d2h_bytes_per_step": op.numel() * 2}
        clocks = clk.stop()
    peak, src = peaks()
    achieved = wbytes / (ms / 1000.0) / 1e9
    cpu = None
    if not args.no_cpu:
        from oracle import oracle as orc
        lay = mix[0]
        tonp = lambda m: (m.w.cpu().numpy().view(np.uint32), m.s.view(torch.int16).cpu().numpy().view(np.uint16),
                          m.b.view(torch.int16).cpu().numpy().view(np.uint16))
        nw = lay["nw"].view(torch.int16).cpu().numpy().view(np.uint16)
        mats = {k: tonp(lay[k]) for k in ("down", "up", "inj", "sg", "su", "sd", "se")}
        hx = h.view(1, -1).view(torch.int16).cpu().numpy().view(np.uint16)
        bx = br.view(1, -1).view(torch.int16).cpu().numpy().view(np.uint16)
        gx = gt.view(1, -1).view(torch.int16).cpu().numpy().view(np.uint16)
        orc.set_threads(os.cpu_count() or 1)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 6.0:
            o = orc.hc_mix(hx, nw, mats["down"], mats["up"], mats["inj"], branch=bx, gate=gx)
            orc.shared_expert(o["mixed"], mats["sg"], mats["su"], mats["sd"], mats["se"])
            n += 1
        mix_per = (time.perf_counter() - t0) / n
        routed_cpu = cpu_layer_sample(6.0)
        routed_per = 1.0 / (routed_cpu["value"] * C1.layers)
        cpu = {"value": round(1.0 / (L * (mix_per + routed_per)), 3), "unit": "tok/s", "cores": orc.num_threads(),
               "kind": "port",
               "sample": f"{n} token-layers of the mixer + shared expert in 6 s plus the routed block's own sample "
                         f"({routed_cpu['sample']}), per-layer times added and extrapolated x{L}; C restatement"}
    line = {"metric": "MoE half of the decoder layer (mixer + routed + shared expert) decode tok/s, 28 layers",
            "value": round(1000.0 / ms, 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8/u4/u2 codes x bf16 -> f32/f64", "data": "synthetic",
            "config": {"workload": "f3moe_hc4x3072_r320_shared768_routed512top10_28layers", "layers": L,
                       "streams": HC, "hidden": H, "rank": R, "shared_inter": Is, "experts": E, "top_k": K,
                       "inter": I, "tokens": 1, "l2": f"weights of {L} layers ({resident_gb:.1f} GB) > L2",
                       "chained": "each layer's mixer writes the previous layer's block output"},
            "per_layer_launches": {"ms_per_step": round(chain_ms, 4), "value": round(1000.0 / chain_ms, 2),
                                   "launches_per_step": 8 * L, "layers_same_routing": layers_same,
                                   "final_branch_rel": round(rel, 5)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "algorithmic_bytes_per_step": wbytes, "mix_shared_bytes_per_step": mix_bytes,
                         "routed_bytes_per_step": routed_bytes, "peak_source": src},
            "clocks": clocks, "gpu_launches": args.steps, "device_error": dev_err, "e2e": e2e, "cpu_baseline": cpu}
    del graph, gchain
    print(json.dumps(line), flush=True)


PRED_RECALL = 0.836     # recall@10 of the reference's next-layer predictor (its README.md:35)


def run_c2(args, rank: int, world: int, local_rank: int) -> None:
    """the 28 x 512 x top-10 stack with the offload cache on (layer 0
    pinned, 102 slots per cached layer, experts in a pinned host pool, synthetic Zipf(1.1)
    routing with 30 % reuse injected as the routed experts while the router still runs,
    next-layer prefetch of the top-12 of a predictor with the reference's recall@10, capped
    at 3 per layer)."""
    import torch

    from moe_offload_b200.offload import (HostExpertPool, OffloadStack, compute_layer_capacities,
                                          synthetic_predictions, zipf_routing)
    from moe_offload_b200.synthetic import C2, dev_bf16_normal, dev_stack

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = C2
    L = args.layers or cfg.layers
    layers = dev_stack(cfg, dev, layers=L)
    routers = [ly.router for ly in layers]
    pools = [HostExpertPool.from_layer(layers[l]) for l in range(1, L)]
    layer0 = layers[0]
    for l in range(1, L):
        layers[l] = None
    torch.cuda.empty_cache()
    caps = compute_layer_capacities(budget_pct=20, num_layers=L, num_experts=cfg.experts,
                                    expert_bytes=cfg.expert_bytes)
    stack = OffloadStack(routers, layer0, pools, caps, cfg.top_k, dev, prefetch=True, prefetch_top_m=12,
                         prefetch_cap=3, expert_bytes=cfg.expert_bytes)
    for c in stack.layers[1:]:
        c.prefetch_ctas = args.prefetch_ctas
    T = args.warmup + args.steps
    routing, bias = zipf_routing(seed=cfg.seed, layers=L, tokens=T, E=cfg.experts, K=cfg.top_k)
    # prefetch driven by a predictor of the reference's measured recall@10 (83.6 %)
    preds = synthetic_predictions(routing, bias, recall=PRED_RECALL, M=12, seed=cfg.seed)
    inject = torch.from_numpy(routing).to(dev)
    pred_dev = torch.from_numpy(preds).to(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed)
    h = dev_bf16_normal((T, 1, cfg.hidden), dev, gen)
    stack.capture(pred_injected=True)    # the warm-up token of the capture runs through the caches too
    for t in range(args.warmup):
        stack.decode_graph(h[t], inject[t], pred_dev[t])
    torch.cuda.synchronize()
    stack.reset_stats()
    torch.cuda.synchronize()
    clk = ClockSampler(local_rank)
    clk.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for t in range(args.warmup, T):
        stack.decode_graph(h[t], inject[t], pred_dev[t])
    e.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    t_ms = s.elapsed_time(e)
    tot = stack.decode_totals()
    req = max(1, tot["decode_requests"])
    fill_bytes = tot["decode_demand_bytes"] + tot["decode_prefetch_bytes"]
    h2d = fill_bytes / (t_ms / 1000.0) / 1e9
    peak_h2d = h2d_peak_gbs(dev)
    from moe_offload_b200 import _lib
    dev_err = int(_lib.call("moe_device_error", 1))
    value = args.steps / (t_ms / 1000.0)
    line = {"metric": "MoE decode tok/s (28-layer offload stack, 20 % LRU slot caches)", "value": round(value, 2),
            "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u2 codes x bf16 -> f32", "data": "synthetic",
            "config": {"workload": cfg.name, "layers": L, "hidden": cfg.hidden, "experts": cfg.experts,
                       "top_k": cfg.top_k, "inter": cfg.inter, "capacity": caps[1], "layer0": "pinned",
                       "routing": "Zipf(1.1) per layer + 30 % reuse, injected; router runs",
                       "prefetch": f"top-12 ranked predictions of recall@10 {PRED_RECALL} (the reference's "
                                   "measured predictor recall; offload.synthetic_predictions), cap 3; the "
                                   "router's own next-layer prediction still runs",
                       "prefetch_fill_ctas": args.prefetch_ctas},
            "cache": {"lru_hit_rate": round(tot["decode_lru_hits"] / req, 4),
                      "prefetch_hit_rate": round(tot["decode_prefetch_hits"] / req, 4),
                      "effective_hit_rate": round((tot["decode_lru_hits"] + tot["decode_prefetch_hits"]) / req, 4),
                      "demand_misses_per_token": round(tot["decode_demand_misses"] / args.steps, 2),
                      "fill_bytes_per_token": int(fill_bytes / args.steps)},
            "roofline": {"bound": "h2d link", "achieved": round(h2d, 2), "peak": round(peak_h2d, 2), "unit": "GB/s",
                         "frac": round(h2d / peak_h2d, 4), "peak_source": "pinned cudaMemcpyAsync measured in this run"},
            "clocks": clocks, "device_error": dev_err}
    print(json.dumps(line), flush=True)
    stack.close()


def run_c3(args, rank: int, world: int, local_rank: int) -> None:
    """prefill of a 2048-token prompt through the resident 28 x 512 x top-10
    stack (c3), or one Nemotron-shaped layer (c3n: 240 experts, top-9, H 2688, I 1856, 1024
    tokens). A step = every layer's moe_prefill_layer (per-row power-of-two RMS input
    normalisation, router + exact top-k, expert-grouped tcgen05 GEMMs, combine + residual)."""
    import dataclasses

    import torch

    from moe_offload_b200 import ops
    from moe_offload_b200.synthetic import C3, C3_TOKENS, NEMOTRON, NEMOTRON_TOKENS, dev_bf16_normal, dev_stack

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg, T = (C3, C3_TOKENS) if args.config == "c3" else (NEMOTRON, NEMOTRON_TOKENS)
    if args.layers:
        cfg = dataclasses.replace(cfg, name=f"{cfg.name}_first{args.layers}", layers=args.layers)
    layers = dev_stack(cfg, dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed + 1000 * rank)
    n_in = args.warmup + args.steps
    h0 = dev_bf16_normal((n_in, T, cfg.hidden), dev, gen)
    bufs = [dict(), dict()]

    def step(h):
        for li, ly in enumerate(layers):
            o = ops.prefill_layer(h, ly.router, ly.gate, ly.up, ly.down, cfg.top_k, norm=True, resid=h,
                                  out=bufs[li & 1])
            h = o["y"]
        return h

    for i in range(args.warmup):
        step(h0[i])
    torch.cuda.synchronize()
    clk = ClockSampler(local_rank)
    clk.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        step(h0[args.warmup + i])
    e.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    t_ms = s.elapsed_time(e)
    value = args.steps * T / (t_ms / 1000.0)

    # breakdown on the first layer: router (with the normalisation) vs the expert GEMMs
    ly = layers[0]
    x = h0[0]
    n_rep = 3
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    r = ops.router_topk(x, ly.router, cfg.top_k)
    ops.prefill_experts(x, r["inds"], r["scores"], ly.gate, ly.up, ly.down, resid=x)
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(n_rep):
        r = ops.router_topk(x, ly.router, cfg.top_k, out=r)
    ev[1].record()
    for _ in range(n_rep):
        ops.prefill_experts(x, r["inds"], r["scores"], ly.gate, ly.up, ly.down, resid=x)
    ev[2].record()
    torch.cuda.synchronize()
    router_ms = ev[0].elapsed_time(ev[1]) / n_rep
    experts_ms = ev[1].elapsed_time(ev[2]) / n_rep

    # routing of one step, layer by layer: experts that receive at least one token (the bytes a
    # layer's GEMMs must read; the synthetic distributions concentrate deep layers' routing)
    active = []
    h = h0[0]
    for li, ly in enumerate(layers):
        o = ops.prefill_layer(h, ly.router, ly.gate, ly.up, ly.down, cfg.top_k, norm=True, resid=h,
                              out=bufs[li & 1])
        active.append(int(torch.unique(o["inds"]).numel()))
        h = o["y"]

    # e2e through the public API: the prompt's hidden states from pinned host memory, the
    # final hidden states back to pinned host memory, every step
    e2e = None
    if not args.no_e2e:
        hh = torch.empty((2, T, cfg.hidden), dtype=torch.bfloat16, pin_memory=True)
        hh.copy_(h0[:2])
        out_host = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, pin_memory=True)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(args.steps):
            hd = hh[i & 1].to(dev, non_blocking=True)
            out_host.copy_(step(hd), non_blocking=True)
        e2.record()
        torch.cuda.synchronize()
        t2 = s2.elapsed_time(e2)
        e2e = {"value": round(args.steps * T / (t2 / 1000.0), 2), "unit": "tok/s",
               "h2d_bytes_per_step": T * cfg.hidden * 2, "d2h_bytes_per_step": T * cfg.hidden * 2,
               "api": "moe_offload_b200.ops.prefill_layer per layer (pinned host prompt in, hidden states out)"}

    H, I, K, E = cfg.hidden, cfg.inter, cfg.top_k, cfg.experts
    flops_layer = 2.0 * T * K * 3 * H * I
    bytes_layer = E * cfg.expert_bytes
    tf_peak = 1661.3
    try:
        tf_peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
        tf_src = "measured"
    except Exception:
        tf_src = "fallback"
    hbm_peak, _ = peaks()
    achieved = flops_layer / (experts_ms / 1000.0) / 1e12
    roof = {"kernel": "moe_prefill_experts (bucketing + grouped tcgen05 gate/up and down GEMMs + combine)",
            "bound": "tensor", "achieved": round(achieved, 2), "peak": tf_peak, "unit": "TFLOP/s",
            "frac": round(achieved / tf_peak, 4), "traffic": None,
            "algorithmic_flops_per_launch": flops_layer, "algorithmic_bytes_per_launch": bytes_layer,
            "launch_ms": round(experts_ms, 4), "hbm_frac": round(bytes_layer / (experts_ms / 1000.0) / 1e9 / hbm_peak, 4),
            "router_ms_per_layer": round(router_ms, 4), "peak_source": tf_src,
            "active_experts_per_layer": {"layer0": active[0], "mean": round(sum(active) / len(active), 1),
                                         "min": min(active), "max": max(active)},
            "active_expert_bytes_per_layer": int(sum(active) / len(active) * cfg.expert_bytes)}
    from moe_offload_b200 import _lib
    dev_err = int(_lib.call("moe_device_error", 1))
    cpu = None
    if not args.no_cpu:
        cpu = cpu_layer_sample()
        cpu["sample"] += "; the restatement computes each prompt token like a decode token"
    line = {"metric": f"MoE prefill tok/s ({cfg.layers}-layer stack, {T}-token prompt)", "value": round(value, 2),
            "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u2 codes -> bf16 x bf16 -> f32", "data": "synthetic",
            "config": {"workload": cfg.name, "layers": cfg.layers, "tokens": T, "hidden": H, "experts": E,
                       "top_k": K, "inter": I, "group_size": cfg.group_size, "scales": "fp16", "router": "bf16",
                       "l2": f"inputs larger than L2: {cfg.layers * bytes_layer / 1e9:.1f} GB of weights per step"},
            "roofline": roof, "clocks": clocks,
            # per layer: row normalisation, router, count, scan, scatter, gate/up GEMM, down GEMM, combine
            "gpu_launches": 8 * cfg.layers * args.steps, "device_error": dev_err, "e2e": e2e,
            "cpu_baseline": cpu}
    print(json.dumps(line), flush=True)


def run_c4(args, rank: int, world: int, local_rank: int) -> None:
    """the 28 x 512 x top-10 stack with the experts split across the N
    ranks (512/N each, contiguous blocks), the routers replicated. A step = a batch of B tokens
    through all 28 layers, the whole step one CUDA graph per rank. Batches of at least 4 tokens
    per rank run token-sharded (each rank owns B/N tokens; per layer a routed all-to-all:
    dispatch of each token's row to the ranks holding its experts, local experts, return of
    each output row to its token's owner, MLX-order combine); smaller batches run with the
    tokens replicated (one NVLink exchange + combine per layer). Default B = 8 * N: a fixed
    number of tokens (and so of expert bytes) per GPU as N grows. B = 4096 is c4's prefill."""
    import torch
    import torch.distributed as dist

    from moe_offload_b200.ep import (A2A_MIN_TOKENS_PER_RANK, EPA2AStack, EPDecodeStack, ep_a2a_layer,
                                     expert_bounds, expert_shard, local_tokens)
    from moe_offload_b200.synthetic import C4, dev_bf16_normal, dev_stack_shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = C4
    L = args.layers or cfg.layers
    B = args.batch or 8 * world
    sharded = (B >= A2A_MIN_TOKENS_PER_RANK * world) if args.ep_mode == "auto" else args.ep_mode == "sharded"
    first, n = expert_shard(cfg.experts, rank, world)
    layers = dev_stack_shard(cfg, dev, first, n, layers=L)
    gen = torch.Generator(device=dev)
    gen.manual_seed(cfg.seed)                       # the same batch on every rank
    n_in = args.warmup + args.steps
    h0 = dev_bf16_normal((n_in, B, cfg.hidden), dev, gen)
    if sharded:
        ef = expert_bounds(cfg.experts, world)
        g0, tn = local_tokens(B, world, rank)
        st = EPA2AStack(layers, cfg.experts, ef, cfg.top_k, B, dev)
        xin = h0[:, g0:g0 + tn]
    else:
        st = EPDecodeStack(layers, cfg.experts, first, cfg.top_k, B, dev)
        g0, tn = 0, B
        xin = h0
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        st.step_device(xin[i])
    torch.cuda.synchronize()
    barrier()
    clk = ClockSampler(local_rank)
    clk.start()
    torch.cuda.synchronize()
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        st.step_device(xin[args.warmup + i])
    e.record()
    torch.cuda.synchronize()
    barrier()
    clocks = clk.stop()
    t_ms = s.elapsed_time(e)
    # routing of the whole batch in the last step (every rank's tokens): each rank's unique
    # local experts per layer give the expert bytes the step had to read
    inds_local = st.inds[:, :max(tn, 1)].clone() if sharded else st.inds.clone()
    if sharded and world > 1:
        parts = [torch.zeros_like(inds_local) for _ in range(world)]
        dist.all_gather(parts, inds_local)
        counts = [local_tokens(B, world, q)[1] for q in range(world)]
        inds_all = torch.cat([p[:, :c] for p, c in zip(parts, counts)], dim=1)
    else:
        inds_all = inds_local
    ia = inds_all.cpu().numpy()
    uniq = sum(len({int(v) for v in ia[l].ravel() if first <= v < first + n}) for l in range(L))
    stats = torch.tensor([t_ms, float(uniq)], dtype=torch.float64, device=dev)
    if world > 1:
        tmax = stats[:1].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        usum = stats[1:].clone()
        dist.all_reduce(usum, op=dist.ReduceOp.SUM)
        t_ms, uniq_all = float(tmax.item()), float(usum.item())
    else:
        uniq_all = float(uniq)
    value = B * args.steps / (t_ms / 1000.0)
    from moe_offload_b200 import _lib
    dev_err = int(_lib.call("moe_device_error", 1))

    e2e = None
    if not args.no_e2e:
        hh = xin.cpu().pin_memory()
        out_host = torch.empty((max(tn, 1), cfg.hidden), dtype=torch.bfloat16, pin_memory=True)[:tn]
        for i in range(min(args.warmup, 3)):
            st.decode(hh[i], out_host)
        torch.cuda.synchronize()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(args.steps):
            st.decode(hh[args.warmup + i], out_host)
        e2.record()
        torch.cuda.synchronize()
        barrier()
        t2 = s2.elapsed_time(e2)
        if world > 1:
            tt = torch.tensor([t2], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t2 = float(tt.item())
        cls = "EPA2AStack" if sharded else "EPDecodeStack"
        e2e = {"value": round(B * args.steps / (t2 / 1000.0), 2), "unit": UNIT,
               "h2d_bytes_per_step": tn * cfg.hidden * 2, "d2h_bytes_per_step": tn * cfg.hidden * 2,
               "api": f"moe_offload_b200.ep.{cls}.decode (each rank: its tokens from pinned host memory in, "
                      "out, sync per step)"}

    # bit-exact check on a small slice: layer 0 on the first batch through the expert-parallel
    # layer, against the single-GPU layer with all 512 experts on rank 0
    check = None
    if sharded and not args.no_check:
        from moe_offload_b200 import ops
        from moe_offload_b200.ep import ExchangeBuffers
        xb = ExchangeBuffers(B, cfg.top_k, cfg.hidden, dev, a2a=True)
        o = ep_a2a_layer(xin[0], layers[0], cfg.experts, ef, cfg.top_k, B, xb, norm=True, resid=xin[0])
        torch.cuda.synchronize()
        ok = torch.tensor([1.0], device=dev)
        if rank == 0:
            import dataclasses
            full = [dev_stack_shard(cfg, dev, *expert_shard(cfg.experts, q, world), layers=1)[0] for q in range(world)]
            cat = lambda f: torch.cat([f(ly) for ly in full])
            from moe_offload_b200.ops import QMatrix
            qm = lambda nm: QMatrix(cat(lambda ly: getattr(ly, nm).w), cat(lambda ly: getattr(ly, nm).s),
                                    cat(lambda ly: getattr(ly, nm).b), 2, 64)
            ref = ops.prefill_layer if B >= 32 else ops.decode_layer
            r = ref(h0[0], layers[0].router, qm("gate"), qm("up"), qm("down"), cfg.top_k, norm=True, resid=h0[0])
            torch.cuda.synchronize()
            eq = all(torch.equal(o[k], r[k][g0:g0 + tn]) for k in ("inds", "scores", "y"))
            ok.fill_(1.0 if eq else 0.0)
            del full, r
        xb.close()
        check = {"layer0_rank0_tokens_bit_exact_vs_single_gpu": bool(ok.item() == 1.0),
                 "reference": "ops.prefill_layer" if B >= 32 else "ops.decode_layer"}
    peak, peak_kind = peaks()
    step_bytes = uniq_all * cfg.expert_bytes + world * L * cfg.router_bytes
    achieved = step_bytes / (t_ms / 1000.0 / args.steps) / 1e9
    roof = {"kernel": ("token-sharded expert-parallel step (router, dispatch all-to-all, local experts, return "
                       "all-to-all + combine per layer)") if sharded else
                      "expert-parallel step (router, gate/up, down, NVLink exchange + combine per layer)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": round(peak * world, 1), "unit": "GB/s",
            "frac": round(achieved / (peak * world), 4), "traffic": None,
            "algorithmic_bytes_per_launch": int(step_bytes), "peak_source": f"{peak_kind} x {world} GPUs",
            "unique_experts_per_layer": round(uniq_all / L, 2),
            "unique_expert_bytes_per_layer": int(uniq_all / L * cfg.expert_bytes)}
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak" if not args.batch else "strong", "vs_baseline": None,
                "dtype": "u2 codes x bf16 -> f32", "data": "synthetic",
                "config": c4_config(cfg, world, B, sharded, L),
                "roofline": roof, "clocks": clocks, "gpu_launches": st.launches_per_step * args.steps,
                "device_error": dev_err, "check": check, "e2e": e2e, "cpu_baseline": None}
        print(json.dumps(line), flush=True)
    st.close()


def run_f4(args, rank: int, world: int, local_rank: int) -> None:
    """f4: the greedy decode loop of the reference's server / generate_greedy (server.py:113-199,
    loader.py:1171-1190) around the c1 stack: per token the embedding row of the previous id,
    the persistent stack launch (28 layers), the LM head over a 248,320-id vocabulary (the
    reference model's, prompt_cache.py:149) and the argmax, captured as one CUDA graph per token
    (tokens.ResidentTokenLoop). Synthetic seeded embedding / head tables of the model's shape.
    `value`: tokens per second with the loop's id kept on the device (graph replays back to
    back); `e2e`: the same loop reading every id back to the host before the next step, as the
    reference does for its stop test."""
    import torch

    from moe_offload_b200 import _lib
    from moe_offload_b200.stack import PersistentStack
    from moe_offload_b200.synthetic import C1, dev_stack
    from moe_offload_b200.tokens import ResidentTokenLoop, TokenHead

    if world > 1:
        raise SystemExit("f4 runs on one GPU")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg, V = C1, 248_320
    layers = dev_stack(cfg, dev)
    stack = PersistentStack(layers, cfg.top_k, dev, release_unpacked=True)
    del layers
    torch.cuda.empty_cache()
    head = TokenHead.synthetic(V, cfg.hidden, dev, seed=cfg.seed + 101)
    loop = ResidentTokenLoop(stack, head)
    loop.start(65)
    for _ in range(args.warmup):
        loop.step()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream(dev)
    clk = ClockSampler(local_rank)
    clk.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    run = loop.graph.replay if loop.graph is not None else loop._body     # the graph, or the direct step
    for _ in range(args.steps):
        run()
    e.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    t_ms = s.elapsed_time(e)
    # the fused LM head + argmax alone (the step's largest read), and the stand-alone argmax
    # over stored logits (moe_sample_tokens at temperature 0), for the step's split
    saved = loop.cur.clone()
    hs, he = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    hs.record()
    for _ in range(args.steps):
        head.argmax(stack.y, out=loop.cur)
    he.record()
    torch.cuda.synchronize()
    head_ms = hs.elapsed_time(he) / args.steps
    head.logits(stack.y, out=loop.logits)
    ss, se = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ss.record()
    for _ in range(args.steps):
        head.sample(loop.logits, out=loop.cur)
    se.record()
    torch.cuda.synchronize()
    argmax_ms = ss.elapsed_time(se) / args.steps
    loop.cur.copy_(saved)
    dev_err = int(_lib.call("moe_device_error", 1))
    e2e = None
    if not args.no_e2e:
        ids = []
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            ids.append(loop.step())
        e2.record()
        torch.cuda.synchronize()
        t2 = s2.elapsed_time(e2)
        e2e = {"value": round(args.steps / (t2 / 1000.0), 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
               "d2h_bytes_per_step": 4, "distinct_ids": len(set(ids)),
               "api": "moe_offload_b200.tokens.ResidentTokenLoop.step (graph replay, next id read back per token)"}
    peak, peak_kind = peaks()
    stack_bytes = cfg.layers * (cfg.top_k * cfg.expert_bytes + cfg.router_bytes)
    step_bytes = stack_bytes + head.head_bytes + cfg.hidden * 2
    step_s = t_ms / 1000.0 / args.steps
    achieved = step_bytes / step_s / 1e9
    head_gbs = head.head_bytes / (head_ms / 1000.0) / 1e9
    roof = {"kernel": "token step (embed + stack_kernel + lm_head_kernel with the argmax folded in)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": None, "algorithmic_bytes_per_launch": step_bytes, "launch_us": round(step_s * 1e6, 2),
            "peak_source": peak_kind,
            "lm_head": {"us": round(head_ms * 1000, 2), "bytes": head.head_bytes, "gbs": round(head_gbs, 1),
                        "frac": round(head_gbs / peak, 4)},
            "separate_argmax_over_logits_us": round(argmax_ms * 1000, 2)}
    line = {"metric": "greedy decode tok/s (embedding + 28-layer expert stack + 248,320-id LM head + argmax)",
            "value": round(args.steps / (t_ms / 1000.0), 2), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u2 codes x bf16 -> f32; bf16 head -> f32 logits",
            "data": "synthetic",
            "config": {"workload": "f4_greedy_loop_c1_stack_vocab248320", "layers": cfg.layers, "hidden": cfg.hidden,
                       "experts": cfg.experts, "top_k": cfg.top_k, "inter": cfg.inter, "vocab": V, "batch": 1,
                       "l2": "inputs larger than L2: 2.2 GB read per token"},
            "roofline": roof, "clocks": clocks, "gpu_launches": loop.launches_per_step * args.steps,
            "device_error": dev_err, "e2e": e2e,
            "cpu_baseline": None if args.no_cpu else cpu_token_sample(V, cfg.hidden)}
    print(json.dumps(line), flush=True)


def main() -> int:
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.config == "c2":
            run_c2(args, rank, world, local_rank)
        elif args.config == "p1":
            run_p1(args, rank, world, local_rank)
        elif args.config == "f3":
            run_f3(args, rank, world, local_rank)
        elif args.config == "f3moe":
            run_f3moe(args, rank, world, local_rank)
        elif args.config == "f4":
            run_f4(args, rank, world, local_rank)
        elif args.config in ("c3", "c3n"):
            run_c3(args, rank, world, local_rank)
        elif args.config == "c4" or (world > 1 and args.config == "c1" and not args.replicas):
            run_c4(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
