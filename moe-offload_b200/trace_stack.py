"""Per-phase timeline of the persistent decode kernel (profiling aid, not part of the op path).

    python moe-offload_b200/build.py --trace          # libmoe_b200_trace.so (MOE_STACK_TRACE)
    python moe-offload_b200/trace_stack.py [--layers 28] [--steps 16] [--fused]

Runs the c1 stack (synthetic BASELINE weights) through the profiling build of the library,
whose kernel stamps %globaltimer at fixed points of every layer, and prints the median over
the middle layers of each point's time from the layer's start (microseconds), over the work-
item CTAs (the first K * I/64) and over the others. --fused: the same routed layers behind the
hyper-connection mixer and with the shared expert, in one launch (ops.F3MoeStack,
f3moe_kernel's stamps).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SLOTS = {"routed": 1, "copies_issued": 2, "unit_bytes_waited": 14, "unit_mma_done": 15, "gateup_done": 3,
         "down_bytes_waited": 10, "item_done": 4, "barrier1_passed": 6, "phaseB_done": 7}
FUSED_SLOTS = {"write_norm_sums": 1, "bar0": 2, "mixer_down": 5, "bar1": 6, "mixer_up_router": 7, "bar2": 8,
               "routed": 9, "shared_gate_up": 11, "unit_bytes_waited": 14, "gateup_done": 3,
               "down_bytes_waited": 10, "items_done": 4, "barA": 12, "phaseB_done": 13}
TRACE_CTAS, TRACE_LAYERS, TRACE_SLOTS = 160, 64, 16


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--fused", action="store_true")
    args = ap.parse_args()
    lib_path = os.path.join(HERE, "libmoe_b200_trace.so")
    if not os.path.exists(lib_path):
        print("build it first: python moe-offload_b200/build.py --trace", file=sys.stderr)
        return 1
    os.environ["MOE_B200_LIB"] = lib_path
    sys.path.insert(0, ROOT)
    import dataclasses

    import numpy as np
    import torch

    from moe_offload_b200.stack import PersistentStack
    from moe_offload_b200.synthetic import C1, dev_bf16_normal, dev_stack

    dev = torch.device("cuda:0")
    cfg = dataclasses.replace(C1, layers=args.layers)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    slots = SLOTS
    if args.fused:
        from bench import f3_mix_layers
        from moe_offload_b200.ops import F3MoeStack
        slots = FUSED_SLOTS
        mix = f3_mix_layers(dev, gen, cfg.layers, 4, cfg.hidden, 320, 768)
        st = F3MoeStack(mix, dev_stack(cfg, dev), cfg.top_k, dev)
        h = dev_bf16_normal((8 + args.steps, 4 * cfg.hidden), dev, gen)
        step = lambda x: st.decode(x)
    else:
        st = PersistentStack(dev_stack(cfg, dev), cfg.top_k, dev, release_unpacked=True)
        h = dev_bf16_normal((8 + args.steps, 1, cfg.hidden), dev, gen)
        step = st.step_device
    for i in range(8):
        step(h[i])
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(8, 8 + args.steps):
        step(h[i])
    e.record()
    torch.cuda.synchronize()
    us_per_token = s.elapsed_time(e) / args.steps * 1000.0
    n = TRACE_CTAS * TRACE_LAYERS * TRACE_SLOTS
    buf = (ctypes.c_ulonglong * n)()
    lib = ctypes.CDLL(lib_path)
    assert lib.moe_stack_trace_read(buf, ctypes.c_size_t(n)) == 0
    t = np.frombuffer(buf, dtype=np.uint64).reshape(TRACE_CTAS, TRACE_LAYERS, TRACE_SLOTS).astype(np.int64)
    G = torch.cuda.get_device_properties(dev).multi_processor_count
    NQ = cfg.top_k * cfg.inter // 64
    L = cfg.layers
    per = {k: [] for k in slots}
    per_idle = {k: [] for k in slots}
    period = []
    for l in range(1, L - 1):
        t0 = t[:G, l, 0].min()
        period.append((t[:G, l + 1, 0].min() - t0) / 1000.0)
        for k, slot in slots.items():
            for dst, rows in ((per, t[:NQ, l, slot]), (per_idle, t[NQ:G, l, slot])):
                v = rows[rows > 0]
                if len(v):
                    dst[k].append(float(np.median(v - t0)) / 1000.0)
    out = {"us_per_token": round(us_per_token, 1), "layer_period_us": round(float(np.median(period)), 2),
           "item_ctas": {k: round(float(np.median(v)), 2) for k, v in per.items() if v},
           "other_ctas": {k: round(float(np.median(v)), 2) for k, v in per_idle.items() if v}}
    print(json.dumps(out, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
