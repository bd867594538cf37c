"""Worker for the expert-parallel GPU test (launched by tests/test_gpu_ep.py through
torch.distributed.run, one process per GPU): every rank builds the same seeded numpy stack,
keeps its block of the experts, runs the expert-parallel decode (layer calls and the
graph-captured stack) and checks that its results equal, bit for bit, the single-GPU
decode layers run on its own GPU with all experts; then the same for the token-sharded layer
(routed all-to-all), its own block of the batch. Exits non-zero on a mismatch."""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> int:
    from moe_offload_b200 import _lib, ops
    from moe_offload_b200.ep import EPDecodeStack, ExchangeBuffers, ep_decode_layer, expert_shard, shard_layer
    from moe_offload_b200.synthetic import ExpertLayer, np_bf16_normal, np_qmatrix, np_to_bf16_tensor, to_device_qmatrix

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    L, T, H, I, E, K = 3, 4, 1024, 256, 64, 6
    rng = np.random.default_rng(4)
    full = [ExpertLayer(np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev),
                        to_device_qmatrix(np_qmatrix(rng, E, I, H), dev), to_device_qmatrix(np_qmatrix(rng, E, I, H), dev),
                        to_device_qmatrix(np_qmatrix(rng, E, H, I), dev)) for _ in range(L)]
    first, n = expert_shard(E, rank, world)
    local = [shard_layer(ly, first, n) for ly in full]
    xs = [np_to_bf16_tensor(np_bf16_normal(rng, (T, H)), dev) for _ in range(3)]
    bad = []

    # single layer calls, twice in a row (the epochs advance), batch sizes T and 1, and a
    # batch of 40 (grouped-GEMM path, compared with the single-GPU prefill layer)
    xb = np_to_bf16_tensor(np_bf16_normal(rng, (40, H)), dev)
    xbuf = ExchangeBuffers(40, K, H, dev)
    for x in (xs[0], xs[1][:1], xs[0], xb, xb):
        o = ep_decode_layer(x, local[0], E, first, K, xbuf, norm=True, resid=x)
        ref = ops.decode_layer if x.shape[0] < 32 else ops.prefill_layer
        r = ref(x, full[0].router, full[0].gate, full[0].up, full[0].down, K, norm=True, resid=x)
        torch.cuda.synchronize()
        for key in ("inds", "scores", "y"):
            if not torch.equal(o[key], r[key]):
                bad.append(f"layer call {key} T={x.shape[0]}")
    xbuf.close()

    # the graph-captured stack against a chain of single-GPU decode layers
    st = EPDecodeStack(local, E, first, K, T, dev)
    for x in xs:
        y = st.step_device(x).clone()
        h = x
        for ly in full:
            h = ops.decode_layer(h, ly.router, ly.gate, ly.up, ly.down, K, norm=True, resid=h)["y"]
        torch.cuda.synchronize()
        if not torch.equal(y, h):
            bad.append("stack output")
    st.close()

    # token-sharded (routed all-to-all): this rank's block of a 40-token batch (grouped GEMMs)
    # and of an 8-token batch (GEMVs), layer calls and the graph-captured stack, against the
    # single-GPU layers on the whole batch
    from moe_offload_b200.ep import EPA2AStack, ep_a2a_layer, expert_bounds, local_tokens
    ef = expert_bounds(E, world)
    for TT in (40, 8):
        xa = np_to_bf16_tensor(np_bf16_normal(rng, (TT, H)), dev)
        g0, nt = local_tokens(TT, world, rank)
        xb2 = ExchangeBuffers(TT, K, H, dev, a2a=True)
        for rep in range(2):
            o = ep_a2a_layer(xa[g0:g0 + nt], local[0], E, ef, K, TT, xb2, norm=True, resid=xa[g0:g0 + nt])
            ref = ops.decode_layer if TT < 32 else ops.prefill_layer
            r = ref(xa, full[0].router, full[0].gate, full[0].up, full[0].down, K, norm=True, resid=xa)
            torch.cuda.synchronize()
            for key in ("inds", "scores", "y"):
                if not torch.equal(o[key], r[key][g0:g0 + nt]):
                    bad.append(f"a2a layer {key} T={TT} call {rep}")
        xb2.close()
        sa = EPA2AStack(local, E, ef, K, TT, dev)
        for _ in range(2):
            xa = np_to_bf16_tensor(np_bf16_normal(rng, (TT, H)), dev)
            y = sa.step_device(xa[g0:g0 + nt]).clone()
            h = xa
            for ly in full:
                fn = ops.decode_layer if TT < 32 else ops.prefill_layer
                h = fn(h, ly.router, ly.gate, ly.up, ly.down, K, norm=True, resid=h)["y"]
            torch.cuda.synchronize()
            if not torch.equal(y, h[g0:g0 + nt]):
                bad.append(f"a2a stack output T={TT}")
        sa.close()
    err = int(_lib.call("moe_device_error", 1))
    if err:
        bad.append(f"device error word {err}")
    res = {"rank": rank, "world": world, "shard": [first, n], "bad": bad}
    print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
