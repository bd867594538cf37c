"""Host-side logic of expert parallelism on the CPU: the expert partition and the ordered
exchange of IPC handles over a two-rank gloo process group."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("E,world", [(512, 1), (512, 2), (512, 8), (240, 7), (64, 3)])
def test_expert_shard_partitions_all_experts(E, world):
    from moe_offload_b200.ep import expert_shard
    seen = []
    sizes = []
    for r in range(world):
        first, n = expert_shard(E, r, world)
        seen.extend(range(first, first + n))
        sizes.append(n)
    assert seen == list(range(E))
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("T,world", [(64, 8), (40, 2), (7, 3), (3, 8), (4096, 8), (1, 1)])
def test_token_blocks_partition_the_batch(T, world):
    """Token-sharded EP: contiguous blocks of ceil(T/world) tokens cover the batch once (the
    last ranks may get fewer or none), and the expert bounds cover every expert once."""
    from moe_offload_b200.ep import expert_bounds, local_tokens
    seen = []
    for r in range(world):
        first, n = local_tokens(T, world, r)
        assert 0 <= n <= -(-T // world)
        seen.extend(range(first, first + n))
    assert seen == list(range(T))
    ef = expert_bounds(512, world)
    assert ef[0] == 0 and ef[-1] == 512 and all(a < b for a, b in zip(ef, ef[1:]))


def test_expert_shard_rejects_bad_splits():
    from moe_offload_b200.ep import expert_shard
    with pytest.raises(ValueError):
        expert_shard(4, 0, 8)
    with pytest.raises(ValueError):
        expert_shard(64, 2, 2)


def _worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from moe_offload_b200.ep import HANDLE_BYTES, gather_handles
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    mine = bytes([rank + 1]) * HANDLE_BYTES
    got = gather_handles(mine)
    out[rank] = [h[0] for h in got] if all(len(h) == HANDLE_BYTES for h in got) else None
    dist.destroy_process_group()


def test_gather_handles_rank_order_gloo():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        assert out[0] == [1, 2] and out[1] == [1, 2]
