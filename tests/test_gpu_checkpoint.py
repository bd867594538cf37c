"""OffloadEngine over a model directory in the reference's layout (experts-XX.safetensors per
layer, routers in base-00.safetensors, config.json): the engine loaded from the files decodes
bit-identically to an offload stack built in memory from the same tensors (bf16 routers and
an 8-bit affine router), and generate_greedy runs on it."""
import json

import pytest
import torch

from moe_offload_b200 import checkpoint as ck

pytestmark = pytest.mark.gpu

L, E, H, I, K, GS = 3, 16, 512, 128, 4, 64


def _tensors(seed):
    g = torch.Generator().manual_seed(seed)
    mats = []
    for _ in range(L):
        m = []
        for rows, cols in ((I, H), (I, H), (H, I)):
            w = torch.randint(-(2 ** 31), 2 ** 31 - 1, (E, rows, cols * 2 // 32), dtype=torch.int32, generator=g)
            s = (torch.rand((E, rows, cols // GS), generator=g) * 0.04 + 0.005).to(torch.bfloat16)
            b = (torch.randn((E, rows, cols // GS), generator=g) * 0.01).to(torch.bfloat16)
            m.append((w, s, b))
        mats.append(m)
    routers = [(torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16) for _ in range(L - 1)]
    # the last layer's router 8-bit affine, like the real model's
    routers.append((torch.randint(-(2 ** 31), 2 ** 31 - 1, (E, H * 8 // 32), dtype=torch.int32, generator=g),
                    (torch.rand((E, H // GS), generator=g) * 0.002 + 0.0005).to(torch.bfloat16),
                    (torch.randn((E, H // GS), generator=g) * 0.05).to(torch.bfloat16)))
    return mats, routers


def test_engine_from_model_dir_matches_in_memory_stack(tmp_path):
    from moe_offload_b200.engine import OffloadEngine
    from moe_offload_b200.offload import HostExpertPool, OffloadStack
    from moe_offload_b200.ops import QMatrix
    from moe_offload_b200.synthetic import ExpertLayer, dev_bf16_normal
    dev = torch.device("cuda:0")
    mats, routers = _tensors(5)
    for l in range(L):
        ck.write_expert_shard(tmp_path / ck.shard_name(l), l, mats[l])
    ck.write_router_shard(tmp_path / "base-00.safetensors", dict(enumerate(routers)))
    (tmp_path / "config.json").write_text(json.dumps({"text_config": {"num_experts_per_tok": K}}))

    eng = OffloadEngine(model_path=tmp_path, budget_pct=50, device=dev, prefetch=True, prefetch_top_m=6,
                        prefetch_cap=2)
    assert (eng.config.layers, eng.config.experts, eng.config.hidden, eng.config.inter, eng.config.top_k) == (L, E, H, I, K)

    def dq(t):
        return QMatrix(t[0].to(dev), t[1].to(dev), t[2].to(dev), 2, GS)
    dev_routers = [routers[0].to(dev), routers[1].to(dev), QMatrix(*(x.to(dev) for x in routers[2]), 8, GS)]
    layer0 = ExpertLayer(dev_routers[0], *(dq(t) for t in mats[0]))
    pools = [HostExpertPool([t for m in mats[l] for t in m], 2, GS) for l in range(1, L)]
    ref = OffloadStack(dev_routers, layer0, pools, eng.capacities, K, dev, prefetch=True, prefetch_top_m=6,
                       prefetch_cap=2)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    for _ in range(6):
        h = dev_bf16_normal((1, H), dev, gen)
        a = eng.stack.decode_token(h).clone()
        b = ref.decode_token(h).clone()
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    out = eng.generate_greedy("hello", max_new_tokens=4)
    assert out["decode_tokens"] == 4 and out["prompt_tokens"] > 0
    eng.close()
    ref.close()
