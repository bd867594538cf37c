"""The MoE half of every decoder layer at decode in ONE launch (moe_f3moe_stack_decode): the
mixer with the previous block's write, the routing of its output, the routed experts and the
shared expert, combined as moe_experts_down combines them with the shared output as its
addend (loader.py:909-914). Checked against the per-layer launches it replaces, with teacher
forcing from the kernel's own block outputs: every layer's mixer output, routing indices and
scores, the last stream gate and the final state bit for bit; the block output within the
persistent routed stack's tolerance (its expert outputs are split-K sums in another order);
and the same bits whatever the number of CTAs."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
REL_TOL = 1e-2


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _mix_layers(dev, L, H, R, Is, seed, inject=True):
    from moe_offload_b200.ops import QMatrix
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def qm(N, K, bits, scale):
        w = torch.randint(-(2 ** 31), 2 ** 31 - 1, (N, K * bits // 32), dtype=torch.int32, device=dev, generator=g)
        s = (torch.rand((N, K // 64), device=dev, generator=g) * scale + scale / 10).to(torch.bfloat16)
        b = (torch.randn((N, K // 64), device=dev, generator=g) * scale * 4).to(torch.bfloat16)
        return QMatrix(w, s, b, bits, 64)

    out = []
    for _ in range(L):
        out.append({"nw": (torch.randn(4 * H, device=dev, generator=g) * 0.05).to(torch.bfloat16),
                    "down": qm(R, 4 * H, 8, 2e-4), "up": qm(4 * H, R, 8, 2e-3),
                    "inj": qm(4, 4 * H, 8, 2e-4) if inject else None,
                    "sg": qm(Is, H, 4, 2e-3), "su": qm(Is, H, 4, 2e-3), "sd": qm(H, Is, 4, 2e-3),
                    "se": qm(1, H, 8, 2e-4)})
    return out, g


def _routed(dev, L, H, I, E, seed):
    from moe_offload_b200.synthetic import ExpertLayer, np_bf16_normal, np_qmatrix, np_to_bf16_tensor, to_device_qmatrix
    rng = np.random.default_rng(seed)
    return [ExpertLayer(np_to_bf16_tensor(np_bf16_normal(rng, (E, H), 0.02), dev),
                        to_device_qmatrix(np_qmatrix(rng, E, I, H), dev), to_device_qmatrix(np_qmatrix(rng, E, I, H), dev),
                        to_device_qmatrix(np_qmatrix(rng, E, H, I), dev)) for _ in range(L)]


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def _check_against_layers(o, mix, routed, K, h, br, gt):
    """Teacher-forced per-layer launches: hc_mix with the kernel's previous block output,
    router_topk, shared_expert, experts_gateup / experts_down (shared output as addend)."""
    from moe_offload_b200 import ops
    from moe_offload_b200.hooks import hc_write
    state, write = h.view(1, -1), (None if br is None else (br.view(1, -1), gt.view(1, -1)))
    L = len(routed)
    for l in range(L):
        ly, rl = mix[l], routed[l]
        mixed, written, inj = ops.hc_mix(state, ly["nw"], ly["down"], ly["up"], ly["inj"], write=write)
        assert torch.equal(o["mixed_all"][l], mixed.view(-1)), (l, "mixer output differs")
        r = ops.router_topk(mixed, rl.router, K)
        assert torch.equal(o["inds"][l], r["inds"].view(-1).to(torch.int32)), (l, "routing differs")
        assert torch.equal(o["scores"][l], r["scores"].view(-1)), (l, "scores differ")
        sh = ops.shared_expert(mixed, ly["sg"], ly["su"], ly["sd"], ly["se"])
        act = ops.experts_gateup(mixed, r["inds"], rl.gate, rl.up)
        y, _ = ops.experts_down(act, r["inds"], rl.down, r["scores"], addend=sh)
        rel = _rel(o["branch_all"][l], y.view(-1))
        assert rel < REL_TOL, (l, rel)
        state, write = written.clone(), (o["branch_all"][l].view(1, -1), inj.clone())
    final = hc_write(state, write[0], write[1])
    assert torch.equal(o["branch"], o["branch_all"][-1])
    assert torch.equal(o["inj"], write[1].view(-1))
    assert torch.equal(o["state"], final.view(-1))


@pytest.mark.parametrize("L,H,R,Is,I,E,K,with_write,inject,ctas", [
    (2, 1024, 128, 256, 256, 64, 4, True, True, 0),
    (3, 3072, 320, 768, 768, 512, 10, True, True, 0),      # the c1 / f3 layer shapes
    (2, 2048, 64, 512, 768, 64, 8, False, False, 128),
])
def test_f3moe_matches_per_layer_launches(dev, L, H, R, Is, I, E, K, with_write, inject, ctas):
    from moe_offload_b200 import ops
    mix, g = _mix_layers(dev, L, H, R, Is, seed=L * 10 + H, inject=inject)
    routed = _routed(dev, L, H, I, E, seed=H + E)
    h = (torch.randn(4 * H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    br = (torch.randn(H, device=dev, generator=g) * 0.3).to(torch.bfloat16) if with_write else None
    gt = (torch.randn(4, device=dev, generator=g) * 0.5).to(torch.bfloat16) if with_write else None
    stack = ops.F3MoeStack(mix, routed, K, dev, num_ctas=ctas)
    for _ in range(2):
        o = stack.decode(h, br, gt, want_all=True)
        torch.cuda.synchronize()
        _check_against_layers(o, mix, routed, K, h, br, gt)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


def test_f3moe_independent_of_cta_count_and_graph(dev):
    """All SMs vs 128 CTAs: every output bit equal; the launch replayed from a CUDA graph too."""
    from moe_offload_b200 import ops
    L, H, R, Is, I, E, K = 3, 2048, 128, 512, 768, 128, 8
    mix, g = _mix_layers(dev, L, H, R, Is, seed=5)
    routed = _routed(dev, L, H, I, E, seed=6)
    h = (torch.randn(4 * H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    br = (torch.randn(H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    gt = (torch.randn(4, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    a = ops.F3MoeStack(mix, routed, K, dev)
    b = ops.F3MoeStack(mix, routed, K, dev, num_ctas=128)
    oa = a.decode(h, br, gt, want_all=True)
    ob = b.decode(h, br, gt, want_all=True)
    torch.cuda.synchronize()
    for k in ("state", "branch", "inj", "inds", "scores", "branch_all", "mixed_all"):
        assert torch.equal(oa[k], ob[k]), k
    ref = {k: v.clone() for k, v in oa.items()}
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        a.decode(h, br, gt, want_all=True, out=oa, stream=s)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        a.decode(h, br, gt, want_all=True, out=oa, stream=s)
    for v in oa.values():
        v.zero_()
    graph.replay()
    torch.cuda.synchronize()
    for k in ref:
        assert torch.equal(oa[k], ref[k]), k
    del graph
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0
