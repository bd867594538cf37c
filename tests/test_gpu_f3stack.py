"""The mixer + shared-expert decode of all layers in one launch (moe_f3_stack_decode) against
the per-layer launches it replaces (moe_hc_mix with the previous block's write, then
moe_shared_expert on its output), chained the same way: every layer's block output, the last
stream gate and the final state bit for bit, whatever the number of CTAs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _layers(dev, L, H, R, I, seed, sb=torch.bfloat16, inject=True):
    from moe_offload_b200.ops import QMatrix
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def qm(N, K, bits, scale):
        w = torch.randint(-(2 ** 31), 2 ** 31 - 1, (N, K * bits // 32), dtype=torch.int32, device=dev, generator=g)
        s = (torch.rand((N, K // 64), device=dev, generator=g) * scale + scale / 10).to(sb)
        b = (torch.randn((N, K // 64), device=dev, generator=g) * scale * 4).to(sb)
        return QMatrix(w, s, b, bits, 64)

    out = []
    for _ in range(L):
        out.append({"nw": (torch.randn(4 * H, device=dev, generator=g) * 0.05).to(torch.bfloat16),
                    "down": qm(R, 4 * H, 8, 2e-4), "up": qm(4 * H, R, 8, 2e-3),
                    "inj": qm(4, 4 * H, 8, 2e-4) if inject else None,
                    "sg": qm(I, H, 4, 2e-3), "su": qm(I, H, 4, 2e-3), "sd": qm(H, I, 4, 2e-3), "se": qm(1, H, 8, 2e-4)})
    return out, g


def _chain(layers, h, br, gt):
    from moe_offload_b200 import ops
    from moe_offload_b200.hooks import hc_write
    state, write, outs = h.view(1, -1), (None if br is None else (br.view(1, -1), gt.view(1, -1))), []
    for ly in layers:
        mixed, written, inj = ops.hc_mix(state, ly["nw"], ly["down"], ly["up"], ly["inj"], write=write)
        sh = ops.shared_expert(mixed, ly["sg"], ly["su"], ly["sd"], ly["se"])
        outs.append(sh.view(-1).clone())
        state, write = written.clone(), (sh, inj.clone())
    final = hc_write(state, write[0], write[1])
    return torch.stack(outs), write[1].view(-1), final.view(-1)


@pytest.mark.parametrize("L,H,R,I,with_write,inject,ctas", [
    (3, 512, 64, 256, True, True, 0), (2, 1024, 128, 512, False, True, 128), (2, 512, 64, 256, True, False, 131),
    (4, 3072, 320, 768, True, True, 0)])
def test_f3_stack_matches_per_layer_launches(dev, L, H, R, I, with_write, inject, ctas):
    from moe_offload_b200 import ops
    layers, g = _layers(dev, L, H, R, I, seed=L * 10 + H, inject=inject)
    h = (torch.randn(4 * H, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    br = (torch.randn(H, device=dev, generator=g) * 0.3).to(torch.bfloat16) if with_write else None
    gt = (torch.randn(4, device=dev, generator=g) * 0.5).to(torch.bfloat16) if with_write else None
    stack = ops.F3Stack(layers, dev, num_ctas=ctas)
    for rep in range(2):
        st, bo, inj, alls = stack.decode(h, br, gt, want_all=True)
        ref_all, ref_inj, ref_state = _chain(layers, h, br, gt)
        torch.cuda.synchronize()
        for l in range(L):
            assert torch.equal(alls[l], ref_all[l]), (rep, l, "block output differs")
        assert torch.equal(bo, ref_all[-1])
        assert torch.equal(inj, ref_inj)
        assert torch.equal(st, ref_state)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


def test_f3_stack_fp16_scales_and_graph(dev):
    """fp16 scales; the launch captured in a CUDA graph replays to the same bits."""
    from moe_offload_b200 import ops
    layers, g = _layers(dev, 2, 512, 64, 256, seed=7, sb=torch.float16)
    h = (torch.randn(4 * 512, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    br = (torch.randn(512, device=dev, generator=g) * 0.3).to(torch.bfloat16)
    gt = (torch.randn(4, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    stack = ops.F3Stack(layers, dev)
    out = {}
    st, bo, inj, _ = stack.decode(h, br, gt, out=out)
    ref_all, ref_inj, ref_state = _chain(layers, h, br, gt)
    torch.cuda.synchronize()
    assert torch.equal(bo, ref_all[-1]) and torch.equal(st, ref_state) and torch.equal(inj, ref_inj)
    want = st.clone()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        stack.decode(h, br, gt, out=out, stream=s)
    torch.cuda.current_stream(dev).wait_stream(s)
    out["state"].zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out["state"], want)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0
