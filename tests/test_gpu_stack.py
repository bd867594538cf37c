"""The persistent stack kernel (one launch, all layers) against the CPU oracle with teacher
forcing (each layer's input taken from the kernel's own hs_out) and against the three-kernel
per-layer path."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu
REL_TOL = 1e-2


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return torch.device("cuda:0")


def _np_layers(rng, L, E, H, I):
    from moe_offload_b200.synthetic import np_bf16_normal, np_qmatrix
    out = []
    for _ in range(L):
        out.append(dict(router=np_bf16_normal(rng, (E, H), 0.02), g=np_qmatrix(rng, E, I, H),
                        u=np_qmatrix(rng, E, I, H), d=np_qmatrix(rng, E, H, I)))
    return out


def _dev_layers(np_layers, dev):
    from moe_offload_b200.synthetic import ExpertLayer, np_to_bf16_tensor, to_device_qmatrix
    return [ExpertLayer(np_to_bf16_tensor(ly["router"], dev), to_device_qmatrix(ly["g"], dev),
                        to_device_qmatrix(ly["u"], dev), to_device_qmatrix(ly["d"], dev)) for ly in np_layers]


# ctas = 0: all SMs (CTAs without a work item exist); (2, 512, 256, 32, 4, 16): one item per CTA;
# (2, 3072, 768, 512, 10, 0): the c1 layer shape of the bench (512 experts, top-10)
@pytest.mark.parametrize("L,H,I,E,K,ctas", [(3, 3072, 768, 64, 10, 0), (6, 2048, 768, 64, 8, 0),
                                           (2, 1024, 256, 32, 4, 40), (2, 512, 256, 32, 4, 16),
                                           (2, 3072, 768, 512, 10, 0)])
def test_persistent_stack_vs_oracle(dev, L, H, I, E, K, ctas):
    from moe_offload_b200.ops import pow2_normalize
    from moe_offload_b200.stack import PersistentStack
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(L * 100 + E)
    nl = _np_layers(rng, L, E, H, I)
    st = PersistentStack(_dev_layers(nl, dev), K, dev, num_ctas=ctas, keep_layer_inputs=True)
    for tok in range(2):
        x = np_bf16_normal(rng, (1, H))
        y = st.step_device(np_to_bf16_tensor(x, dev))
        torch.cuda.synchronize()
        hs = bf16_tensor_to_np(st.hs)
        inds = st.inds.cpu().numpy().astype(np.uint32)
        scores = bf16_tensor_to_np(st.scores)
        assert np.array_equal(hs[0], x[0])
        assert np.array_equal(bf16_tensor_to_np(y)[0], hs[L])
        for li, ly in enumerate(nl):
            hin = hs[li][None]
            xin = pow2_normalize(hin)          # the layer's MoE input (exact power-of-two rescale)
            _, ri, rs = orc.softmax_topk(orc.router_logits(xin, ly["router"], E), K)
            assert np.array_equal(inds[li], ri[0]), f"token {tok} layer {li}: indices differ"
            assert np.array_equal(scores[li], rs[0]), f"token {tok} layer {li}: scores differ"
            ref = orc.experts(xin, ri, rs, ly["g"], ly["u"], ly["d"], sb_fp16=True, resid=hin)["y"]
            a = orc.bf16_to_f32(hs[li + 1]).astype(np.float64) - orc.bf16_to_f32(hin[0])
            b = orc.bf16_to_f32(ref[0]).astype(np.float64) - orc.bf16_to_f32(hin[0])
            rel = np.linalg.norm(a - b) / np.linalg.norm(b)
            assert rel < REL_TOL, (tok, li, rel)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


def test_persistent_stack_results_independent_of_cta_count(dev):
    """All SMs (CTAs without a work item, other phase-B row blocks and logit-replica spread) vs
    exactly one CTA per item: every layer's routing, scores and output bits agree."""
    from moe_offload_b200.stack import PersistentStack
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(33)
    L, H, I, E, K = 6, 2048, 768, 64, 8
    layers = _dev_layers(_np_layers(rng, L, E, H, I), dev)
    a = PersistentStack(layers, K, dev, keep_layer_inputs=True)
    b = PersistentStack(layers, K, dev, num_ctas=K * I // 64, keep_layer_inputs=True)
    for _ in range(4):
        x = np_to_bf16_tensor(np_bf16_normal(rng, (1, H)), dev)
        a.step_device(x)
        b.step_device(x)
        torch.cuda.synchronize()
        assert torch.equal(a.inds, b.inds)
        assert torch.equal(a.scores, b.scores)
        assert torch.equal(a.hs, b.hs)
    assert int(__import__("moe_offload_b200")._lib.call("moe_device_error", 1)) == 0


def test_persistent_stack_host_decode_graph(dev):
    """The host-facing decode (H2D, launch and D2H captured as one graph) returns the same bits
    as the device-side step, token after token."""
    from moe_offload_b200.stack import PersistentStack
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(41)
    L, H, I, E, K = 3, 2048, 768, 64, 8
    layers = _dev_layers(_np_layers(rng, L, E, H, I), dev)
    st = PersistentStack(layers, K, dev)
    out = torch.empty((1, H), dtype=torch.bfloat16, pin_memory=True)
    for _ in range(4):
        x = np_to_bf16_tensor(np_bf16_normal(rng, (1, H)), dev)
        y_dev = st.step_device(x).clone()
        inds_dev = st.inds.clone()
        torch.cuda.synchronize()
        st.decode(x.cpu().pin_memory(), out)
        assert torch.equal(out, y_dev.cpu())
        assert torch.equal(st.inds, inds_dev)
    assert st._decode_graph is not None or st._graph_failed


def test_persistent_stack_matches_layer_path(dev):
    """Same weights and input through the per-layer kernels: indices identical, outputs close."""
    from moe_offload_b200.stack import DecodeStack, PersistentStack
    from moe_offload_b200.synthetic import np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(9)
    L, H, I, E, K = 4, 3072, 768, 64, 10
    layers = _dev_layers(_np_layers(rng, L, E, H, I), dev)
    a = PersistentStack(layers, K, dev)
    b = DecodeStack(layers, K, dev, use_graph=False)
    for _ in range(3):
        x = np_to_bf16_tensor(np_bf16_normal(rng, (1, H)), dev)
        ya = a.step_device(x).clone()
        yb = b.step_device(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(a.inds, b.inds.view(L, K)), "per-layer routing differs"
        rel = (ya.float() - yb.float()).norm() / yb.float().norm()
        assert rel < REL_TOL


def test_layer_path_with_norm_vs_oracle(dev):
    """The three-kernel fused layer with the power-of-two input normalisation."""
    from moe_offload_b200 import ops
    from moe_offload_b200.ops import pow2_normalize
    from moe_offload_b200.synthetic import bf16_tensor_to_np, np_bf16_normal, np_to_bf16_tensor
    rng = np.random.default_rng(21)
    H, I, E, K = 3072, 768, 48, 10
    ly = _np_layers(rng, 1, E, H, I)[0]
    dl = _dev_layers([ly], dev)[0]
    h = np_bf16_normal(rng, (1, H), 37.0)        # far from unit RMS
    # no residual: the MoE output itself is compared (a large residual would hide it in bf16)
    out = ops.decode_layer(np_to_bf16_tensor(h, dev), dl.router, dl.gate, dl.up, dl.down, K, norm=True)
    torch.cuda.synchronize()
    x = pow2_normalize(h)
    _, ri, rs = orc.softmax_topk(orc.router_logits(x, ly["router"], E), K)
    assert np.array_equal(out["inds"].cpu().numpy().astype(np.uint32), ri)
    ref = orc.experts(x, ri, rs, ly["g"], ly["u"], ly["d"], sb_fp16=True)["y"]
    a = orc.bf16_to_f32(bf16_tensor_to_np(out["y"])).astype(np.float64)
    b = orc.bf16_to_f32(ref).astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < REL_TOL
