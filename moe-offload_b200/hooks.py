"""Per-layer decode hooks: the reference's install_offload_hooks / hooked_layer_call
(mlx-qwen38/loader.py:827-1001) over a MoE-only model.

The reference hooks every decoder layer of its MLX model so that a decode step runs, per
layer: hyper-connection mixer -> router (softmax, top-k, renormalised scores) -> shared
expert -> routed experts -> combine -> write, with the expert cache driven in a fixed order:

  layer 0 (pinned)    experts on the resident stack; then, with prefetch on, the written
                      state goes through layer 1's mixer and router, and layer 1's top-M
                      prediction starts its prefetch (loader.py:920-946)
  layers 1..L-1       with prefetch on (and a next layer), the next layer's mixer and router
                      on this layer's pre-MoE state give the top-M prediction; the LRU step of
                      this layer's routed experts (demand fills), the experts on their slots
                      and the combine; then the next layer's prefetch (loader.py:948-986)

Here the same order runs on the GPU with nothing read back to the host: the LRU step, the
fills and the prefetch are device work ordered on the streams (CachedSwitchGLU), where the
reference synchronises on the router's indices every layer. Attention and the rest of the
language model are outside this library, so a layer here is the MoE half of the reference's
decoder layer: an optional hyper-connection mixer (ops.hc_mix, kernels.cpp:1363-1560), the
router weight, the routed experts (a resident ExpertLayer or a CachedSwitchGLU) and an
optional shared expert (ops.shared_expert). Without a mixer the layer's state is one row of
H values, the block input is its per-row power-of-two normalisation (moe_pow2_rows, the
synthetic stack's stand-in for the pre-MoE norm) and the write is a residual add.

  MoEBlock(gate, switch_mlp, top_k, shared_expert=None)   the reference layer's `mlp`
  MoEDecoderLayer(mlp, mlp_hyper_connection=None)          one layer; __call__ = the plain path
  MoEModel(layers)                                          decode/prefill over the layers
  install_offload_hooks(model, prefetch_enabled, prefetch_top_m, prefetch_cap)
"""
from __future__ import annotations

import torch

from . import ops
from ._lib import call
from .offload import CachedSwitchGLU
from .ops import QMatrix

PREFETCH_TOP_M = 12       # loader.py:85
PREFETCH_MAX_CAP = 3      # loader.py:86


class SharedExpert:
    """The layer's shared expert: sigmoid(x . We) * down(SwiGLU(gate(x), up(x)))
    (engine.cpp:394-400, loader.py:909-910)."""

    def __init__(self, gate: QMatrix, up: QMatrix, down: QMatrix, expert_gate: QMatrix):
        self.gate, self.up, self.down, self.expert_gate = gate, up, down, expert_gate

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return ops.shared_expert(x, self.gate, self.up, self.down, self.expert_gate)


class HyperConnection:
    """The mixer in front of the MoE block (run_hc, kernels.cpp:1363-1560): called with the
    layer's state [T, hc*H] and an optional pending write (branch [T, H], gate [T, hc]), it
    returns (mixed [T, H], written state [T, hc*H], inject gate [T, hc])."""

    def __init__(self, norm_w: torch.Tensor, down: QMatrix, up: QMatrix, inject: QMatrix | None = None,
                 eps: float = 1e-6, hc: int = 4):
        self.norm_w, self.down, self.up, self.inject, self.eps, self.hc = norm_w, down, up, inject, eps, hc

    def __call__(self, h: torch.Tensor, write=None):
        return ops.hc_mix(h, self.norm_w, self.down, self.up, self.inject, write=write, eps=self.eps, hc=self.hc)


def hc_write(h: torch.Tensor, branch: torch.Tensor, gate: torch.Tensor, hc: int = 4) -> torch.Tensor:
    """_hc_write: stream c of h [T, hc*H] gets bf16(branch * gate[:, c]) added (one bf16
    rounding for the product, one for the sum), as the mixer's fused write does."""
    T = branch.shape[0]
    H = branch.shape[-1]
    add = (branch.float().view(T, 1, H) * gate.float().view(T, hc, 1)).to(torch.bfloat16)
    return (h.view(T, hc, H).float() + add.float()).to(torch.bfloat16).view(T, hc * H)


class MoEBlock:
    """The MoE module of one layer: router weight `gate` (bf16 [E, H] or an affine QMatrix),
    routed experts `switch_mlp` (ExpertLayer resident in HBM, or CachedSwitchGLU), top_k and
    an optional shared expert."""

    def __init__(self, gate, switch_mlp, top_k: int, shared_expert: SharedExpert | None = None):
        self.gate, self.switch_mlp, self.top_k, self.shared_expert = gate, switch_mlp, top_k, shared_expert
        self._r_out = {}      # decode output buffers, one set per prediction width M
        # the buffers of this layer's prediction made by the previous layer: the prefetch
        # stream reads them after this call returns, so nothing else may write them before
        # this layer's LRU step has waited for that prefetch
        self._pred_out = {}

    def route(self, x: torch.Tensor, *, w_next=None, M: int = 0) -> dict:
        """softmax(precise) -> argpartition top-k -> renormalised scores (loader.py:903-908);
        with w_next, also the sorted top-M of x . w_next (topk_sorted_indices, loader.py:237).
        Decode rows reuse the block's output buffers (valid until its next route call)."""
        out = self._r_out.setdefault(M, {}) if x.shape[0] == 1 else None
        return ops.router_topk(x, self.gate, self.top_k, w_next=w_next, M=M, out=out)

    def experts(self, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor,
                addend: torch.Tensor | None) -> torch.Tensor:
        """sum_k scores_k * expert_k(x) (+ addend), the MLX-order combine (loader.py:914,965)."""
        sw = self.switch_mlp
        T, K = inds.shape
        if T == 1:
            if isinstance(sw, CachedSwitchGLU):
                return sw.forward_combined(x, inds, scores, addend=addend)
            act = ops.experts_gateup(x, inds, sw.gate, sw.up)
            y, _ = ops.experts_down(act, inds, sw.down, scores, addend=addend)
            return y
        if not isinstance(sw, CachedSwitchGLU):     # resident: the expert-grouped prefill GEMMs
            y = ops.prefill_experts(x, inds, scores, sw.gate, sw.up, sw.down)
            return y if addend is None else (y.float() + addend.float()).to(torch.bfloat16)
        yk = sw.prefill(x, inds)
        y = torch.empty((T, x.shape[1]), dtype=torch.bfloat16, device=x.device)
        call("moe_combine_rows", yk.data_ptr(), T, K, x.shape[1], scores.data_ptr(),
             addend.data_ptr() if addend is not None else None, y.data_ptr(),
             torch.cuda.current_stream(x.device).cuda_stream)
        return y


class MoEDecoderLayer:
    """The MoE half of a decoder layer. __call__ follows the reference layer's signature
    (loader.py:855-866; the attention arguments are accepted and unused) and is the plain,
    un-hooked path: no prediction, no prefetch, a cached switch_mlp takes its LRU step."""

    is_linear = False

    def __init__(self, mlp: MoEBlock, mlp_hyper_connection: HyperConnection | None = None):
        self.mlp = mlp
        self.mlp_hyper_connection = mlp_hyper_connection

    def __contains__(self, name: str) -> bool:       # the reference tests `"ple" in self_layer`
        return getattr(self, name, None) is not None

    def __getitem__(self, name: str):
        return getattr(self, name)

    def mix(self, hidden_states: torch.Tensor, write=None):
        """(mixed, h_pre_moe, inject gate): the block input, the state the block's output is
        written into, and the write's stream gate (None without a mixer)."""
        hc = self.mlp_hyper_connection
        if hc is not None:
            return hc(hidden_states, write=write)
        h = hidden_states
        if write is not None:
            h = (h.float() + write[0].float()).to(torch.bfloat16)
        x = torch.empty_like(h)
        call("moe_pow2_rows", h.data_ptr(), h.shape[0], h.shape[1], x.data_ptr(),
             torch.cuda.current_stream(h.device).cuda_stream)
        return x, h, None

    def write(self, h_pre: torch.Tensor, branch: torch.Tensor, inj) -> torch.Tensor:
        if self.mlp_hyper_connection is not None:
            return hc_write(h_pre, branch, inj, self.mlp_hyper_connection.hc)
        return (h_pre.float() + branch.float()).to(torch.bfloat16)

    def __call__(self, hidden_states, input_ids=None, mask=None, cache=None, position_ids=None, gdn_sink=None,
                 target_verify: bool = False, write=None, defer_write: bool = False):
        mixed, h_pre, inj = self.mix(hidden_states, write)
        r = self.mlp.route(mixed)
        shared_y = self.mlp.shared_expert(mixed) if self.mlp.shared_expert is not None else None
        branch = self.mlp.experts(mixed, r["inds"], r["scores"], shared_y)
        if defer_write:
            return h_pre, branch, inj
        return self.write(h_pre, branch, inj)


class MoEModel:
    """Layers applied in order with each layer's write deferred into the next layer's mixer
    (the reference's `write=` / `defer_write` chaining); the last write is applied at the end."""

    def __init__(self, layers: list[MoEDecoderLayer]):
        self.layers = layers

    def __call__(self, hidden_states: torch.Tensor) -> torch.Tensor:
        h, write = hidden_states, None
        for layer in self.layers:
            h, branch, inj = layer(h, write=write, defer_write=True)
            write = (branch, inj)
        return self.layers[-1].write(h, *write)


def _predict(layer: MoEDecoderLayer, state: torch.Tensor, top_m: int) -> torch.Tensor:
    """The next layer's top-M prediction from a state: its mixer, then the sorted top-M of its
    router logits (loader.py:932-935, 953-956)."""
    m_next = layer.mix(state)[0]
    blk = layer.mlp
    out = blk._pred_out.setdefault(top_m, {})
    return ops.router_topk(m_next, blk.gate, blk.top_k, w_next=blk.gate, M=top_m, out=out)["pred"].view(-1)


def install_offload_hooks(model: MoEModel, prefetch_enabled: bool = True, prefetch_top_m: int = PREFETCH_TOP_M,
                          prefetch_cap: int = PREFETCH_MAX_CAP) -> None:
    """loader.py:827-1001: replaces each layer's __call__ (a per-layer subclass, as the
    reference does) by the offload decode order. Layer 0 must hold resident experts, layers
    1.. CachedSwitchGLU caches. Prefill rows (T > 1) take the plain path. The settings live on
    the model (model._prefetch_enabled / _prefetch_top_m / _prefetch_cap) and may be changed
    between calls."""
    layers = model.layers
    num_layers = len(layers)
    for il, layer in enumerate(layers):
        cached = isinstance(layer.mlp.switch_mlp, CachedSwitchGLU)
        if (il == 0) == cached:
            raise ValueError(f"layer {il}: layer 0 resident, later layers cached expected")
    model._prefetch_enabled = prefetch_enabled
    model._prefetch_top_m = prefetch_top_m
    model._prefetch_cap = prefetch_cap

    def make_layer_call(layer_idx: int):
        def hooked_layer_call(self_layer, hidden_states, input_ids=None, mask=None, cache=None, position_ids=None,
                              gdn_sink=None, target_verify: bool = False, write=None, defer_write: bool = False):
            moe_block = self_layer.mlp
            if hidden_states.shape[0] != 1:            # prefill: the plain path
                return MoEDecoderLayer.__call__(self_layer, hidden_states, write=write, defer_write=defer_write)
            mixed, h_pre, inj = self_layer.mix(hidden_states, write)
            prefetch = model._prefetch_enabled and layer_idx + 1 < num_layers
            top_m, cap = model._prefetch_top_m, model._prefetch_cap
            nxt = layers[layer_idx + 1] if prefetch else None
            # the next layer's prediction rides on this layer's router launch when both read
            # the same block input (no mixers); otherwise its own mixer + router
            fused_pred = (prefetch and layer_idx > 0 and self_layer.mlp_hyper_connection is None
                          and nxt.mlp_hyper_connection is None)
            r = moe_block.route(mixed, w_next=nxt.mlp.gate if fused_pred else None, M=top_m if fused_pred else 0)
            shared_y = moe_block.shared_expert(mixed) if moe_block.shared_expert is not None else None
            if layer_idx == 0:
                branch = moe_block.experts(mixed, r["inds"], r["scores"], shared_y)
                if prefetch:
                    h_post_0 = self_layer.write(h_pre, branch, inj)
                    pred = _predict(nxt, h_post_0, top_m)
                    nxt.mlp.switch_mlp.start_prefetch(pred, cap)
            else:
                pred = None
                if prefetch:
                    pred = r["pred"].view(-1) if fused_pred else _predict(nxt, h_pre, top_m)
                branch = moe_block.experts(mixed, r["inds"], r["scores"], shared_y)   # LRU step + experts
                if pred is not None:
                    nxt.mlp.switch_mlp.start_prefetch(pred, cap)
            if defer_write:
                return h_pre, branch, inj
            return self_layer.write(h_pre, branch, inj)

        return hooked_layer_call

    for il, layer in enumerate(layers):
        hooked_cls = type(f"OffloadMoEDecoderLayer_{il}", (type(layer),), {"__call__": make_layer_call(il)})
        layer.__class__ = hooked_cls
