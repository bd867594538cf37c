"""Resident decode stack: L MoE layers, every expert resident in HBM, batch-1 decode.

Each layer computes h_{l+1} = h_l + MoE_l(x_l) with x_l = h_l * 2^-k_l, the power of two
nearest h_l's RMS (norm=True; the model's pre-MoE RMSNorm, kept exact by using a power of
two). Without it the residual stream of a random-weight stack grows without bound.

`DecodeStack.step_device` runs one token through all layers
as one CUDA-graph replay of 3*L PDL-chained kernels; `DecodeStack.decode` is the host-facing
call (pinned host hidden state in, host result out) a user of the library makes.
This is the stack the reference's OffloadEngine decode loop drives when every layer is
resident (mlx-qwen38/loader.py:1176-1195 around the hooked layers, 903-922 per layer).
"""
from __future__ import annotations

import torch

from . import ops
from .synthetic import ExpertLayer


class DecodeStack:
    def __init__(self, layers: list[ExpertLayer], top_k: int, device, use_graph: bool = True,
                 predict_top_m: int = 0, norm: bool = True):
        self.norm = norm
        self.layers = layers
        self.K = top_k
        self.M = predict_top_m
        self.device = torch.device(device)
        self.H = layers[0].router.shape[1]
        self.E = layers[0].router.shape[0]
        self.I = layers[0].gate.w.shape[1]
        L = len(layers)
        self.x_in = torch.zeros((1, self.H), dtype=torch.bfloat16, device=self.device)
        self.ys = [torch.empty((1, self.H), dtype=torch.bfloat16, device=self.device) for _ in range(L)]
        self.inds = torch.empty((L, 1, top_k), dtype=torch.int32, device=self.device)
        self.scores = torch.empty((L, 1, top_k), dtype=torch.bfloat16, device=self.device)
        self.preds = torch.empty((L, 1, max(predict_top_m, 1)), dtype=torch.int32, device=self.device)
        self.ws = ops.decode_workspace(self.device, 1, self.H, self.I, self.E, top_k, predict_top_m)
        self.stream = torch.cuda.Stream(device=self.device)
        self.graph = None
        self.launches_per_step = 3 * L
        if use_graph:
            self._capture()

    def _layers_once(self) -> torch.Tensor:
        y = self.x_in
        L = len(self.layers)
        for li, ly in enumerate(self.layers):
            nxt = self.layers[li + 1].router if (self.M > 0 and li + 1 < L) else None
            out = {"y": self.ys[li], "inds": self.inds[li], "scores": self.scores[li]}
            if nxt is not None:
                out["pred"] = self.preds[li]
            ops.decode_layer(y, ly.router, ly.gate, ly.up, ly.down, self.K, router_next=nxt,
                             M=self.M if nxt is not None else 0, resid=y, norm=self.norm, out=out,
                             workspace=self.ws)
            y = self.ys[li]
        return y

    def _capture(self) -> None:
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self._layers_once()           # warm: sets kernel attributes, loads the module
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self._layers_once()
        self.graph = g

    def step_device(self, x: torch.Tensor | None = None) -> torch.Tensor:
        """One token through all layers on the current stream; x (bf16 [1,H], device) is
        copied into the stack's input buffer when given. Returns the last layer's output."""
        if x is not None:
            self.x_in.copy_(x)
        if self.graph is not None:
            self.graph.replay()          # launches on the current stream
        else:
            self._layers_once()
        return self.ys[-1]

    def decode(self, h_host: torch.Tensor, out_host: torch.Tensor | None = None) -> torch.Tensor:
        """Host-facing decode step: pinned host hidden state [1,H] bf16 in, host result out."""
        cur = torch.cuda.current_stream(self.device)
        self.x_in.copy_(h_host, non_blocking=True)
        y = self.step_device()
        if out_host is None:
            out_host = torch.empty((1, self.H), dtype=torch.bfloat16, pin_memory=True)
        out_host.copy_(y, non_blocking=True)
        cur.synchronize()
        return out_host


def pack_layer_experts(layer: ExpertLayer, device) -> torch.Tensor:
    """The layer's E experts in the packed layout of moe_pack_experts ([E, expert_bytes] u8)."""
    from ._lib import call

    E, H = layer.router.shape
    I = layer.gate.w.shape[1]
    nbytes = int(call("moe_packed_expert_bytes", H, I))
    out = torch.empty((E, nbytes), dtype=torch.uint8, device=device)
    g, u, d = layer.gate, layer.up, layer.down
    call("moe_pack_experts", E, H, I, g.w.data_ptr(), g.s.data_ptr(), g.b.data_ptr(), u.w.data_ptr(),
         u.s.data_ptr(), u.b.data_ptr(), d.w.data_ptr(), d.s.data_ptr(), d.b.data_ptr(), out.data_ptr(),
         torch.cuda.current_stream(device).cuda_stream)
    return out


class PersistentStack:
    """The same resident stack as DecodeStack, run by the persistent kernel: one cooperative
    launch per token with all layers inside (moe_stack_decode). The experts are repacked once
    at construction (pack_layer_experts); with release_unpacked the MLX-layout tensors of
    `layers` are dropped afterwards (their memory is freed when the caller holds no other
    reference)."""

    def __init__(self, layers: list[ExpertLayer], top_k: int, device, num_ctas: int = 0,
                 keep_layer_inputs: bool = False, norm: bool = True, release_unpacked: bool = False):
        from ._lib import call

        self.norm = norm
        self._call = call
        self.K = top_k
        self.device = torch.device(device)
        self.L = len(layers)
        if not all(isinstance(ly.router, torch.Tensor) and ly.router.dtype == torch.bfloat16 for ly in layers):
            raise ValueError("the persistent stack reads bf16 [E, H] routers; route affine ones per layer")
        self.E, self.H = layers[0].router.shape
        self.I = layers[0].gate.w.shape[1]
        self.sb_fp16 = layers[0].gate.sb_fp16
        self.num_ctas = num_ctas
        # transposed routers ([H][E]), packed experts and the device array of layer descriptors
        self.router_t = [ly.router.t().contiguous() for ly in layers]
        self.packed = []
        for i in range(self.L):
            self.packed.append(pack_layer_experts(layers[i], self.device))
            if release_unpacked:
                torch.cuda.current_stream(self.device).synchronize()
                layers[i] = None
        self.layers = None if release_unpacked else layers
        desc = [[rt.data_ptr(), pk.data_ptr()] for rt, pk in zip(self.router_t, self.packed)]
        self.desc = torch.tensor(desc, dtype=torch.int64).to(self.device)
        nbytes = int(call("moe_stack_workspace_bytes", self.H, self.I, self.E, self.K))
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self.x_in = torch.zeros((1, self.H), dtype=torch.bfloat16, device=self.device)
        self.y = torch.empty((1, self.H), dtype=torch.bfloat16, device=self.device)
        self.inds = torch.empty((self.L, top_k), dtype=torch.int32, device=self.device)
        self.scores = torch.empty((self.L, top_k), dtype=torch.bfloat16, device=self.device)
        self.hs = (torch.empty((self.L + 1, self.H), dtype=torch.bfloat16, device=self.device)
                   if keep_layer_inputs else None)
        self.launches_per_step = 1
        self._decode_graph = None        # host-facing step as one CUDA graph (decode)
        self._graph_failed = False

    def step_device(self, x: torch.Tensor | None = None) -> torch.Tensor:
        if x is not None:
            self.x_in.copy_(x)
        self._call("moe_stack_decode", self.desc.data_ptr(), self.L, self.H, self.I, self.E, self.K,
                   self.sb_fp16, int(self.norm), self.x_in.data_ptr(), self.y.data_ptr(), self.inds.data_ptr(),
                   self.scores.data_ptr(), None if self.hs is None else self.hs.data_ptr(), self.ws.data_ptr(),
                   self.ws.numel(), self.num_ctas, torch.cuda.current_stream(self.device).cuda_stream)
        return self.y

    def _capture_decode(self) -> None:
        """Records the host-facing step (H2D copy from a fixed pinned buffer, workspace reset +
        persistent launch, D2H copy into a fixed pinned buffer) as one CUDA graph, so a token
        costs one graph launch instead of four host-issued operations."""
        self._h_pin = torch.zeros((1, self.H), dtype=torch.bfloat16, pin_memory=True)
        self._o_pin = torch.empty((1, self.H), dtype=torch.bfloat16, pin_memory=True)
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        try:
            with torch.cuda.stream(s):
                self.x_in.copy_(self._h_pin, non_blocking=True)      # warm-up outside the graph
                self.step_device()
                self._o_pin.copy_(self.y, non_blocking=True)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.x_in.copy_(self._h_pin, non_blocking=True)
                self.step_device()
                self._o_pin.copy_(self.y, non_blocking=True)
            self._decode_graph = g
        except RuntimeError:
            # a driver that cannot capture a cooperative launch: keep the direct path
            self._graph_failed = True
            torch.cuda.synchronize(self.device)
        torch.cuda.current_stream(self.device).wait_stream(s)

    def decode(self, h_host: torch.Tensor, out_host: torch.Tensor | None = None) -> torch.Tensor:
        """Host-facing decode step: host hidden state [1,H] bf16 in, host result out (the
        result also stays in self.y). Runs the captured graph when available."""
        cur = torch.cuda.current_stream(self.device)
        if self._decode_graph is None and not self._graph_failed:
            self._capture_decode()
        if out_host is None:
            out_host = torch.empty((1, self.H), dtype=torch.bfloat16, pin_memory=True)
        if self._decode_graph is not None:
            self._h_pin.copy_(h_host)
            self._decode_graph.replay()
            cur.synchronize()
            out_host.copy_(self._o_pin)
            return out_host
        self.x_in.copy_(h_host, non_blocking=True)
        y = self.step_device()
        out_host.copy_(y, non_blocking=True)
        cur.synchronize()
        return out_host
