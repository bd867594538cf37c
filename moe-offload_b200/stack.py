"""Resident decode stack: L MoE layers, every expert resident in HBM, batch-1 decode.

`DecodeStack.step_device` runs one token through all layers (h_{l+1} = h_l + MoE_l(h_l))
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
                 predict_top_m: int = 0):
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
                             M=self.M if nxt is not None else 0, resid=y, out=out, workspace=self.ws)
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
