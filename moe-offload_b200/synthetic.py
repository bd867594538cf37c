"""Seeded synthetic inputs with the shapes and value distributions of the benchmark
configurations (the reference's real checkpoints and prompts are not available here):

  expert codes   uniform in {0..3} (every packed uint32 word uniform)
  scales         fp16 N(0.02, 0.005) clamped > 0
  biases         fp16 N(0, 0.01)
  router         bf16 N(0, 0.02) [E, H]
  hidden states  bf16 N(0, 1)

Two generators: numpy (CPU, small sizes, for the oracle tests) and torch on the device
(full BASELINE sizes, tens of GB, generated in place on the GPU).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .ops import QMatrix


@dataclass(frozen=True)
class StackConfig:
    """One benchmark configuration of the routed-expert stack."""

    name: str
    layers: int
    hidden: int          # H
    experts: int         # E
    top_k: int           # K
    inter: int           # I
    group_size: int = 64
    bits: int = 2
    seed: int = 0

    @property
    def expert_bytes(self) -> int:
        """HBM bytes of one routed expert (codes + fp16 scales + biases, gate+up+down)."""
        H, I, gs = self.hidden, self.inter, self.group_size
        codes = 3 * H * I * self.bits // 8
        sb = 2 * 2 * (2 * I * (H // gs) + H * (I // gs))
        return codes + sb

    @property
    def router_bytes(self) -> int:
        return self.experts * self.hidden * 2


# BASELINE.json configs
C0 = StackConfig("c0_single_layer_h2048_e64_top8", 1, 2048, 64, 8, 768, seed=0)
C1 = StackConfig("c1_qwen38_shape_28x512_top10", 28, 3072, 512, 10, 768, seed=1)
C2 = StackConfig("c2_offload_28x512_top10_cap102", 28, 3072, 512, 10, 768, seed=2)
C3 = StackConfig("c3_prefill_28x512_top10_T2048", 28, 3072, 512, 10, 768, seed=3)
C3_TOKENS = 2048
NEMOTRON = StackConfig("c3_nemotron_shape_240_top9", 1, 2688, 240, 9, 1856, seed=3)
NEMOTRON_TOKENS = 1024
C4 = StackConfig("c4_expert_parallel_28x512_top10", 28, 3072, 512, 10, 768, seed=4)


# ------------------------------------------------------------------------------ numpy

def np_qmatrix(rng: np.random.Generator, n: int, rows: int, cols: int, bits: int = 2, gs: int = 64,
               sb_fp16: bool = True):
    """(codes uint32 [n, rows, cols*bits/32], scales u16 bits, biases u16 bits)."""
    words = cols * bits // 32
    w = rng.integers(0, 2**32, size=(n, rows, words), dtype=np.uint64).astype(np.uint32)
    ng = cols // gs
    s = np.clip(rng.normal(0.02, 0.005, size=(n, rows, ng)), 1e-4, None)
    b = rng.normal(0.0, 0.01, size=(n, rows, ng))
    if sb_fp16:
        s16 = s.astype(np.float16).view(np.uint16)
        b16 = b.astype(np.float16).view(np.uint16)
    else:
        s16 = _np_bf16(s)
        b16 = _np_bf16(b)
    return w, s16, b16


def _np_bf16(a) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def np_bf16_normal(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return _np_bf16(rng.normal(0.0, std, size=shape))


def to_device_qmatrix(t, device, bits: int = 2, gs: int = 64, sb_fp16: bool = True) -> QMatrix:
    w, s, b = t
    sbd = torch.float16 if sb_fp16 else torch.bfloat16
    return QMatrix(torch.from_numpy(w.view(np.int32)).to(device),
                   torch.from_numpy(s.view(np.int16)).to(device).view(sbd),
                   torch.from_numpy(b.view(np.int16)).to(device).view(sbd), bits, gs)


def np_to_bf16_tensor(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).to(device).view(torch.bfloat16)


def bf16_tensor_to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


# ------------------------------------------------------------------------------ torch (device)

def dev_qmatrix(n: int, rows: int, cols: int, device, gen: torch.Generator, bits: int = 2,
                gs: int = 64) -> QMatrix:
    """Full-size synthetic stack generated on the device (fp16 scales/biases)."""
    words = cols * bits // 32
    w = torch.randint(-(2**31), 2**31, (n, rows, words), dtype=torch.int32, device=device, generator=gen)
    ng = cols // gs
    s = torch.empty((n, rows, ng), dtype=torch.float32, device=device).normal_(0.02, 0.005, generator=gen)
    s = s.clamp_(min=1e-4).to(torch.float16)
    b = torch.empty((n, rows, ng), dtype=torch.float32, device=device).normal_(0.0, 0.01, generator=gen)
    return QMatrix(w, s, b.to(torch.float16), bits, gs)


def dev_bf16_normal(shape, device, gen: torch.Generator, std: float = 1.0) -> torch.Tensor:
    return torch.empty(shape, dtype=torch.float32, device=device).normal_(0.0, std, generator=gen).to(torch.bfloat16)


@dataclass
class ExpertLayer:
    """One layer's resident weights: router [E, H] bf16 and the three expert stacks."""

    router: torch.Tensor
    gate: QMatrix
    up: QMatrix
    down: QMatrix


def dev_stack(cfg: StackConfig, device, layers: int | None = None) -> list[ExpertLayer]:
    gen = torch.Generator(device=device)
    gen.manual_seed(cfg.seed)
    out = []
    for _ in range(cfg.layers if layers is None else layers):
        router = dev_bf16_normal((cfg.experts, cfg.hidden), device, gen, 0.02)
        gate = dev_qmatrix(cfg.experts, cfg.inter, cfg.hidden, device, gen, cfg.bits, cfg.group_size)
        up = dev_qmatrix(cfg.experts, cfg.inter, cfg.hidden, device, gen, cfg.bits, cfg.group_size)
        down = dev_qmatrix(cfg.experts, cfg.hidden, cfg.inter, device, gen, cfg.bits, cfg.group_size)
        out.append(ExpertLayer(router, gate, up, down))
    return out


def dev_stack_shard(cfg: StackConfig, device, first: int, count: int, layers: int | None = None) -> list[ExpertLayer]:
    """An expert-parallel rank's part of a synthetic stack: every layer's whole router (the
    same on every rank: one generator seeded with cfg.seed) and experts [first, first + count)
    (a generator seeded with the seed and the block's first expert)."""
    gr = torch.Generator(device=device)
    gr.manual_seed(cfg.seed)
    ge = torch.Generator(device=device)
    ge.manual_seed(cfg.seed * 1_000_003 + first)
    out = []
    for _ in range(cfg.layers if layers is None else layers):
        router = dev_bf16_normal((cfg.experts, cfg.hidden), device, gr, 0.02)
        gate = dev_qmatrix(count, cfg.inter, cfg.hidden, device, ge, cfg.bits, cfg.group_size)
        up = dev_qmatrix(count, cfg.inter, cfg.hidden, device, ge, cfg.bits, cfg.group_size)
        down = dev_qmatrix(count, cfg.hidden, cfg.inter, device, ge, cfg.bits, cfg.group_size)
        out.append(ExpertLayer(router, gate, up, down))
    return out
