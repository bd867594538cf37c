"""Expert shards in the reference's checkpoint layout (mlx-qwen38/loader.py:306-366, 1044-1060).

A model directory holds one `experts-XX.safetensors` per layer (XX = layer index, two digits).
Shard XX stores the layer's routed experts as nine stacked tensors
`language_model.model.layers.{XX}.mlp.switch_mlp.{gate,up,down}_proj.{weight,scales,biases}`:
`weight` U32 [E, rows, in * bits / 32] (MLX affine codes), `scales` / `biases` BF16 (or F16)
[E, rows, in / group_size]. The reference opens layers 1.. as caches that pread one expert's
row of every tensor at `8 + header_len + data_offsets[0] + eid * row_bytes`, and loads layer 0
whole (it stays resident).

Here a shard becomes:
  - `load_expert_pool`: the pinned host pool of a cached layer (`offload.HostExpertPool`),
    read with pread straight into pinned memory;
  - `load_expert_layer`: the device tensors of a resident layer (layer 0);
  - `shard_rows`: the nine (file offset, row bytes) pairs that the reference passes to
    `c_layer_init` / `P1IoScheduler::layer_init`, for `io_sched.P1IoScheduler.layer_init` and
    the file-backed fills.
`load_model_dir` puts a whole directory together for the offload engine: the routers from
`base-*.safetensors` (`language_model.model.layers.{XX}.mlp.gate.weight`, bf16 [E, H], or U32
codes with `.scales` / `.biases`: the affine-quantised router of the real model), layer 0
resident, layers 1.. as pinned pools, top-k from `config.json` (`num_experts_per_tok`).
`write_expert_shard` / `write_router_shard` write the same layout (tests; exporting a
synthetic stack)."""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

PROJS = ("gate_proj", "up_proj", "down_proj")
PARTS = ("weight", "scales", "biases")
NAME = "language_model.model.layers.{layer}.mlp.switch_mlp.{proj}.{part}"
ROUTER = "language_model.model.layers.{layer}.mlp.gate.{part}"

_DTYPES = {"U32": (torch.int32, 4), "BF16": (torch.bfloat16, 2), "F16": (torch.float16, 2)}


def shard_name(layer: int) -> str:
    return f"experts-{layer:02d}.safetensors"


@dataclass
class ShardTensor:
    name: str
    dtype: str
    shape: tuple
    offset: int          # absolute file offset of the tensor's first byte
    nbytes: int

    @property
    def row_bytes(self) -> int:
        return self.nbytes // self.shape[0]


def read_header(path) -> tuple[dict, int]:
    """The safetensors header (dict) and the file offset where the data section starts."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file")
        (n,) = struct.unpack("<Q", raw)
        hdr = json.loads(f.read(n))
    return hdr, 8 + n


def expert_tensors(path, layer: int, group_size: int = 64) -> list[ShardTensor]:
    """The nine expert tensors of `layer` in pool order (gate w/s/b, up w/s/b, down w/s/b),
    checked against each other: one expert count, codes U32, scales and biases of one float
    type, group counts that match the code widths."""
    hdr, start = read_header(path)
    out = []
    for proj in PROJS:
        for part in PARTS:
            name = NAME.format(layer=layer, proj=proj, part=part)
            if name not in hdr:
                raise KeyError(f"{path}: tensor {name} missing")
            info = hdr[name]
            b0, b1 = info["data_offsets"]
            t = ShardTensor(name, info["dtype"], tuple(info["shape"]), start + b0, b1 - b0)
            if len(t.shape) != 3 or t.dtype not in _DTYPES:
                raise ValueError(f"{name}: dtype {t.dtype} shape {t.shape} unsupported")
            if t.nbytes != int(np.prod(t.shape)) * _DTYPES[t.dtype][1]:
                raise ValueError(f"{name}: {t.nbytes} bytes for shape {t.shape}")
            out.append(t)
    E = out[0].shape[0]
    sb = out[1].dtype
    for i, t in enumerate(out):
        if t.shape[0] != E:
            raise ValueError(f"{t.name}: {t.shape[0]} experts, {E} expected")
        want = "U32" if i % 3 == 0 else sb
        if t.dtype != want or (i % 3 and sb not in ("BF16", "F16")):
            raise ValueError(f"{t.name}: dtype {t.dtype}, {want} expected")
    for p in range(3):
        w, s, b = out[3 * p: 3 * p + 3]
        if s.shape != b.shape or s.shape[:2] != w.shape[:2]:
            raise ValueError(f"{w.name}: scales/biases shape {s.shape} / {b.shape} vs codes {w.shape}")
        in_dim = s.shape[2] * group_size
        if (w.shape[2] * 32) % in_dim:
            raise ValueError(f"{w.name}: {w.shape[2]} words for {in_dim} inputs")
    return out


def shard_rows(path, layer: int, group_size: int = 64) -> tuple[list[int], list[int]]:
    """(file offsets, row bytes) of the nine tensors: expert e's row of tensor t is
    row_bytes[t] bytes at offsets[t] + e * row_bytes[t]."""
    ts = expert_tensors(path, layer, group_size)
    return [t.offset for t in ts], [t.row_bytes for t in ts]


def quant_params(path, layer: int, group_size: int = 64) -> dict:
    """bits, group size, experts, the layer's inter (I) and hidden (H) sizes, scale dtype."""
    ts = expert_tensors(path, layer, group_size)
    g, d = ts[0], ts[6]
    in_h = ts[1].shape[2] * group_size
    bits = g.shape[2] * 32 // in_h
    return {"bits": bits, "group_size": group_size, "experts": g.shape[0], "inter": g.shape[1], "hidden": in_h,
            "down_rows": d.shape[1], "sb_dtype": ts[1].dtype}


def _pread_into(fd: int, dst: torch.Tensor, offset: int, chunk: int = 64 << 20) -> None:
    view = dst.view(torch.uint8).reshape(-1).numpy()
    done, n = 0, view.nbytes
    while done < n:
        got = os.preadv(fd, [memoryview(view[done:min(n, done + chunk)])], offset + done)
        if got <= 0:
            raise IOError(f"short read at offset {offset + done}")
        done += got


def load_expert_tensors(path, layer: int, group_size: int = 64, pin: bool = True) -> list[torch.Tensor]:
    """The nine tensors as host tensors (pinned by default): codes int32 (the U32 bits),
    scales/biases bfloat16 or float16, in pool order."""
    ts = expert_tensors(path, layer, group_size)
    fd = os.open(path, os.O_RDONLY)
    try:
        out = []
        for t in ts:
            dt, _ = _DTYPES[t.dtype]
            h = torch.empty(t.shape, dtype=dt, pin_memory=pin)
            _pread_into(fd, h, t.offset)
            out.append(h)
        return out
    finally:
        os.close(fd)


def load_expert_pool(path, layer: int, group_size: int = 64):
    """A cached layer's pinned host pool (offload.HostExpertPool) from its shard."""
    from .offload import HostExpertPool
    q = quant_params(path, layer, group_size)
    return HostExpertPool(load_expert_tensors(path, layer, group_size), q["bits"], group_size)


def load_expert_layer(path, layer: int, router: torch.Tensor, device, group_size: int = 64):
    """A resident layer (ExpertLayer: router + three device QMatrix stacks) from its shard."""
    from .ops import QMatrix
    from .synthetic import ExpertLayer
    q = quant_params(path, layer, group_size)
    ts = [t.to(device) for t in load_expert_tensors(path, layer, group_size, pin=False)]
    mats = [QMatrix(ts[3 * p], ts[3 * p + 1], ts[3 * p + 2], q["bits"], group_size) for p in range(3)]
    return ExpertLayer(router.to(device), *mats)


def write_expert_shard(path, layer: int, mats: Sequence) -> None:
    """Writes one layer's experts (three (codes, scales, biases) triples or QMatrix: gate, up,
    down) in the shard layout above. Codes: int32 / uint32 (the U32 bits); scales/biases:
    bfloat16 or float16."""
    tensors = {}
    for proj, m in zip(PROJS, mats):
        w, s, b = (m.w, m.s, m.b) if hasattr(m, "w") else m
        for part, t in zip(PARTS, (w, s, b)):
            tensors[NAME.format(layer=layer, proj=proj, part=part)] = t
    _write_safetensors(path, tensors)


def _tensor_bytes(t: torch.Tensor) -> tuple[str, bytes]:
    t = torch.as_tensor(t).detach().cpu().contiguous()
    if t.dtype in (torch.int32, torch.uint32):
        return "U32", t.view(torch.int32).numpy().tobytes()
    if t.dtype == torch.bfloat16:
        return "BF16", t.view(torch.int16).numpy().tobytes()
    if t.dtype == torch.float16:
        return "F16", t.view(torch.int16).numpy().tobytes()
    raise TypeError(f"dtype {t.dtype} not supported")


def _write_safetensors(path, tensors: dict) -> None:
    hdr, blobs, off = {}, [], 0
    for name in sorted(tensors):
        dt, raw = _tensor_bytes(tensors[name])
        hdr[name] = {"dtype": dt, "shape": list(torch.as_tensor(tensors[name]).shape),
                     "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(hdr, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in blobs:
            f.write(raw)


def write_router_shard(path, routers: dict) -> None:
    """Writes routers {layer: bf16 [E, H] tensor, or a (codes, scales, biases) triple / QMatrix}
    with the reference's names (a base-*.safetensors shard holding only the routers)."""
    tensors = {}
    for layer, r in routers.items():
        if isinstance(r, torch.Tensor):
            tensors[ROUTER.format(layer=layer, part="weight")] = r
        else:
            w, s, b = (r.w, r.s, r.b) if hasattr(r, "w") else r
            for part, t in zip(PARTS, (w, s, b)):
                tensors[ROUTER.format(layer=layer, part=part)] = t
    _write_safetensors(path, tensors)


def _read_tensor(path, info, start) -> torch.Tensor:
    dt, _ = _DTYPES[info["dtype"]]
    t = torch.empty(tuple(info["shape"]), dtype=dt)
    fd = os.open(path, os.O_RDONLY)
    try:
        _pread_into(fd, t, start + info["data_offsets"][0])
    finally:
        os.close(fd)
    return t


def load_router(model_dir, layer: int, group_size: int = 64):
    """Layer `layer`'s router from the directory's base-*.safetensors: a bf16 [E, H] tensor, or
    an ops.QMatrix (affine codes + scales + biases). Host memory."""
    from pathlib import Path

    from .ops import QMatrix
    for f in sorted(Path(model_dir).glob("base-*.safetensors")):
        hdr, start = read_header(f)
        wname = ROUTER.format(layer=layer, part="weight")
        if wname not in hdr:
            continue
        w = _read_tensor(f, hdr[wname], start)
        if w.dtype == torch.bfloat16:
            return w
        s = _read_tensor(f, hdr[ROUTER.format(layer=layer, part="scales")], start)
        b = _read_tensor(f, hdr[ROUTER.format(layer=layer, part="biases")], start)
        bits = w.shape[1] * 32 // (s.shape[1] * group_size)
        return QMatrix(w, s, b, bits, group_size)
    raise KeyError(f"{model_dir}: no base-*.safetensors holds layer {layer}'s router")


def _router_to(r, device):
    from .ops import QMatrix
    if isinstance(r, torch.Tensor):
        return r.to(device)
    return QMatrix(r.w.to(device), r.s.to(device), r.b.to(device), r.bits, r.group_size)


def load_model_dir(model_dir, device, top_k: int | None = None, group_size: int = 64) -> dict:
    """Everything the offload engine needs from a model directory in the reference's layout:
    {"config": synthetic.StackConfig of the shapes, "routers": [device routers], "layer0":
    resident ExpertLayer, "pools": [HostExpertPool for layers 1..]}."""
    from pathlib import Path

    from .synthetic import StackConfig
    d = Path(model_dir)
    L = 0
    while (d / shard_name(L)).exists():
        L += 1
    if L == 0:
        raise FileNotFoundError(f"{d}: no {shard_name(0)}")
    q = quant_params(d / shard_name(0), 0, group_size)
    if top_k is None:
        cfg = json.loads((d / "config.json").read_text()) if (d / "config.json").exists() else {}
        top_k = cfg.get("num_experts_per_tok", cfg.get("text_config", {}).get("num_experts_per_tok"))
        if top_k is None:
            raise ValueError(f"{d}: top_k not given and config.json has no num_experts_per_tok")
    conf = StackConfig(name=f"checkpoint:{d.name}", layers=L, hidden=q["hidden"], experts=q["experts"],
                       top_k=int(top_k), inter=q["inter"], group_size=group_size, bits=q["bits"])
    routers = [_router_to(load_router(d, l, group_size), device) for l in range(L)]
    layer0 = load_expert_layer(d / shard_name(0), 0, torch.empty(0), device, group_size)
    layer0.router = routers[0]
    pools = [load_expert_pool(d / shard_name(l), l, group_size) for l in range(1, L)]
    return {"config": conf, "routers": routers, "layer0": layer0, "pools": pools}
