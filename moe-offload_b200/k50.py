"""The reference's K50 expert pack (mlx-qwen38/cpp/src/loader.cpp:1187-1470, cpp/README.md:63-86):
one directory per layer (L00 .. L47) with codes.bin, scales.bf16, bias.bf16 and index.json,
expert records per projection of kind "tern" (base-3, five digits per byte), "2t" (the same
ternary values as MLX 2-bit codes with bias = -scale), "2", "3", "4", "6" or "8" (MLX affine
codes), plus dense records.

  K50Pack(layer_dir)            the parsed index (moe_k50_open, C++): record(), materialize()
  load_k50_pool(layer_dir, E)   a cached layer's pinned host pool (offload.HostExpertPool) of
                                experts 0..E-1, each expert materialised straight into its
                                pinned rows
  write_k50_layer(...)          writes a layer directory in the same format (for converted or
                                synthetic weights; the tests' fixtures)

The expert kernels run 2-bit codes, so a pool takes layers whose expert records are all of a
2-bit kind (tern, 2t, 2); a layer holding 3/4/6/8-bit experts is read and materialised
(K50Pack) but load_k50_pool refuses it with the kinds it found.
"""
from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import torch

from ._lib import MoeError, call, load

PROJS = ("gate_proj", "up_proj", "down_proj")
KINDS = ("tern", "2t", "2", "3", "4", "6", "8")
UNITS = ("hot", "warm", "mid", "cold", "dense")


def layer_dir(model_dir, layer: int) -> Path:
    return Path(model_dir) / f"L{layer:02d}"


class K50Pack:
    """One layer directory, parsed by the library (moe_k50_open)."""

    def __init__(self, layer_dir_path):
        self.path = Path(layer_dir_path)
        lib = load()
        self.h = lib.moe_k50_open(str(self.path).encode())
        if not self.h:
            raise MoeError("moe_k50_open", -22, (lib.moe_last_error() or b"").decode(errors="replace"))

    def close(self) -> None:
        if self.h:
            load().moe_k50_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def count(self, proj: str) -> int:
        return int(call("moe_k50_count", self.h, proj.encode()))

    def dense_names(self) -> list[str]:
        out = []
        buf = ctypes.create_string_buffer(512)
        for i in range(self.count("dense")):
            call("moe_k50_dense_name", self.h, i, buf, len(buf))
            out.append(buf.value.decode())
        return out

    def record(self, proj: str, expert: int = -1) -> dict:
        """Geometry of a record's materialised form; expert < 0: the dense record `proj`."""
        o = (ctypes.c_int64 * 8)()
        call("moe_k50_record", self.h, proj.encode(), int(expert), o)
        return {"bits": o[0], "group_size": o[1], "rows": o[2], "cols": o[3], "words": o[4], "groups": o[5],
                "kind": KINDS[o[6]] if 0 <= o[6] < len(KINDS) else None,
                "unit": UNITS[o[7]] if 0 <= o[7] < len(UNITS) else None}

    def materialize(self, proj: str, expert: int = -1):
        """(codes uint32 [rows, words], scales bf16 bits uint16 [rows, groups], biases idem)."""
        r = self.record(proj, expert)
        w = np.empty((r["rows"], r["words"]), dtype=np.uint32)
        s = np.empty((r["rows"], r["groups"]), dtype=np.uint16)
        b = np.empty_like(s)
        call("moe_k50_materialize", self.h, proj.encode(), int(expert), w.ctypes.data, s.ctypes.data, b.ctypes.data)
        return w, s, b


def load_k50_pool(path, num_experts: int):
    """Experts 0..num_experts-1 of a layer directory as a pinned HostExpertPool (MLX layout,
    bf16 scales and biases), materialised by the library into the pinned rows."""
    from .offload import HostExpertPool
    with K50Pack(path) as pk:
        recs = {p: [pk.record(p, e) for e in range(num_experts)] for p in PROJS}
        kinds = sorted({r["kind"] for p in PROJS for r in recs[p]})
        bits = {r["bits"] for p in PROJS for r in recs[p]}
        gss = {r["group_size"] for p in PROJS for r in recs[p]}
        if bits != {2} or len(gss) != 1:
            raise ValueError(f"{path}: expert kinds {kinds} (group sizes {sorted(gss)}): the expert kernels run "
                             "2-bit codes of one group size (kinds tern, 2t, 2)")
        tensors = []
        for p in PROJS:
            shapes = {(r["rows"], r["words"], r["groups"]) for r in recs[p]}
            if len(shapes) != 1:
                raise ValueError(f"{path}: {p} records of different shapes {sorted(shapes)}")
            rows, words, groups = shapes.pop()
            w = torch.empty((num_experts, rows, words), dtype=torch.int32, pin_memory=True)
            s = torch.empty((num_experts, rows, groups), dtype=torch.bfloat16, pin_memory=True)
            b = torch.empty((num_experts, rows, groups), dtype=torch.bfloat16, pin_memory=True)
            for e in range(num_experts):
                call("moe_k50_materialize", pk.h, p.encode(), e, w[e].data_ptr(), s[e].data_ptr(), b[e].data_ptr())
            tensors += [w, s, b]
        return HostExpertPool(tensors, 2, gss.pop())


# ------------------------------------------------------------------------------- writing

def ternary_to_base3(digits: np.ndarray) -> np.ndarray:
    """[rows, cols] digits in {0, 1, 2} -> [rows, cols / 5] bytes, five digits per byte, the
    first digit least significant (the layout the reader unpacks)."""
    d = np.asarray(digits, dtype=np.uint16)
    rows, cols = d.shape
    if cols % 5 or d.max(initial=0) > 2:
        raise ValueError("ternary digits: cols must be a multiple of 5 and digits in {0, 1, 2}")
    g = d.reshape(rows, cols // 5, 5)
    return (g * np.array([1, 3, 9, 27, 81], dtype=np.uint16)).sum(axis=-1).astype(np.uint8)


def codes_to_digits(codes: np.ndarray, cols: int) -> np.ndarray:
    """MLX 2-bit codes [rows, cols / 16] -> [rows, cols] values 0..3."""
    c = np.asarray(codes, dtype=np.uint32)
    shifts = (np.arange(16, dtype=np.uint32) * 2)[None, None, :]
    return ((c[:, :, None] >> shifts) & 3).reshape(c.shape[0], cols).astype(np.uint8)


def write_k50_layer(path, experts: dict, dense: dict | None = None, group_size: int = 64) -> None:
    """Writes a layer directory. experts: {proj: [rec, ...]} with rec a dict of kind ("tern",
    "2t", "2", "3", "4", "6", "8"), unit ("hot", ...), shape (rows, cols), scales (uint16 bf16
    bits [rows, cols / group_size]) and either codes (uint32 MLX words [rows, words]) with
    biases (uint16 bf16 bits, omitted for bias = -scale), or, for "tern", digits (uint8 values
    0..2 [rows, cols]); the record's position in the list is its expert id. dense: {name: rec}
    in the same form."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    code_f, scale_f, bias_f = bytearray(), bytearray(), bytearray()
    index: dict = {"version": "k50-synthetic", "experts": {}, "dense": {}}

    def put(rec, expert):
        rows, cols = (int(v) for v in rec["shape"])
        kind = rec["kind"]
        gs = int(rec.get("group_size", group_size))
        sc = np.ascontiguousarray(rec["scales"], dtype=np.uint16)
        if sc.shape != (rows, cols // gs):
            raise ValueError(f"scales of shape {sc.shape}, expected {(rows, cols // gs)}")
        out = {"kind": kind, "unit": rec.get("unit", "cold"), "shape": [rows, cols], "group_size": gs}
        if expert is not None:
            out["expert"] = expert
        if kind == "tern":
            raw = ternary_to_base3(rec["digits"])
            out["row_bytes"] = cols // 5
            bias = b""
        else:
            raw = np.ascontiguousarray(rec["codes"], dtype=np.uint32)
            out["row_bytes"] = raw.shape[1] * 4
            bias = b"" if rec.get("biases") is None else np.ascontiguousarray(rec["biases"], dtype=np.uint16).tobytes()
        out.update(code_off=len(code_f), code_nbytes=raw.nbytes, scale_off=len(scale_f), scale_nbytes=sc.nbytes,
                   bias_off=len(bias_f), bias_nbytes=len(bias))
        code_f.extend(raw.tobytes())
        scale_f.extend(sc.tobytes())
        bias_f.extend(bias)
        return out

    for proj, recs in experts.items():
        index["experts"][proj] = [put(r, e) for e, r in enumerate(recs)]
    for name, rec in (dense or {}).items():
        index["dense"][name] = put(rec, None)
    (path / "codes.bin").write_bytes(bytes(code_f))
    (path / "scales.bf16").write_bytes(bytes(scale_f))
    (path / "bias.bf16").write_bytes(bytes(bias_f))
    (path / "index.json").write_text(json.dumps(index, indent=1))
