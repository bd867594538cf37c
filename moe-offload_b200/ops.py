"""Torch-facing wrappers over the libmoe_b200 C ABI (device tensors in, device tensors out).

Tensor conventions
  x, act, y      torch.bfloat16
  expert weights MLX affine layout (transpose=True): codes int32/uint32 [cap, rows, cols*bits/32],
                 scales/biases float16 or bfloat16 [cap, rows, cols/group_size]
  indices/slots  int32 (bit-identical to the uint32 the reference uses)
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._lib import call

_CODE_DTYPES = (torch.int32, torch.uint32)
_SB_DTYPES = (torch.float16, torch.bfloat16)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _need(t: torch.Tensor, name: str, dtypes, dev=None) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype not in dtypes:
        raise ValueError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dev is not None and t.device != dev:
        raise ValueError(f"{name} is on {t.device}, expected {dev}")


@dataclass
class QMatrix:
    """One affine-quantised weight stack (codes, scales, biases) in MLX layout."""

    w: torch.Tensor
    s: torch.Tensor
    b: torch.Tensor
    bits: int = 2
    group_size: int = 64

    @property
    def sb_fp16(self) -> int:
        return int(self.s.dtype == torch.float16)

    def check(self, name: str, dev) -> None:
        _need(self.w, f"{name}.w", _CODE_DTYPES, dev)
        _need(self.s, f"{name}.s", _SB_DTYPES, dev)
        _need(self.b, f"{name}.b", (self.s.dtype,), dev)


# ----------------------------------------------------------------------------- router

_WS: dict = {}


def router_workspace(device, T: int, E: int, M: int) -> torch.Tensor:
    """Zero-filled router workspace (kept zero by the kernel between calls), cached per
    (device, T, E, M)."""
    key = (torch.device(device), T, E, M)
    ws = _WS.get(key)
    if ws is None:
        nbytes = int(call("moe_router_workspace_bytes", T, E, M))
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def _router_format(w) -> tuple:
    """(bits, group size, fp16 scales) of a router: bf16 tensors are (16, 0, False)."""
    return (w.bits, w.group_size, bool(w.sb_fp16)) if isinstance(w, QMatrix) else (16, 0, False)


def router_topk(x: torch.Tensor, w, K: int, *, w_next=None, M: int = 0, pred_bias=None,
                want_logits: bool = False, want_probs: bool = False, out: dict | None = None,
                stream=None) -> dict:
    """Router for T token rows of x [T, H] bf16.

    w / w_next: bf16 [E, H] tensors, or QMatrix (affine router, 2/4/8 bits).
    Returns dict with inds int32 [T,K] (MLX argpartition order), scores bf16 [T,K] and,
    when requested, pred int32 [T,M], logits bf16 [T,E], probs bf16 [T,E]."""
    _need(x, "x", (torch.bfloat16,))
    T, H = x.shape
    dev = x.device
    if M > 0 and w_next is not None and _router_format(w_next) != _router_format(w):
        # one launch reads both routers in one format: a next-layer router of another format
        # (e.g. an 8-bit router after bf16 ones) gets its own launch, which routes with it and
        # returns its top-M (the same prediction the fused launch computes)
        o = out if out is not None else {}
        router_topk(x, w, K, want_logits=want_logits, want_probs=want_probs, out=o, stream=stream)
        En = w_next.w.shape[0] if isinstance(w_next, QMatrix) else w_next.shape[0]
        po = router_topk(x, w_next, min(K, En), w_next=w_next, M=M, pred_bias=pred_bias,
                         out=o.setdefault("_next_route", {}), stream=stream)
        o["pred"] = po["pred"]
        return o
    if isinstance(w, QMatrix):
        w.check("w", dev)
        E = w.w.shape[0]
        rbits, gs, sbf = w.bits, w.group_size, w.sb_fp16
        wp, wsp, wbp = w.w.data_ptr(), w.s.data_ptr(), w.b.data_ptr()
    else:
        _need(w, "w", (torch.bfloat16,), dev)
        E = w.shape[0]
        rbits, gs, sbf = 16, 64, 0
        wp, wsp, wbp = w.data_ptr(), None, None
    wnp = wnsp = wnbp = None
    if M > 0:
        if w_next is None:
            raise ValueError("M > 0 needs w_next")
        if isinstance(w_next, QMatrix):
            w_next.check("w_next", dev)
            wnp, wnsp, wnbp = w_next.w.data_ptr(), w_next.s.data_ptr(), w_next.b.data_ptr()
        else:
            _need(w_next, "w_next", (torch.bfloat16,), dev)
            wnp = w_next.data_ptr()
    if pred_bias is not None:
        _need(pred_bias, "pred_bias", (torch.float32,), dev)
    o = out if out is not None else {}
    if "inds" not in o:
        o["inds"] = torch.empty((T, K), dtype=torch.int32, device=dev)
    if "scores" not in o:
        o["scores"] = torch.empty((T, K), dtype=torch.bfloat16, device=dev)
    if M > 0 and "pred" not in o:
        o["pred"] = torch.empty((T, M), dtype=torch.int32, device=dev)
    if want_logits and "logits" not in o:
        o["logits"] = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
    if want_probs and "probs" not in o:
        o["probs"] = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
    ws = router_workspace(dev, T, E, M)
    call("moe_router_topk", x.data_ptr(), T, H, E, K, wp, wsp, wbp, rbits, gs, sbf, wnp, wnsp, wnbp,
         M, _ptr(pred_bias), _ptr(o.get("logits")), _ptr(o.get("probs")), o["inds"].data_ptr(),
         o["scores"].data_ptr(), _ptr(o.get("pred")), ws.data_ptr(), ws.numel(), _stream(stream))
    return o


# ----------------------------------------------------------------------------- experts

def experts_gateup(x: torch.Tensor, slots: torch.Tensor, gate: QMatrix, up: QMatrix,
                   act: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """act [T, K, I] = SwiGLU(gate(x), up(x)) for the K routed slots of each token."""
    _need(x, "x", (torch.bfloat16,))
    dev = x.device
    _need(slots, "slots", (torch.int32, torch.uint32), dev)
    gate.check("gate", dev)
    up.check("up", dev)
    T, H = x.shape
    K = slots.shape[-1]
    I = gate.w.shape[1]
    if act is None:
        act = torch.empty((T, K, I), dtype=torch.bfloat16, device=dev)
    call("moe_experts_gateup", x.data_ptr(), T, H, I, K, gate.w.shape[0], slots.data_ptr(), gate.w.data_ptr(),
         gate.s.data_ptr(), gate.b.data_ptr(), up.w.data_ptr(), up.s.data_ptr(), up.b.data_ptr(),
         gate.bits, gate.group_size, gate.sb_fp16, act.data_ptr(), _stream(stream))
    return act


def experts_down(act: torch.Tensor, slots: torch.Tensor, down: QMatrix, scores=None, *,
                 addend=None, resid=None, y=None, want_yk: bool = False, yk=None, stream=None):
    """y [T, H] = sum_k down(act[:, k]) * scores[:, k] (+ addend) (+ resid); optionally the
    unweighted per-expert outputs yk [T, K, H]. Returns (y, yk)."""
    _need(act, "act", (torch.bfloat16,))
    dev = act.device
    _need(slots, "slots", (torch.int32, torch.uint32), dev)
    down.check("down", dev)
    T, K, I = act.shape
    H = down.w.shape[1]
    if scores is not None:
        _need(scores, "scores", (torch.bfloat16,), dev)
        if y is None:
            y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    else:
        y = None
    if want_yk and yk is None:
        yk = torch.empty((T, K, H), dtype=torch.bfloat16, device=dev)
    for name, t in (("addend", addend), ("resid", resid)):
        if t is not None:
            _need(t, name, (torch.bfloat16,), dev)
    call("moe_experts_down", act.data_ptr(), T, H, I, K, down.w.shape[0], slots.data_ptr(), _ptr(scores),
         down.w.data_ptr(), down.s.data_ptr(), down.b.data_ptr(), down.bits, down.group_size,
         down.sb_fp16, _ptr(addend), _ptr(resid), _ptr(y), _ptr(yk), _stream(stream))
    return y, yk


# ----------------------------------------------------------------------------- shared expert

def _lin_dims(name: str, m: QMatrix, dev):
    m.check(name, dev)
    if m.w.dim() != 2:
        raise ValueError(f"{name}.w must be 2-D [N, K*bits/32], got {tuple(m.w.shape)}")
    return m.w.shape[0], m.w.shape[1] * 32 // m.bits


def affine_linear(x: torch.Tensor, w: QMatrix, *, y=None, stream=None) -> torch.Tensor:
    """y [T, N] = x [T, K] . W^T for one affine-quantised matrix (QLinear::forward,
    cpp/src/kernels.cpp:997-1019)."""
    _need(x, "x", (torch.bfloat16,))
    N, K = _lin_dims("w", w, x.device)
    T = x.numel() // K if x.shape[-1] == K else -1
    if T < 1:
        raise ValueError(f"x has shape {tuple(x.shape)}, expected [..., {K}]")
    if y is None:
        y = torch.empty((T, N), dtype=torch.bfloat16, device=x.device)
    call("moe_affine_linear", x.data_ptr(), T, K, N, w.w.data_ptr(), w.s.data_ptr(), w.b.data_ptr(), w.bits,
         w.group_size, w.sb_fp16, y.data_ptr(), _stream(stream))
    return y


_SWS: dict = {}


def shared_expert(x: torch.Tensor, gate: QMatrix, up: QMatrix, down: QMatrix, expert_gate: QMatrix, *,
                  y=None, stream=None) -> torch.Tensor:
    """shared_y [T, H] = sigmoid(x . We^T) * down(SwiGLU(x . Wg^T, x . Wu^T)): the layer's
    shared expert (engine.cpp:394-400, loader.py:909-910), the addend of experts_down /
    decode_layer."""
    _need(x, "x", (torch.bfloat16,))
    dev = x.device
    I, H = _lin_dims("gate", gate, dev)
    if _lin_dims("up", up, dev) != (I, H) or _lin_dims("down", down, dev) != (H, I) or \
            _lin_dims("expert_gate", expert_gate, dev) != (1, H):
        raise ValueError("shared expert matrices disagree on H / I")
    if (up.bits, down.bits, up.group_size, down.group_size) != (gate.bits,) * 2 + (gate.group_size,) * 2:
        raise ValueError("gate/up/down must share bits and group_size")
    if len({gate.sb_fp16, up.sb_fp16, down.sb_fp16, expert_gate.sb_fp16}) != 1:
        raise ValueError("scales/biases of the shared expert must share one dtype")
    T = x.numel() // H
    if x.shape[-1] != H or T < 1:
        raise ValueError(f"x has shape {tuple(x.shape)}, expected [..., {H}]")
    need = call("moe_shared_expert_workspace_bytes", T, H, I)
    key = (dev, stream)
    ws = _SWS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        _SWS[key] = ws
    if y is None:
        y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    call("moe_shared_expert", x.data_ptr(), T, H, I, gate.w.data_ptr(), gate.s.data_ptr(), gate.b.data_ptr(),
         up.w.data_ptr(), up.s.data_ptr(), up.b.data_ptr(), down.w.data_ptr(), down.s.data_ptr(),
         down.b.data_ptr(), gate.bits, gate.group_size, expert_gate.w.data_ptr(), expert_gate.s.data_ptr(),
         expert_gate.b.data_ptr(), expert_gate.bits, expert_gate.group_size, gate.sb_fp16, y.data_ptr(),
         ws.data_ptr(), ws.numel(), _stream(stream))
    return y


# ----------------------------------------------------------------------------- hyper-connections

_HWS: dict = {}


def hc_mix(h: torch.Tensor, norm_w: torch.Tensor, down: QMatrix, up: QMatrix, inject=None, *, write=None,
           eps: float = 1e-6, hc: int = 4, stream=None):
    """run_hc (kernels.cpp:1363-1560) for quantised mixer matrices: returns (mixed [T, H],
    written [T, hc*H], inj [T, hc]). h: [..., hc*H] bf16; write: (branch [..., H],
    gate [..., hc]) or None (then written is h itself); inject None = the mixer without inject
    weights (inj zeros). T <= 16 rows follow the reference's decode rounding, more rows its
    prefill rounding."""
    _need(h, "h", (torch.bfloat16,))
    dev = h.device
    R, W = _lin_dims("down", down, dev)
    if _lin_dims("up", up, dev) != (W, R):
        raise ValueError("up must be [hc*H, R] for down [R, hc*H]")
    if inject is not None and _lin_dims("inject", inject, dev) != (hc, W):
        raise ValueError(f"inject must be [{hc}, {W}]")
    if h.shape[-1] != W:
        raise ValueError(f"h has shape {tuple(h.shape)}, expected [..., {W}]")
    _need(norm_w, "norm_w", (torch.bfloat16,), dev)
    if norm_w.numel() != W:
        raise ValueError(f"norm_w has {norm_w.numel()} values, expected {W}")
    H = W // hc
    T = h.numel() // W
    mixed = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    inj = torch.empty((T, hc), dtype=torch.bfloat16, device=dev)
    branch = gate = written = None
    if write is not None:
        branch, gate = write
        _need(branch, "branch", (torch.bfloat16,), dev)
        _need(gate, "gate", (torch.bfloat16,), dev)
        if branch.numel() != T * H or gate.numel() != T * hc:
            raise ValueError("write tensors must be [T, H] and [T, hc]")
        written = torch.empty((T, W), dtype=torch.bfloat16, device=dev)
    need = call("moe_hc_workspace_bytes", T, hc, H, R)
    key = (dev, stream)
    ws = _HWS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        _HWS[key] = ws
    i_w = i_s = i_b = None
    i_bits, i_gs = 8, 64
    if inject is not None:
        i_w, i_s, i_b, i_bits, i_gs = inject.w, inject.s, inject.b, inject.bits, inject.group_size
    if len({down.sb_fp16, up.sb_fp16} | ({inject.sb_fp16} if inject is not None else set())) != 1:
        raise ValueError("mixer matrices must share one scale dtype")
    call("moe_hc_mix", h.data_ptr(), T, hc, H, R, _ptr(branch), _ptr(gate), norm_w.data_ptr(), float(eps),
         down.w.data_ptr(), down.s.data_ptr(), down.b.data_ptr(), down.bits, down.group_size, up.w.data_ptr(),
         up.s.data_ptr(), up.b.data_ptr(), up.bits, up.group_size, _ptr(i_w), _ptr(i_s), _ptr(i_b), i_bits, i_gs,
         down.sb_fp16, _ptr(written), mixed.data_ptr(), inj.data_ptr(), ws.data_ptr(), ws.numel(),
         _stream(stream))
    return mixed, (written if written is not None else h.reshape(T, W)), inj


# ----------------------------------------------------------------------------- fused layer

_DWS: dict = {}


def decode_workspace(device, T: int, H: int, I: int, E: int, K: int, M: int) -> torch.Tensor:
    key = (torch.device(device), T, H, I, E, K, M)
    ws = _DWS.get(key)
    if ws is None:
        nbytes = int(call("moe_decode_workspace_bytes", T, H, I, E, K, M))
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _DWS[key] = ws
    return ws


def decode_layer(x: torch.Tensor, router: torch.Tensor, gate: QMatrix, up: QMatrix, down: QMatrix,
                 K: int, *, router_next=None, M: int = 0, pred_bias=None, addend=None, resid=None,
                 norm: bool = False, out: dict | None = None, workspace: torch.Tensor | None = None,
                 stream=None) -> dict:
    """One decode step of an all-resident layer: router -> experts -> combine (three kernels).
    norm=True feeds the MoE block x * 2^-k (power of two nearest x's RMS; see the C header).
    Returns dict(y, inds, scores[, pred])."""
    _need(x, "x", (torch.bfloat16,))
    dev = x.device
    T, H = x.shape
    _need(router, "router", (torch.bfloat16,), dev)
    E = router.shape[0]
    I = gate.w.shape[1]
    for name, q in (("gate", gate), ("up", up), ("down", down)):
        q.check(name, dev)
    o = out if out is not None else {}
    o.setdefault("y", torch.empty((T, H), dtype=torch.bfloat16, device=dev))
    o.setdefault("inds", torch.empty((T, K), dtype=torch.int32, device=dev))
    o.setdefault("scores", torch.empty((T, K), dtype=torch.bfloat16, device=dev))
    if M > 0:
        _need(router_next, "router_next", (torch.bfloat16,), dev)
        o.setdefault("pred", torch.empty((T, M), dtype=torch.int32, device=dev))
    ws = workspace if workspace is not None else decode_workspace(dev, T, H, I, E, K, M)
    call("moe_decode_layer", x.data_ptr(), T, H, I, E, K, router.data_ptr(), _ptr(router_next if M else None),
         M, _ptr(pred_bias), gate.w.data_ptr(), gate.s.data_ptr(), gate.b.data_ptr(), up.w.data_ptr(),
         up.s.data_ptr(), up.b.data_ptr(), down.w.data_ptr(), down.s.data_ptr(), down.b.data_ptr(),
         gate.sb_fp16, int(norm), _ptr(addend), _ptr(resid), o["inds"].data_ptr(), o["scores"].data_ptr(),
         _ptr(o.get("pred")), o["y"].data_ptr(), ws.data_ptr(), ws.numel(), _stream(stream))
    return o


# ----------------------------------------------------------------------------- host helpers

def pow2_rms_shift(h_bits) -> int:
    """k such that h * 2^-k has RMS in [2^-0.5, 2^0.5): k = floor(e / 2) with mean(h^2) in
    [2^(e-1), 2^e) (the rule the kernels apply for norm=True). h_bits: bf16 bit patterns."""
    import numpy as np

    v = (np.asarray(h_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    ss = float(np.sum(v * v))
    if not ss > 0.0:
        return 0
    _, e = np.frexp(ss / v.size)
    return int(e) // 2


def pow2_normalize(h_bits):
    """bf16 bits of h * 2^-k (exact) for k = pow2_rms_shift(h)."""
    import numpy as np

    k = pow2_rms_shift(h_bits)
    f = (np.asarray(h_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    return (np.ascontiguousarray(f * np.float32(2.0 ** -k)).view(np.uint32) >> 16).astype(np.uint16)


# ----------------------------------------------------------------------------- prefill

_PWS: dict = {}


def prefill_experts(x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor, gate: QMatrix, up: QMatrix,
                    down: QMatrix, *, resid=None, y=None, stream=None) -> torch.Tensor:
    """Prefill of T tokens through the routed experts (expert-grouped tcgen05 GEMMs):
    y [T, H] = (resid +) sum_k bf16(expert_k(x) * scores[:, k]). x bf16 [T, H], inds int32
    [T, K], scores bf16 [T, K] (router order), experts in the MLX layout [E, ...]."""
    _need(x, "x", (torch.bfloat16,))
    dev = x.device
    _need(inds, "inds", (torch.int32, torch.uint32), dev)
    _need(scores, "scores", (torch.bfloat16,), dev)
    for n, q in (("gate", gate), ("up", up), ("down", down)):
        q.check(n, dev)
    T, H = x.shape
    K = inds.shape[-1]
    E, I = gate.w.shape[0], gate.w.shape[1]
    if resid is not None:
        _need(resid, "resid", (torch.bfloat16,), dev)
    if y is None:
        y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    nb = int(call("moe_prefill_workspace_bytes", T, H, I, E, K))
    key = (dev, nb)
    ws = _PWS.get(key)
    if ws is None:
        ws = torch.empty(nb, dtype=torch.uint8, device=dev)
        _PWS.clear()
        _PWS[key] = ws
    call("moe_prefill_experts", x.data_ptr(), T, H, I, E, K, inds.data_ptr(), scores.data_ptr(),
         gate.w.data_ptr(), gate.s.data_ptr(), gate.b.data_ptr(), up.w.data_ptr(), up.s.data_ptr(),
         up.b.data_ptr(), down.w.data_ptr(), down.s.data_ptr(), down.b.data_ptr(), gate.sb_fp16,
         _ptr(resid), y.data_ptr(), None, ws.data_ptr(), ws.numel(), _stream(stream))
    return y


_PLWS: dict = {}


def prefill_layer(x: torch.Tensor, router: torch.Tensor, gate: QMatrix, up: QMatrix, down: QMatrix, K: int, *,
                  norm: bool = True, resid=None, out: dict | None = None, stream=None) -> dict:
    """One resident layer's prefill of T rows: router (bit-exact top-k) -> expert-grouped
    tcgen05 GEMMs -> combine. norm=True feeds router and experts the per-row power-of-two
    RMS normalisation of x; resid (bf16 [T, H], typically x) is added once. Returns
    dict(y, inds, scores)."""
    _need(x, "x", (torch.bfloat16,))
    dev = x.device
    T, H = x.shape
    _need(router, "router", (torch.bfloat16,), dev)
    E = router.shape[0]
    I = gate.w.shape[1]
    for n, q in (("gate", gate), ("up", up), ("down", down)):
        q.check(n, dev)
    if resid is not None:
        _need(resid, "resid", (torch.bfloat16,), dev)
    o = out if out is not None else {}
    o.setdefault("y", torch.empty((T, H), dtype=torch.bfloat16, device=dev))
    o.setdefault("inds", torch.empty((T, K), dtype=torch.int32, device=dev))
    o.setdefault("scores", torch.empty((T, K), dtype=torch.bfloat16, device=dev))
    nb = int(call("moe_prefill_layer_workspace_bytes", T, H, I, E, K))
    key = (dev, T, H, I, E, K)
    ws = _PLWS.get(key)
    if ws is None:
        ws = torch.zeros(nb, dtype=torch.uint8, device=dev)
        _PLWS.clear()
        _PLWS[key] = ws
    call("moe_prefill_layer", x.data_ptr(), T, H, I, E, K, router.data_ptr(), gate.w.data_ptr(), gate.s.data_ptr(),
         gate.b.data_ptr(), up.w.data_ptr(), up.s.data_ptr(), up.b.data_ptr(), down.w.data_ptr(), down.s.data_ptr(),
         down.b.data_ptr(), gate.sb_fp16, int(norm), _ptr(resid), o["inds"].data_ptr(), o["scores"].data_ptr(),
         o["y"].data_ptr(), ws.data_ptr(), ws.numel(), _stream(stream))
    return o


# ----------------------------------------------------------------------------- mixer + shared, all layers

def f3_layer_rows(layers: list[dict], device):
    """Checks mixer + shared-expert layers (F3Stack's dict form) and returns (H, R, I, sb_fp16,
    rows): rows[l] = the 22 device pointers of moe_f3_layer (norm weight, then codes, scales,
    biases of down, up, inject (0 when absent), shared gate, up, down and the scalar gate)."""
    ly0 = layers[0]
    R, W = ly0["down"].w.shape[0], ly0["down"].w.shape[1] * 32 // ly0["down"].bits
    H, I = W // 4, ly0["sg"].w.shape[0]
    sbs = set()
    rows = []
    for ly in layers:
        want = {"down": (8, R, W), "up": (8, W, R), "inj": (8, 4, W), "sg": (4, I, H), "su": (4, I, H),
                "sd": (4, H, I), "se": (8, 1, H)}
        if ly["nw"].data_ptr() % 16:
            raise ValueError("f3 layer: norm weight must be 16-byte aligned")
        ptrs = [ly["nw"].data_ptr()]
        for k in F3Stack.KEYS:
            q = ly.get(k)
            if q is None:
                if k != "inj":
                    raise ValueError(f"f3 layer: {k} missing")
                ptrs += [0, 0, 0]
                continue
            bits, n, kin = want[k]
            if q.bits != bits or q.group_size != 64 or q.w.shape[0] != n or q.w.shape[1] * 32 // q.bits != kin:
                raise ValueError(f"f3 layer: {k} must be {bits}-bit g64 [{n}, {kin}]")
            q.check(k, device)
            sbs.add(q.sb_fp16)
            ptrs += [q.w.data_ptr(), q.s.data_ptr(), q.b.data_ptr()]
        rows.append(ptrs)
    if len(sbs) != 1:
        raise ValueError("f3 layers: one scale dtype expected")
    return H, R, I, sbs.pop(), rows


class F3MoeStack:
    """The MoE half of every decoder layer for a decode token, all layers in ONE launch
    (moe_f3moe_stack_decode): per layer the hyper-connection mixer with the previous block's
    write, the routed block on the mixer output (router, precise softmax, MLX-order top-k,
    renorm, experts) and the shared expert, the block output being the routed combine with the
    shared output as its addend (loader.py:909-914). mix_layers: F3Stack's dicts; routed:
    ExpertLayer per layer (router [E, H] bf16, 2-bit g64 experts), packed once here."""

    def __init__(self, mix_layers: list[dict], routed: list, top_k: int, device, eps: float = 1e-6,
                 num_ctas: int = 0):
        from .stack import pack_layer_experts
        if len(mix_layers) != len(routed):
            raise ValueError("one routed layer per mixer layer expected")
        self.device = torch.device(device)
        self.L, self.K = len(routed), int(top_k)
        self.eps, self.num_ctas = float(eps), int(num_ctas)
        self.H, self.R, self.Is, self.sb_mix, rows = f3_layer_rows(mix_layers, self.device)
        if not all(isinstance(ly.router, torch.Tensor) and ly.router.dtype == torch.bfloat16 for ly in routed):
            raise ValueError("the fused stack reads bf16 [E, H] routers")
        self.E, H = routed[0].router.shape
        self.I = routed[0].gate.w.shape[1]
        if H != self.H:
            raise ValueError(f"routed layers of H={H}, mixer layers of H={self.H}")
        self.sb_exp = routed[0].gate.sb_fp16
        self.router_t = [ly.router.t().contiguous() for ly in routed]
        self.packed = [pack_layer_experts(ly, self.device) for ly in routed]
        self.mix_layers = mix_layers                   # the table points into these tensors
        table = [r + [rt.data_ptr(), pk.data_ptr()] for r, rt, pk in zip(rows, self.router_t, self.packed)]
        self.table = torch.tensor(table, dtype=torch.int64, device=self.device)
        nb = int(call("moe_f3moe_stack_workspace_bytes", self.H, self.R, self.Is, self.I, self.E, self.K))
        self.ws = torch.empty(nb, dtype=torch.uint8, device=self.device)
        self.launches_per_step = 1

    def decode(self, h: torch.Tensor, branch=None, gate=None, *, want_all: bool = False, out=None, stream=None):
        """h bf16 [4H]; branch / gate: the pending write (bf16 [H] / [4]) or None. Returns a dict:
        state [4H] (after the last block's write), branch [H] and inj [4] (the last block output
        and its gate), inds [L, K] / scores [L, K] (every layer's routing), and with want_all
        branch_all [L, H] and mixed_all [L, H] (every layer's block output and block input)."""
        _need(h, "h", (torch.bfloat16,), self.device)
        o = out if out is not None else {}
        dv, bf = self.device, torch.bfloat16
        st = o.setdefault("state", torch.empty(4 * self.H, dtype=bf, device=dv))
        br = o.setdefault("branch", torch.empty(self.H, dtype=bf, device=dv))
        inj = o.setdefault("inj", torch.empty(4, dtype=bf, device=dv))
        inds = o.setdefault("inds", torch.empty((self.L, self.K), dtype=torch.int32, device=dv))
        scores = o.setdefault("scores", torch.empty((self.L, self.K), dtype=bf, device=dv))
        ball = mall = None
        if want_all:
            ball = o.setdefault("branch_all", torch.empty((self.L, self.H), dtype=bf, device=dv))
            mall = o.setdefault("mixed_all", torch.empty((self.L, self.H), dtype=bf, device=dv))
        call("moe_f3moe_stack_decode", self.table.data_ptr(), self.L, self.H, self.R, self.Is, self.I, self.E, self.K,
             int(self.sb_mix), int(self.sb_exp), self.eps, h.data_ptr(), _ptr(branch), _ptr(gate), st.data_ptr(),
             br.data_ptr(), inj.data_ptr(), inds.data_ptr(), scores.data_ptr(), _ptr(ball), _ptr(mall),
             self.ws.data_ptr(), self.ws.numel(), self.num_ctas, _stream(stream))
        return o


class F3Stack:
    """The step in front of every MoE block for a decode token, all layers in one launch
    (moe_f3_stack_decode): per layer the hyper-connection mixer with the previous block's write
    and the shared expert on its output, the shared expert's output being the block output
    (the same bits as hc_mix + shared_expert per layer). layers: dicts with "nw" (bf16 [4H]),
    "down" [R, 4H], "up" [4H, R], "inj" [4, 4H] or None (8-bit g64), "sg" / "su" [I, H], "sd"
    [H, I] (4-bit g64), "se" [1, H] (8-bit g64), all QMatrix with one scale dtype."""

    KEYS = ("down", "up", "inj", "sg", "su", "sd", "se")

    def __init__(self, layers: list[dict], device, eps: float = 1e-6, num_ctas: int = 0):
        self.device = torch.device(device)
        self.L = len(layers)
        self.eps, self.num_ctas = float(eps), int(num_ctas)
        self.H, self.R, self.I, self.sb_fp16, rows = f3_layer_rows(layers, self.device)
        self.layers = layers                       # the table points into these tensors
        self.table = torch.tensor(rows, dtype=torch.int64, device=self.device)
        nb = int(call("moe_f3_stack_workspace_bytes", self.H, self.R, self.I))
        self.ws = torch.empty(nb, dtype=torch.uint8, device=self.device)

    def decode(self, h: torch.Tensor, branch=None, gate=None, *, want_all: bool = False, out=None, stream=None):
        """h bf16 [4H] (or [1, 4H]); branch / gate: the pending write (bf16 [H] / [4]) or None.
        Returns (state [4H] after the last block's write, last block output [H], its gate [4],
        every layer's block output [L, H] or None)."""
        _need(h, "h", (torch.bfloat16,), self.device)
        o = out if out is not None else {}
        st = o.setdefault("state", torch.empty(4 * self.H, dtype=torch.bfloat16, device=self.device))
        br = o.setdefault("branch", torch.empty(self.H, dtype=torch.bfloat16, device=self.device))
        inj = o.setdefault("inj", torch.empty(4, dtype=torch.bfloat16, device=self.device))
        alls = None
        if want_all:
            alls = o.setdefault("all", torch.empty((self.L, self.H), dtype=torch.bfloat16, device=self.device))
        call("moe_f3_stack_decode", self.table.data_ptr(), self.L, self.H, self.R, self.I, self.sb_fp16, self.eps,
             h.data_ptr(), _ptr(branch), _ptr(gate), st.data_ptr(), br.data_ptr(), inj.data_ptr(), _ptr(alls),
             self.ws.data_ptr(), self.ws.numel(), self.num_ctas, _stream(stream))
        return st, br, inj, alls
