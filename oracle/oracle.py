"""ctypes wrapper over oracle/liboracle.so -- TEST INFRASTRUCTURE ONLY.

The CPU restatement of the routed-expert MoE block (see moe_oracle.c for the arithmetic
model and the reference citations). Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / --impl reference legs import this module; the product package never does.

All arrays are numpy; bf16 tensors travel as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def build() -> None:
    """Compile liboracle.so (and the reference LRU under _ref/ when the sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        I = ctypes.c_int
        L.orc_router_logits.argtypes = [P, I, I, I, I, P, P, P, I, I, P, P]
        L.orc_softmax_topk.argtypes = [P, I, I, I, P, P, P]
        L.orc_topm_sorted.argtypes = [P, I, I, I, P]
        L.orc_experts.argtypes = [P, I, I, I, I, P, P] + [P] * 9 + [I, I, I, P, P, P, P, P]
        L.orc_f64_to_bf16.argtypes = [ctypes.c_double]
        L.orc_f64_to_bf16.restype = ctypes.c_uint16
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_num_threads.restype = I
        L.orc_hc_mix.argtypes = [ctypes.c_void_p, I, I, I, I, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_float] + [ctypes.c_void_p] * 3 + [I, I] + [ctypes.c_void_p] * 3 + [I, I] + \
            [ctypes.c_void_p] * 3 + [I, I, I] + [ctypes.c_void_p] * 4
        L.orc_set_num_threads.argtypes = [I]
        for f in ("orc_router_logits", "orc_softmax_topk", "orc_topm_sorted", "orc_experts",
                  "orc_affine_linear", "orc_shared_expert", "orc_hc_mix"):
            getattr(L, f).restype = I
        _LIB = L
    return _LIB


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _chk(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed with status {rc}")


# ---------------------------------------------------------------- bf16 helpers (numpy)

def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ---------------------------------------------------------------- router

def router_logits(x_bf16: np.ndarray, w, E: int, rbits: int = 16, scales=None, biases=None,
                  group_size: int = 64, sb_fp16: bool = False, bias_f32=None) -> np.ndarray:
    """x [T,H] uint16(bf16); w: bf16 [E,H] (rbits=16) or uint32 [E,H*rbits/32]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T, H = x.shape
    w = np.ascontiguousarray(w)
    s = None if scales is None else np.ascontiguousarray(scales, dtype=np.uint16)
    b = None if biases is None else np.ascontiguousarray(biases, dtype=np.uint16)
    bias = None if bias_f32 is None else np.ascontiguousarray(bias_f32, dtype=np.float32)
    out = np.empty((T, E), dtype=np.uint16)
    _chk(lib().orc_router_logits(_p(x), T, H, E, rbits, _p(w), _p(s), _p(b), group_size,
                                 int(sb_fp16), _p(bias), _p(out)), "router_logits")
    return out


def softmax_topk(logits_bf16: np.ndarray, K: int):
    """-> (probs bf16 [T,E], inds u32 [T,K] in MLX argpartition order, scores bf16 [T,K])"""
    lg = np.ascontiguousarray(logits_bf16, dtype=np.uint16)
    T, E = lg.shape
    probs = np.empty((T, E), dtype=np.uint16)
    inds = np.empty((T, K), dtype=np.uint32)
    scores = np.empty((T, K), dtype=np.uint16)
    _chk(lib().orc_softmax_topk(_p(lg), T, E, K, _p(probs), _p(inds), _p(scores)), "softmax_topk")
    return probs, inds, scores


def topm_sorted(logits_bf16: np.ndarray, M: int) -> np.ndarray:
    lg = np.ascontiguousarray(logits_bf16, dtype=np.uint16)
    T, E = lg.shape
    pred = np.empty((T, M), dtype=np.uint32)
    _chk(lib().orc_topm_sorted(_p(lg), T, E, M, _p(pred)), "topm_sorted")
    return pred


# ---------------------------------------------------------------- experts

def experts(x_bf16, slots, scores_bf16, gate, up, down, bits: int = 2, group_size: int = 64,
            sb_fp16: bool = True, addend=None, resid=None, want_act=False, want_yk=False):
    """gate/up/down: (w u32, scales u16, biases u16) slot buffers in MLX layout.
    Returns dict(y=bf16 [T,H] or None, act=[T,K,I], yk=[T,K,H])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T, H = x.shape
    sl = np.ascontiguousarray(slots, dtype=np.uint32).reshape(T, -1)
    K = sl.shape[1]
    sc = None if scores_bf16 is None else np.ascontiguousarray(scores_bf16, dtype=np.uint16).reshape(T, K)
    wg, sg, bg = (np.ascontiguousarray(a) for a in gate)
    wu, su, bu = (np.ascontiguousarray(a) for a in up)
    wd, sd, bd = (np.ascontiguousarray(a) for a in down)
    I = wg.shape[-2]
    ad = None if addend is None else np.ascontiguousarray(addend, dtype=np.uint16).reshape(T, H)
    rs = None if resid is None else np.ascontiguousarray(resid, dtype=np.uint16).reshape(T, H)
    y = np.empty((T, H), dtype=np.uint16) if sc is not None else None
    act = np.empty((T, K, I), dtype=np.uint16) if want_act else None
    yk = np.empty((T, K, H), dtype=np.uint16) if want_yk else None
    _chk(lib().orc_experts(_p(x), T, H, I, K, _p(sl), _p(sc), _p(wg), _p(sg), _p(bg), _p(wu),
                           _p(su), _p(bu), _p(wd), _p(sd), _p(bd), bits, group_size, int(sb_fp16),
                           _p(ad), _p(rs), _p(y), _p(act), _p(yk)), "experts")
    return {"y": y, "act": act, "yk": yk}



# ---------------------------------------------------------------- shared expert

def affine_linear(x_bf16, w, bits: int, group_size: int, sb_fp16: bool = False):
    """y [T, N] bf16 bits = x [T, K] . W^T for W = (codes u32 [N, K*bits/32], scales, biases)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    wq, s, b = (np.ascontiguousarray(a) for a in w)
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    x = x.reshape(-1, K)
    T = x.shape[0]
    y = np.empty((T, N), dtype=np.uint16)
    _chk(lib().orc_affine_linear(_p(x), T, K, N, _p(wq), _p(s), _p(b), bits, group_size, int(sb_fp16), _p(y)),
         "affine_linear")
    return y


def shared_expert(x_bf16, gate, up, down, expert_gate, bits: int = 4, group_size: int = 64, gate_bits: int = 8,
                  gate_group_size: int = 64, sb_fp16: bool = False):
    """The shared expert (engine.cpp:394-400). gate/up/down/expert_gate: (codes, scales, biases)
    2-D matrices. Returns dict(y=[T, H], act=[T, I], o=[T, H]) as bf16 bits."""
    wg, sg, bg = (np.ascontiguousarray(a) for a in gate)
    wu, su, bu = (np.ascontiguousarray(a) for a in up)
    wd, sd, bd = (np.ascontiguousarray(a) for a in down)
    we, se, be = (np.ascontiguousarray(a) for a in expert_gate)
    I, H = wg.shape[0], wg.shape[1] * 32 // bits
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, H)
    T = x.shape[0]
    y = np.empty((T, H), dtype=np.uint16)
    act = np.empty((T, I), dtype=np.uint16)
    o = np.empty((T, H), dtype=np.uint16)
    _chk(lib().orc_shared_expert(_p(x), T, H, I, _p(wg), _p(sg), _p(bg), _p(wu), _p(su), _p(bu), _p(wd), _p(sd),
                                 _p(bd), bits, group_size, _p(we), _p(se), _p(be), gate_bits, gate_group_size,
                                 int(sb_fp16), _p(y), _p(act), _p(o)), "shared_expert")
    return {"y": y, "act": act, "o": o}



# ---------------------------------------------------------------- hyper-connection mixer

def hc_mix(h_bf16, norm_w, down, up, inject=None, branch=None, gate=None, hc: int = 4, eps: float = 1e-6,
           bits: int = 8, group_size: int = 64, sb_fp16: bool = False):
    """run_hc (kernels.cpp:1363-1560) for T rows of HC*H stream values. down/up/inject:
    (codes, scales, biases) with `bits` / `group_size`; inject None = the mixer without inject
    weights; branch [T, H] and gate [T, HC] bf16 = the write. Returns dict(mixed=[T, H],
    written=[T, HC*H], normed=[T, HC*H], inj=[T, HC]) as bf16 bits."""
    wd, sd, bd = (np.ascontiguousarray(a) for a in down)
    wu, su, bu = (np.ascontiguousarray(a) for a in up)
    R = wd.shape[0]
    W = wu.shape[0]
    H = W // hc
    h = np.ascontiguousarray(h_bf16, dtype=np.uint16).reshape(-1, W)
    T = h.shape[0]
    wi = si = bi = None
    if inject is not None:
        wi, si, bi = (np.ascontiguousarray(a) for a in inject)
    br = None if branch is None else np.ascontiguousarray(branch, dtype=np.uint16).reshape(T, H)
    gt = None if gate is None else np.ascontiguousarray(gate, dtype=np.uint16).reshape(T, hc)
    nw = np.ascontiguousarray(norm_w, dtype=np.uint16).reshape(-1)
    out = {"mixed": np.empty((T, H), np.uint16), "written": np.empty((T, W), np.uint16),
           "normed": np.empty((T, W), np.uint16), "inj": np.empty((T, hc), np.uint16)}
    _chk(lib().orc_hc_mix(_p(h), T, hc, H, R, _p(br), _p(gt), _p(nw), eps, _p(wd), _p(sd), _p(bd), bits, group_size,
                          _p(wu), _p(su), _p(bu), bits, group_size, _p(wi), _p(si), _p(bi), bits, group_size,
                          int(sb_fp16), _p(out["written"]), _p(out["normed"]), _p(out["mixed"]), _p(out["inj"])),
         "hc_mix")
    return out


def ref_lru_lib(version: int = 1):
    """The reference's own expert_io.c compiled under oracle/_ref (None when absent)."""
    name = "libexpert_io_ref.so" if version == 1 else "libexpert_io_ref_v2.so"
    path = os.path.join(HERE, "_ref", name)
    if not os.path.exists(path):
        return None
    return ctypes.CDLL(path)


# ---------------------------------------------------------------- token loop (numpy)
#
# The step after the routed block: the LM head and the next-token choice of the reference's
# decode loop (mlx-qwen38/server.py:93-110 `_sample_next_token`, loader.py:1153-1180
# `mx.argmax(out.logits[:, -1:, :])`), restated with the arithmetic the library documents for
# moe_lm_head_logits / moe_sample_tokens: exact bf16 x bf16 products, double sums in the
# kernel's fixed order (lane l of 32 takes the 8-element chunks l, l + 32, ... in order, then an
# xor butterfly over the lanes), one rounding to fp32; argmax = first index of the maximum;
# sampling = Gumbel-max over the top-p set with a splitmix64 hash of (seed, counter, row, index).

def lm_head_logits(head_bf16: np.ndarray, x_bf16: np.ndarray) -> np.ndarray:
    """head u16 [V, H], x u16 [T, H] -> fp32 [T, V]."""
    w = bf16_to_f32(np.ascontiguousarray(head_bf16, dtype=np.uint16))
    x = bf16_to_f32(np.ascontiguousarray(x_bf16, dtype=np.uint16))
    V, H = w.shape
    T = x.shape[0]
    nch = H // 8
    out = np.empty((T, V), dtype=np.float32)
    for v0 in range(0, V, 256):
        wv = w[v0:v0 + 256]
        prod = (wv[None, :, :] * x[:, None, :]).astype(np.float64)          # exact products
        prod = prod.reshape(T, wv.shape[0], nch, 8)
        lanes = np.zeros((T, wv.shape[0], 32), dtype=np.float64)
        for lane in range(32):
            seq = prod[:, :, lane::32, :].reshape(T, wv.shape[0], -1)
            if seq.shape[-1]:
                lanes[:, :, lane] = np.cumsum(seq, axis=-1)[..., -1]          # sequential order
        idx = np.arange(32)
        for off in (16, 8, 4, 2, 1):
            lanes = lanes + lanes[..., idx ^ off]
        out[:, v0:v0 + 256] = lanes[..., 0].astype(np.float32)
    return out


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xbf58476d1ce4e5b9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94d049bb133111eb)
    return z ^ (z >> np.uint64(31))


def sample_uniform(seed: int, counter: int, row: int, V: int) -> np.ndarray:
    """The library's uniform variates in (0, 1) for indices 0..V-1 of one row."""
    with np.errstate(over="ignore"):
        s = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) ^ (np.uint64(counter & 0xFFFFFFFFFFFFFFFF) *
                                                    np.uint64(0x9e3779b97f4a7c15))
        base = _mix64(np.array([s], dtype=np.uint64))[0]
        key = (np.uint64(row & 0xFFFFFFFF) << np.uint64(32)) | np.arange(V, dtype=np.uint64)
        z = _mix64(base ^ key)
    return ((z >> np.uint64(11)).astype(np.float64) + 0.5) * 2.0 ** -53


def sample_tokens(logits: np.ndarray, temperature: float = 0.0, top_p: float = 1.0, seed: int = 0,
                  counter: int = 0) -> np.ndarray:
    """fp32 [T, V] -> int32 [T] (moe_sample_tokens' rule)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    T, V = lg.shape
    out = np.empty(T, dtype=np.int32)
    for t in range(T):
        if not temperature > 0.0:
            out[t] = int(np.argmax(lg[t]))
            continue
        s = lg[t] / np.float32(temperature)
        p = np.exp(s - s.max()).astype(np.float32)
        keep = p > 0
        if 0.0 < top_p < 1.0:
            z = float(p.astype(np.float64).sum())
            need = top_p * z
            lo, hi = 0, int(np.float32(1.0).view(np.uint32))
            while lo < hi:
                mid = lo + (hi - lo + 1) // 2
                fm = np.uint32(mid).view(np.float32)
                if float(p[p >= fm].astype(np.float64).sum()) >= need:
                    lo = mid
                else:
                    hi = mid - 1
            keep &= p >= np.uint32(lo).view(np.float32)
        u = sample_uniform(seed, counter, t, V)
        key = (s.astype(np.float64) - np.log(-np.log(u))).astype(np.float32)
        key = np.where(keep, key, -np.inf).astype(np.float32)
        out[t] = int(np.argmax(key))
    return out
