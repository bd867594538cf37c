#!/usr/bin/env python3
"""Regenerate the committed golden fixtures under tests/golden/ (run in a container that
has the reference checkout; the GPU box only reads the committed outputs).

Outputs
-------
moe_fixture.safetensors
    The `moe.*` tensors of the reference's own golden file
    mlx-qwen38/cpp/tests/fixtures.safetensors (written by cpp/tests/gen_fixtures.py:469-575
    through the real MLX modules, checked bit-exactly by cpp/tests/test_kernels.cpp:436-540):
    an MoE block with H=256, 16 experts, top-4, I=128; router 8-bit affine g64, routed
    experts 2-bit affine g64 with bf16 scales/biases; decode input x_dec [1,1,256] and
    prefill input x_pre [1,20,256]; MLX outputs inds_*, scores_*, sh_* (shared expert) and
    y_* (block output). Copied byte-for-byte, no recomputation.

hc_fixture.safetensors
    The `hc.*` and `pred_next.*` tensors of the same file (gen_fixtures.py:105-177,
    685-705; checked by test_kernels.cpp:57-92,216-283): the hyper-connection mixer in front
    of the MoE block with hidden 2560, 4 streams, low rank 320, 8-bit affine g64 down / up /
    inject matrices; inputs h_in [1,rows,10240], branch br_in [1,rows,2560] and gate gt_in
    [1,rows,4] for rows 1, 8 and 18; MLX outputs m_* (mixed input), h_write (written
    stream), inj_* (inject weights), mix_* (the use_combine=False mixer), and the next-layer
    top-12 predictions of an 8-bit 64-expert gate on m. h_nowrite and h_mix_write are left
    out when they equal h_in / h_write (the generator asserts which).

lru_trace.npz
    Hit/miss/slot/LRU-order trace of the reference's own LRU slot cache
    (mlx-qwen38/expert_io.c, compiled unmodified by oracle/Makefile into
    oracle/_ref/libexpert_io_ref.so) driven by a seeded synthetic decode sequence: per
    layer, top-k expert draws with Zipf popularity and token-to-token reuse, interleaved
    with next-layer top-M prefetch calls, plus a prefill-style set_lru_state in the middle.

Usage:  python tests/golden/make_golden.py [--ref <checkout of Jakevin/moe-offload>]
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def make_moe_fixture(ref_root: str) -> None:
    from safetensors.torch import load_file, save_file

    src = os.path.join(ref_root, "mlx-qwen38", "cpp", "tests", "fixtures.safetensors")
    allt = load_file(src)
    keep = {k: v.contiguous() for k, v in allt.items() if k.startswith("moe.")}
    dst = os.path.join(HERE, "moe_fixture.safetensors")
    save_file(keep, dst, metadata={"source": "mlx-qwen38/cpp/tests/fixtures.safetensors (moe.* keys)"})
    print(f"wrote {dst}: {len(keep)} tensors, {os.path.getsize(dst)} bytes")


def make_hc_fixture(ref_root: str) -> None:
    import torch
    from safetensors.torch import load_file, save_file

    src = os.path.join(ref_root, "mlx-qwen38", "cpp", "tests", "fixtures.safetensors")
    allt = load_file(src)
    keep = {k: v.contiguous() for k, v in allt.items() if k.startswith(("hc.", "pred_next."))}
    dropped = []
    for tag in ("r1", "r8", "r18"):
        for k, same in ((f"hc.{tag}.h_nowrite", f"hc.{tag}.h_in"), (f"hc.{tag}.h_mix_write", f"hc.{tag}.h_write")):
            if torch.equal(keep[k].view(torch.int16), keep[same].view(torch.int16)):
                del keep[k]
                dropped.append(f"{k}=={same}")
    dst = os.path.join(HERE, "hc_fixture.safetensors")
    save_file(keep, dst, metadata={"source": "mlx-qwen38/cpp/tests/fixtures.safetensors (hc.*, pred_next.* keys)",
                                   "dropped_equal": ",".join(dropped)})
    print(f"wrote {dst}: {len(keep)} tensors, {os.path.getsize(dst)} bytes; dropped {dropped}")


def lru_sequence(seed: int, n_layers: int, steps: int, E: int, K: int, M: int):
    """Seeded synthetic routing: Zipf(1.1) popularity over a per-layer permutation, each of
    the K slots reuses one of the previous token's experts with p=0.3; predictions are the
    next token's experts for the next layer mixed with popular experts (ranked list)."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, E + 1, dtype=np.float64)
    pop = ranks ** -1.1
    pop /= pop.sum()
    perms = [rng.permutation(E) for _ in range(n_layers)]
    prev = [None] * n_layers
    seq = []  # list of (layer, eids[K], preds[M] for layer+1 or None)
    draws = {}
    for t in range(steps):
        for l in range(n_layers):
            chosen: list[int] = []
            while len(chosen) < K:
                if prev[l] is not None and rng.random() < 0.3:
                    e = int(prev[l][rng.integers(0, K)])
                else:
                    e = int(perms[l][rng.choice(E, p=pop)])
                if e not in chosen:
                    chosen.append(e)
            prev[l] = chosen
            draws[(t, l)] = chosen
    for t in range(steps):
        for l in range(n_layers):
            pred = None
            if l + 1 < n_layers:
                nxt = list(draws[(t, l + 1)])
                rng.shuffle(nxt)
                cand = nxt[: M // 2]
                while len(cand) < M:
                    e = int(perms[l + 1][rng.choice(E, p=pop)])
                    if e not in cand:
                        cand.append(e)
                pred = cand
            seq.append((l, draws[(t, l)], pred))
    return seq


def make_lru_trace(lib_path: str) -> None:
    lib = ctypes.CDLL(lib_path)
    u64 = ctypes.c_uint64
    E, K, M, CAP, PCAP, NL, STEPS = 512, 10, 12, 102, 3, 4, 160
    seq = lru_sequence(seed=2, n_layers=NL, steps=STEPS, E=E, K=K, M=M)
    slot_bufs = {}
    zeros9 = (u64 * 9)()
    for l in range(NL):
        buf = (ctypes.c_uint32 * 16)()
        slot_bufs[l] = buf
        lib.c_layer_init(l, -1, CAP, zeros9, zeros9, zeros9, u64(ctypes.addressof(buf)))
    n_miss_all, slots_all, stats_after = [], [], []
    eids_all, preds_all, layers_all, kinds_all = [], [], [], []
    order_snap = []
    for i, (l, eids, pred) in enumerate(seq):
        arr = (ctypes.c_uint32 * K)(*eids)
        n = lib.c_layer_step_decode_ex(l, arr, K, 1)
        n_miss_all.append(n)
        slots_all.append(list(slot_bufs[l])[:K])
        eids_all.append(list(eids))
        layers_all.append(l)
        kinds_all.append(0)
        preds_all.append(list(pred) if pred is not None else [-1] * M)
        if pred is not None:
            parr = (ctypes.c_int32 * M)(*pred)
            lib.c_layer_start_prefetch(l + 1, parr, M, PCAP)
        if i == len(seq) // 2:
            # a prefill-style state rewrite on layer 1: keep the 40 most recent entries,
            # re-slotted positionally, to exercise c_layer_set_lru_state
            oe = (ctypes.c_int32 * 512)()
            os_ = (ctypes.c_int32 * 512)()
            cnt = ctypes.c_int(0)
            lib.c_layer_get_lru_state(1, oe, os_, ctypes.byref(cnt))
            keep_e = list(oe)[: cnt.value][-40:]
            keep_s = list(range(40))
            lib.c_layer_set_lru_state(1, (ctypes.c_int32 * 40)(*keep_e), (ctypes.c_int32 * 40)(*keep_s), 40, u64(400), u64(350), u64(12))
    for l in range(NL):
        st = (u64 * 18)()
        lib.c_layer_get_stats(l, st)
        stats_after.append(list(st))
        oe = (ctypes.c_int32 * 512)()
        os_ = (ctypes.c_int32 * 512)()
        cnt = ctypes.c_int(0)
        lib.c_layer_get_lru_state(l, oe, os_, ctypes.byref(cnt))
        snap = np.full((2, 512), -1, dtype=np.int32)
        snap[0, : cnt.value] = list(oe)[: cnt.value]
        snap[1, : cnt.value] = list(os_)[: cnt.value]
        order_snap.append(snap)
    tot = (u64 * 6)()
    lib.c_get_decode_totals(NL, tot)
    dst = os.path.join(HERE, "lru_trace.npz")
    np.savez_compressed(
        dst,
        params=np.array([E, K, M, CAP, PCAP, NL, STEPS], dtype=np.int64),
        layers=np.array(layers_all, dtype=np.int32),
        eids=np.array(eids_all, dtype=np.int32),
        preds=np.array(preds_all, dtype=np.int32),
        n_miss=np.array(n_miss_all, dtype=np.int32),
        slots=np.array(slots_all, dtype=np.int32),
        stats=np.array(stats_after, dtype=np.uint64),
        lru_state=np.stack(order_snap),
        totals=np.array(list(tot), dtype=np.uint64),
        set_state_at=np.array([len(seq) // 2], dtype=np.int64),
    )
    print(f"wrote {dst}: {len(seq)} decode steps, misses {sum(n_miss_all)}")


def main() -> int:
    ap = argparse.ArgumentParser()
    # the reference checkout: $MOE_REF_ROOT, else a directory named `reference` beside this repository
    ap.add_argument("--ref", default=os.environ.get("MOE_REF_ROOT",
                                                    os.path.join(os.path.dirname(ROOT), "reference")))
    args = ap.parse_args()
    make_moe_fixture(args.ref)
    make_hc_fixture(args.ref)
    lib = os.path.join(ROOT, "oracle", "_ref", "libexpert_io_ref.so")
    if not os.path.exists(lib):
        print("oracle/_ref/libexpert_io_ref.so missing: run `make -C oracle` first", file=sys.stderr)
        return 1
    make_lru_trace(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
