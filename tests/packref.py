"""Numpy restatement of the packed expert layout (moe_pack_experts): test infrastructure
only, used to check the CUDA packer byte for byte."""
import numpy as np


def pack_experts_np(g, u, d, H: int, I: int) -> np.ndarray:
    """g, u: (codes u32 [E, I, H/16], scales u16 [E, I, H/64], biases u16); d: (codes u32
    [E, H, I/16], scales u16 [E, H, I/64], biases u16). Returns u8 [E, I/64 * 60 * H]."""
    E = g[0].shape[0]
    ngH, ngI = H // 64, I // 64
    out = np.zeros((E, ngI, 60 * H), np.uint8)
    for G in range(ngI):
        for uu in range(8):
            rows = 64 * G + 8 * uu + np.arange(8)
            base = uu * 5 * H
            for m, mat in enumerate((g, u)):
                w = mat[0][:, rows, :].reshape(E, 8, ngH // 4, 4, 4)       # [E, g, j, t, word]
                chunks = np.ascontiguousarray(w.transpose(0, 2, 1, 3, 4))  # [E, j, g, t, word]
                out[:, G, base + m * 2 * H: base + (m + 1) * 2 * H] = chunks.reshape(E, -1).view(np.uint8)
            parts = []
            for a in (g[1], g[2], u[1], u[2]):
                v = a[:, rows, :].reshape(E, 8, ngH // 4, 4)                # [E, g, j, t]
                parts.append(v.transpose(0, 2, 1, 3))
            rec = np.ascontiguousarray(np.stack(parts, axis=-1).astype(np.uint16))   # [E, j, g, t, 4]
            out[:, G, base + 4 * H: base + 5 * H] = rec.reshape(E, -1).view(np.uint8)
        dc = np.ascontiguousarray(d[0][:, :, 4 * G: 4 * G + 4])                # [E, H, 4]
        out[:, G, 40 * H: 56 * H] = dc.reshape(E, -1).view(np.uint8)
        ds = np.ascontiguousarray(np.stack([d[1][:, :, G], d[2][:, :, G]], axis=-1).astype(np.uint16))
        out[:, G, 56 * H: 60 * H] = ds.reshape(E, -1).view(np.uint8)
    return out.reshape(E, -1)
