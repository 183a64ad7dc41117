"""Forward versions of the reference library's gfx950 layouts, for generating import test inputs
of any size (test infrastructure only; checked against the layouts the reference's own functions
produced, tests/golden/golden.npz imp_*):

  preshuffle_ref: include/mxfp6/preprocess.hpp:182-207 of eeezio/mxfp6-gemm. Per (32-column,
    64-deep) tile of B^T, 1536 bytes: entry t (0..63) covers column 32*tile + t%32 and K half t/32
    (24 packed bytes), split 16 bytes at t*16 and 8 bytes at 1024 + t*8.
  tile_scales_ref: tile_scale(preprocess_scale(raw, dim, Kp), group, subs), preprocess.hpp:136-162
    and 216-233. Byte ((((g*k_tiles + kt)*64 + lane)*subs + sub)*group_pad + j) holds raw scale
    (row (g*group + j)*32 + lane%32, block 2*(kt*subs + sub) + lane/32); pad bytes are 0.
"""
from __future__ import annotations

import numpy as np


def preshuffle_ref(Bt: np.ndarray, Kp_ref: int) -> np.ndarray:
    N = Bt.shape[0]
    k64 = Kp_ref // 64
    rows = np.ascontiguousarray(Bt[:, :k64 * 48]).reshape(N // 32, 32, k64, 2, 24)  # nt, c, ki, h, bytes
    first = rows[..., :16].transpose(0, 2, 3, 1, 4).reshape(N // 32, k64, 1024)    # t = c + 32h
    second = rows[..., 16:].transpose(0, 2, 3, 1, 4).reshape(N // 32, k64, 512)
    return np.concatenate([first, second], axis=2).reshape(-1)


def tile_scales_ref(raw: np.ndarray, dim: int, Kp_ref: int, group: int, subs: int = 3) -> np.ndarray:
    group_pad = (group + 3) // 4 * 4
    k_tiles = Kp_ref // 64 // subs
    ng = dim // 32 // group
    out = np.zeros((ng, k_tiles, 64, subs, group_pad), np.uint8)
    lane = np.arange(64)
    for g in range(ng):
        for j in range(group):
            row = (g * group + j) * 32 + lane % 32
            for kt in range(k_tiles):
                for sub in range(subs):
                    block = 2 * (kt * subs + sub) + lane // 32
                    out[g, kt, :, sub, j] = raw[row, block]
    return out.reshape(-1)
