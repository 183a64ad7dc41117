"""Column-parallel (N) sharding of an MXFP6 GEMM across ranks.

D[M, N] = A[M, K] · B[K, N] splits with no exchange step: rank r of g holds all of A and the B^T
rows [r·N/g, (r+1)·N/g) with their scale rows, and computes the D column slab of the same range.
Concatenating the slabs along columns gives D. The optional all-gather of D moves the slabs,
which arrive stacked as [g][M][N/g], into row-major D[M][N] with assemble_columns().
"""
from __future__ import annotations

import numpy as np


def shard_range(N: int, world: int, rank: int) -> tuple[int, int]:
    """Columns [lo, hi) of rank `rank`; N must split into equal multiples of 128."""
    if N % world or (N // world) % 128:
        raise ValueError(f"N={N} does not split into {world} shards of a multiple of 128 columns")
    w = N // world
    return rank * w, (rank + 1) * w


def shard_B(Bt: np.ndarray, sB: np.ndarray, world: int, rank: int):
    """This rank's rows of B^T (packed) and of its raw scales. Tile the scales per shard."""
    lo, hi = shard_range(Bt.shape[0], world, rank)
    return np.ascontiguousarray(Bt[lo:hi]), np.ascontiguousarray(sB[lo:hi])


def assemble_columns(stacked):
    """[g][M][N/g] slabs (numpy or torch) -> row-major [M][N]."""
    g, M, w = stacked.shape
    if hasattr(stacked, "permute"):
        return stacked.permute(1, 0, 2).reshape(M, g * w)
    return np.ascontiguousarray(np.transpose(stacked, (1, 0, 2)).reshape(M, g * w))
