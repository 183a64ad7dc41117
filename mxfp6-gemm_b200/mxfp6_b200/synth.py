"""Seeded synthetic MXFP6 operands with the BASELINE configurations' value distributions.

No dataset is involved anywhere in this library's measurements: every benchmark and parity case
draws its operands here.

  kind="codes"  E2M3 codes uniform over all 64 codes (so the packed bytes are uniform random
                bytes), E8M0 scale exponents uniform in [lo, hi]          (BASELINE cfgs 1-4)
  kind="uniform" floats U(-1, 1) quantised per 32-block (the reference test's recipe,
                tests/test_gemm.cpp:64-91), K-tail past K zero-padded
  kind="normal" A ~ N(0, sigma_a), B ~ N(0, sigma_b) quantised per 32-block     (BASELINE cfg 5)

Operands are returned in the library's host layouts: A packed [M][3Kp/4] row-major, B^T packed
[N][3Kp/4], raw scales [rows][Kp/32]; tiled scales come from preprocess_scale().
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Operands:
    M: int
    N: int
    K: int
    Kp: int
    A: np.ndarray    # uint8 [M][3Kp/4]
    sA: np.ndarray   # uint8 [M][Kp/32]
    Bt: np.ndarray   # uint8 [N][3Kp/4]
    sB: np.ndarray   # uint8 [N][Kp/32]

    @property
    def row_bytes(self) -> int:
        return self.Kp * 3 // 4


def _kpad(K: int) -> int:
    return (K + 127) // 128 * 128


def make_operands(M: int, N: int, K: int, kind: str = "codes", seed: int = 0,
                  exp_range=(120, 134), sigma=(1.0, 0.02), threads: int = 0) -> Operands:
    from . import quantize_to_mxfp6  # library host helper

    Kp = _kpad(K)
    rng = np.random.default_rng(seed)
    rb = Kp * 3 // 4
    if kind == "codes":
        A = rng.integers(0, 256, (M, rb), dtype=np.uint8)
        Bt = rng.integers(0, 256, (N, rb), dtype=np.uint8)
        lo, hi = exp_range
        sA = rng.integers(lo, hi + 1, (M, Kp // 32), dtype=np.uint8)
        sB = rng.integers(lo, hi + 1, (N, Kp // 32), dtype=np.uint8)
        if K < Kp:  # zero K-tail on both operands (codes 0), finite scales
            kb = K * 3 // 4
            A[:, kb:] = 0
            Bt[:, kb:] = 0
        return Operands(M, N, K, Kp, A, sA, Bt, sB)
    if kind == "uniform":
        af = np.zeros((M, Kp), np.float32)
        bf = np.zeros((N, Kp), np.float32)
        af[:, :K] = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        bf[:, :K] = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    elif kind == "normal":
        af = np.zeros((M, Kp), np.float32)
        bf = np.zeros((N, Kp), np.float32)
        af[:, :K] = rng.standard_normal((M, K), dtype=np.float32) * np.float32(sigma[0])
        bf[:, :K] = rng.standard_normal((N, K), dtype=np.float32) * np.float32(sigma[1])
    else:
        raise ValueError(kind)
    qa = quantize_to_mxfp6(af, threads)
    qb = quantize_to_mxfp6(bf, threads)
    return Operands(M, N, K, Kp, qa.packed_data, qa.scales, qb.packed_data, qb.scales)
