"""Generate tests/golden/golden.npz from the REFERENCE's own CPU functions.

The reference (eeezio/mxfp6-gemm) ships no golden vectors, so they are produced here by running
its functions, compiled from its sources by oracle/Makefile into oracle/_ref/libmxfp6ref.so
(ref_shim.cpp forwards to the reference's fp6_e2m3_to_float, float_to_fp6_e2m3, e8m0_to_float,
float_to_e8m0, pack_fp6, quantize_to_mxfp6 and mxfp6_gemm_ref). The fixture then travels with the
repository, so the oracle can be pinned where the reference sources do not exist.

Run:  make -C oracle && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import Reference  # noqa: E402


def fp6_inputs(rng: np.random.Generator) -> np.ndarray:
    """Floats that exercise every rounding branch of the E2M3 encoder."""
    grid = np.arange(-9.0, 9.0 + 1e-9, 1.0 / 64, dtype=np.float64).astype(np.float32)
    # exact ties between neighbouring codes in each binade, and their float neighbours
    ties = []
    for step, lo, hi in ((0.125, 0.0, 1.0), (0.125, 1.0, 2.0), (0.25, 2.0, 4.0), (0.5, 4.0, 7.5)):
        t = np.arange(lo + step / 2, hi, step, dtype=np.float64).astype(np.float32)
        ties += [t, np.nextafter(t, np.float32(np.inf)), np.nextafter(t, np.float32(-np.inf))]
    ties = np.concatenate(ties)
    special = np.array([0.0, -0.0, 7.5, 7.75, 8.0, 1e9, np.inf, -np.inf, 1e-30, -1e-30, 0.0625,
                        -0.0625, 0.0624, 0.0626, 7.4999, 7.25, 7.2499, 7.2501, 0.9375, 0.9376,
                        1.9375, 1.9376, 3.875, 3.876, 1e-45], np.float32)
    rnd = np.concatenate([rng.normal(0, 2, 2000), rng.uniform(-10, 10, 2000),
                          rng.normal(0, 0.1, 1000)]).astype(np.float32)
    return np.concatenate([grid, ties, -ties, special, rnd]).astype(np.float32)


def e8m0_inputs(rng: np.random.Generator) -> np.ndarray:
    p2 = np.ldexp(np.float32(1.0), np.arange(-149, 128)).astype(np.float32)
    near = np.concatenate([p2 * np.float32(1.41421356), p2 * np.float32(1.4142135),
                           p2 * np.float32(1.4142137), np.nextafter(p2, np.float32(np.inf)),
                           np.nextafter(p2, np.float32(0))])
    special = np.array([0.0, -0.0, -1.0, np.inf, 3.4e38, 1e-45, 5e-39], np.float32)
    rnd = np.exp(rng.uniform(-80, 80, 2000)).astype(np.float32)
    v = np.concatenate([p2, near, special, rnd]).astype(np.float32)
    return v[np.isfinite(v) | np.isinf(v)]


def main() -> None:
    ref = Reference()
    rng = np.random.default_rng(20261201)
    out: dict[str, np.ndarray] = {}

    codes = np.arange(64, dtype=np.uint8)
    out["fp6_decode"] = np.array([ref.fp6_to_float(int(c)) for c in codes], np.float32)
    out["e8m0_decode"] = np.array([ref.e8m0_to_float(int(c)) for c in range(256)], np.float32)

    x = fp6_inputs(rng)
    out["fp6_encode_in"] = x
    out["fp6_encode_out"] = np.array([ref.float_to_fp6(float(v)) for v in x], np.uint8)
    y = e8m0_inputs(rng)
    out["e8m0_encode_in"] = y
    out["e8m0_encode_out"] = np.array([ref.float_to_e8m0(float(v)) for v in y], np.uint8)

    c = rng.integers(0, 64, 4096, dtype=np.uint8)
    out["pack_in"] = c
    out["pack_out"] = ref.pack(c)

    # quantisation of a seeded matrix with a few special rows (zeros, a NaN, huge, tiny)
    mat = rng.normal(0, 1, (64, 256)).astype(np.float32)
    mat[1] = 0.0
    mat[2, 5] = np.nan
    mat[3] *= np.float32(1e30)
    mat[4] *= np.float32(1e-30)
    mat[5, ::3] = np.float32(7.5)
    out["quant_in"] = mat
    out["quant_packed"], out["quant_scales"] = ref.quantize(mat)

    # GEMM: random codes over all 64 E2M3 values, scale exponents in [120, 134] (BASELINE cfg 1
    # distribution), small enough for the single-threaded reference.
    M, N, K = 128, 128, 256
    a_codes = rng.integers(0, 64, (M, K), dtype=np.uint8)
    b_codes = rng.integers(0, 64, (N, K), dtype=np.uint8)
    A = np.stack([ref.pack(r) for r in a_codes])
    Bt = np.stack([ref.pack(r) for r in b_codes])
    sA = rng.integers(120, 135, (M, K // 32), dtype=np.uint8)
    sB = rng.integers(120, 135, (N, K // 32), dtype=np.uint8)
    out["gemm_A"], out["gemm_sA"], out["gemm_Bt"], out["gemm_sB"] = A, sA, Bt, sB
    out["gemm_D"] = ref.gemm(A, sA, Bt, sB, K)

    # GEMM on quantised real data (the reference's own test recipe: U(-1,1) floats)
    M2, N2, K2 = 128, 256, 384
    af = rng.uniform(-1, 1, (M2, K2)).astype(np.float32)
    bf = rng.uniform(-1, 1, (K2, N2)).astype(np.float32)
    A2, sA2 = ref.quantize(af)
    B2, sB2 = ref.quantize(np.ascontiguousarray(bf.T))
    out["gemmq_A"], out["gemmq_sA"], out["gemmq_Bt"], out["gemmq_sB"] = A2, sA2, B2, sB2
    out["gemmq_D"] = ref.gemm(A2, sA2, B2, sB2, K2)

    # Reference device layouts (gfx950) for the import path: preshuffle_B and tile_scale with the
    # reference's K_TILE = 192 (subs = 3) and its route groupings, on a small K = 384 problem.
    N3, K3 = 256, 384
    b3 = rng.uniform(-1, 1, (N3, K3)).astype(np.float32)
    B3, sB3 = ref.quantize(b3)
    a3 = rng.uniform(-1, 1, (128, K3)).astype(np.float32)
    A3, sA3 = ref.quantize(a3)
    out["imp_Bt"], out["imp_sB"], out["imp_A"], out["imp_sA"] = B3, sB3, A3, sA3
    out["imp_Bsh"] = ref.preshuffle_B(B3, sB3, K3)
    for grp in (2, 3, 4):
        out[f"imp_sB_tiled_g{grp}"] = ref.tile_scales(sB3, N3, K3, grp, 3) if (N3 // 32) % grp == 0 else np.zeros(0, np.uint8)
        out[f"imp_sA_tiled_g{grp}"] = ref.tile_scales(sA3, 128, K3, grp, 3) if (128 // 32) % grp == 0 else np.zeros(0, np.uint8)

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
