"""Pin the CPU oracle (oracle/mxfp6_oracle.c) to the reference.

1. Against tests/golden/golden.npz, produced by the reference's own functions
   (tests/golden/make_golden.py): codecs, packing, quantisation and the GEMM, bit for bit.
2. Against the reference library itself (oracle/_ref), when it was built on this machine.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import Reference, reference_available


def f32bits(x):
    return np.asarray(x, np.float32).view(np.uint32)


def test_fp6_decode_all_codes(oracle, golden):
    got = np.array([oracle.fp6_to_float(c) for c in range(64)], np.float32)
    assert np.array_equal(f32bits(got), f32bits(golden["fp6_decode"]))


def test_e8m0_decode_all_codes(oracle, golden):
    got = np.array([oracle.e8m0_to_float(c) for c in range(256)], np.float32)
    exp = golden["e8m0_decode"]
    assert np.isnan(got[255]) and np.isnan(exp[255])
    assert np.array_equal(f32bits(got[:255]), f32bits(exp[:255]))


def test_fp6_encode(oracle, golden):
    x = golden["fp6_encode_in"]
    got = np.array([oracle.float_to_fp6(float(v)) for v in x], np.uint8)
    bad = np.nonzero(got != golden["fp6_encode_out"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first inputs {x[bad[:5]]}"


def test_e8m0_encode(oracle, golden):
    x = golden["e8m0_encode_in"]
    got = np.array([oracle.float_to_e8m0(float(v)) for v in x], np.uint8)
    bad = np.nonzero(got != golden["e8m0_encode_out"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first inputs {x[bad[:5]]}"


def test_pack_matches_golden(golden, lib):
    packed = lib.pack_codes(golden["pack_in"].reshape(1, -1)).reshape(-1)
    assert np.array_equal(packed, golden["pack_out"])
    assert np.array_equal(lib.unpack_codes(packed.reshape(1, -1)).reshape(-1), golden["pack_in"])


def test_quantize(oracle, golden):
    packed, scales = oracle.quantize(golden["quant_in"])
    assert np.array_equal(scales, golden["quant_scales"])
    assert np.array_equal(packed, golden["quant_packed"])


@pytest.mark.parametrize("case", ["gemm", "gemmq"])
def test_gemm_bit_exact(oracle, golden, case):
    A, sA, Bt, sB, D = (golden[f"{case}_{k}"] for k in ("A", "sA", "Bt", "sB", "D"))
    K = sA.shape[1] * 32
    got = oracle.gemm(A, sA, Bt, sB, K)
    assert np.array_equal(f32bits(got), f32bits(D))
    # row subsets and thread counts do not change a single bit
    rows = np.array([5, 0, 127, 64])
    sub = oracle.gemm(A, sA, Bt, sB, K, rows=rows, threads=3)
    assert np.array_equal(f32bits(sub), f32bits(D[rows]))


def test_gemm_f64_companion_close(oracle, golden):
    A, sA, Bt, sB, D = (golden[f"gemm_{k}"] for k in ("A", "sA", "Bt", "sB", "D"))
    d64 = oracle.gemm(A, sA, Bt, sB, sA.shape[1] * 32, f64=True)
    assert np.max(np.abs(d64 - D)) / np.max(np.abs(d64)) < 1e-6


def test_output_rounding_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.normal(0, 1e3, 10000), rng.normal(0, 1e-5, 1000),
                        [65504, 65519.99, 65520, 7e4, -7e4, 6e-8, 3e-8, 2.98e-8, np.inf, -np.inf]]).astype(np.float32)
    assert np.array_equal(oracle.round_f16_bits(x), x.astype(np.float16).view(np.uint16))
    import torch
    bf = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.round_bf16_bits(x), bf)


needs_ref = pytest.mark.skipif(not reference_available(), reason="reference CPU path not built here")


@needs_ref
def test_oracle_vs_reference_random():
    from oracle import Oracle
    o, r = Oracle(), Reference()
    rng = np.random.default_rng(11)
    xs = np.concatenate([rng.normal(0, 3, 20000), rng.uniform(-8, 8, 20000)]).astype(np.float32)
    assert all(o.float_to_fp6(float(v)) == r.float_to_fp6(float(v)) for v in xs)
    mat = rng.normal(0, 5, (96, 512)).astype(np.float32)
    assert all(np.array_equal(a, b) for a, b in zip(o.quantize(mat), r.quantize(mat)))
    M, N, K = 96, 160, 640
    A, sA = r.quantize(rng.uniform(-1, 1, (M, K)).astype(np.float32))
    B, sB = r.quantize(rng.uniform(-1, 1, (N, K)).astype(np.float32))
    assert np.array_equal(f32bits(o.gemm(A, sA, B, sB, K)), f32bits(r.gemm(A, sA, B, sB, K)))
    assert np.array_equal(f32bits(r.gemm(A, sA, B, sB, K, threads=4)), f32bits(r.gemm(A, sA, B, sB, K)))
