"""Seeded random shapes through every route. For each case (M and N multiples of 128 up to a few
thousand, so 256-wide tiles are often partial; K any multiple of 32, so the last 128-deep slab is
often partly zero; every output type):

* the routed call matches the oracle on sampled rows (full N and K);
* every unsplit route -- 128x128, 128x256, the CTA pair, and the pair with its stream-K tail where
  the tiles leave a partial last wave -- gives the same bits: each sums an element's K blocks in
  the same order, whatever the tile or schedule;
* one forced K split (a random factor, its segments short enough for the FP32 tolerance) matches
  the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FP32_SEGMENT_K = 12288  # the route's FP32 accuracy bound on one accumulator's K (route.hpp)


def _cases(n=28, seed=2026):
    rng = np.random.default_rng(seed)
    outs = ["F32", "F16", "BF16"]
    cases = []
    for i in range(n):
        M = 128 * int(rng.integers(1, 17))
        N = 128 * int(rng.integers(1, 25))
        K = 32 * int(rng.integers(1, 257))
        cases.append((M, N, K, outs[i % 3]))
    # shapes whose 256x256 tiles leave a partial last wave of 74 CTA pairs (stream-K engages)
    cases += [(2304, 2304, 2080, "BF16"), (2048, 3072, 1344, "F16"), (2432, 2560, 992, "F32")]
    return cases


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _bits(t):
    return t.view(torch.int32) if t.dtype == torch.float32 else t.view(torch.int16)


@pytest.mark.parametrize("M,N,K,out", _cases())
def test_random_shape_every_route(lib, oracle, M, N, K, out):
    from gpu_helpers import DeviceOperands, check, run_gemm, sample_rows
    from mxfp6_b200.synth import make_operands
    ops = make_operands(M, N, K, kind="codes", seed=M * 131 + N * 17 + K, exp_range=(109, 127))
    dev = DeviceOperands(ops)
    o = lib.OutType[out]
    rows = sample_rows(M, 40)
    ref = oracle.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp, rows=rows)
    label = f"{M}x{N}x{K} {out}"

    check(run_gemm(dev, o), ref, o, oracle, rows=rows, label=f"{label} routed")

    slabs = ops.Kp // 128
    if out != "F32" or ops.Kp <= FP32_SEGMENT_K:
        unsplit = [run_gemm(dev, o, force=(128, 128, 1)), run_gemm(dev, o, force=(128, 256, 1)),
                   run_gemm(dev, o, force=(256, 256, 1))]
        tiles = -(-M // 256) * -(-N // 256)
        if tiles >= 74 and tiles % 74:
            unsplit.append(run_gemm(dev, o, force=(256, 256, 1, 1)))
        for D in unsplit[1:]:
            assert torch.equal(_bits(D), _bits(unsplit[0])), f"{label}: unsplit routes differ"
        check(unsplit[0], ref, o, oracle, rows=rows, label=f"{label} unsplit")

    rng = np.random.default_rng(M + N + K)
    lo = max(2, -(-ops.Kp // FP32_SEGMENT_K)) if out == "F32" else 2
    if slabs >= lo:
        S = int(rng.integers(lo, min(slabs, max(lo, 9)) + 1))
        MT, NT = [(128, 128), (128, 256), (256, 256)][int(rng.integers(0, 3))]
        D = run_gemm(dev, o, force=(MT, NT, S))
        check(D, ref, o, oracle, rows=rows, label=f"{label} {MT}x{NT} S={S}")
