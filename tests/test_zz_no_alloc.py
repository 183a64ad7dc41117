"""mxfp6_gemm_static_workspace: the entry point for callers that cannot call cudaMalloc (a plugin
whose host application owns all device memory, a foreign-function binding that only forwards
pointers it was given). It runs the same route as mxfp6_gemm, with split-K partials in the
library's fixed device array instead of a caller workspace.

This file sorts last on purpose: if it fails, a run that stops at the first failure has already
run every other test. It must also pass alone in a fresh process (the first call on a device
looks the array's address up).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

# Shapes whose route needs scratch that fits the 32 MiB array: FP16 output splits
# 2048x1024x105728 two ways; FP32 output keeps split segments short (9 ways at this K), so it
# uses a smaller M x N.
SHAPES = {"F16": (2048, 1024, 105728), "F32": (1024, 512, 105728)}


def _operands(M, N, K):
    from gpu_helpers import DeviceOperands
    from mxfp6_b200.synth import make_operands
    ops = make_operands(M, N, K, kind="codes", seed=77, exp_range=(109, 127))
    return ops, DeviceOperands(ops)


def test_static_workspace_rejects_oversized_split(lib, capfd):
    """A split that needs more scratch than the array holds is refused before any device work."""
    need = None
    for m, n, k in [(1024, 4096, 105728), (1536, 4096, 105728), (1024, 8192, 105728), (2048, 4096, 105728),
                    (1024, 6144, 105728), (512, 8192, 105728), (1024, 3840, 105728)]:
        # the query for the output type of the call below, so the call is refused on the host
        ws = lib.gemm_workspace_size(m, n, k, lib.OutType.F32)
        if ws > lib.static_workspace_bytes():
            need = (m, n, k)
            break
    assert need is not None, "no test shape splits beyond the static workspace"
    m, n, k = need
    assert lib.gemm_workspace_size(m, n, k, lib.OutType.F32) > lib.static_workspace_bytes()
    rb = k * 3 // 4
    # The addresses are never dereferenced: the size check refuses the call before any launch.
    lib.gemm_static_workspace(lib.OutType.F32, m, n, k, 0x10000, 0x20000, 0x30000, 0x40000, 0x50000, rb, rb)
    assert lib.last_error() == lib.ERR_WORKSPACE
    assert "static workspace" in capfd.readouterr().err


@pytest.mark.gpu
@pytest.mark.parametrize("ot", ["F32", "F16"])
def test_static_workspace_matches_caller_workspace(lib, oracle, ot):
    """Two calls in a row through the C ABI give the same bits, within the output type's
    tolerance of the oracle (sampled rows, full K and N), like mxfp6_gemm with a caller
    workspace."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpu_helpers import check, run_gemm, sample_rows
    M, N, K = SHAPES[ot]
    assert lib.gemm_workspace_size(M, N, K, lib.OutType[ot]) > 0
    ops, dev = _operands(M, N, K)
    o = lib.OutType[ot]
    rows = sample_rows(M, 48)
    ref = oracle.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp, rows=rows)
    check(run_gemm(dev, o), ref, o, oracle, rows=rows, label="caller workspace")
    tdt = torch.float32 if o == lib.OutType.F32 else torch.float16
    got = []
    for call in range(2):
        D = torch.empty((M, N), dtype=tdt, device="cuda")
        D.view(torch.uint8).fill_(0x5A + call)
        lib.gemm_static_workspace(o, M, N, ops.Kp, dev.A, dev.Bt, dev.sA, dev.sB, D, ops.row_bytes, ops.row_bytes)
        assert lib.last_error() == lib.OK, lib.last_error_string()
        assert lib.device_status() == 0
        got.append(D.cpu())
    v = (lambda t: t.view(torch.int32)) if o == lib.OutType.F32 else (lambda t: t.view(torch.int16))
    assert torch.equal(v(got[0]), v(got[1]))
    check(got[0], ref, o, oracle, rows=rows, label="static workspace")
