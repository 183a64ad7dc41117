"""GEMMs captured in a CUDA graph. The library's kernels are launched with programmatic stream
serialization (each waits for the previous kernel in its stream before touching global memory),
so a chain of calls captured once and replayed must give the results of the same calls made
eagerly, bit for bit: a plain tile route, a split-K route (GEMM then reduce, the reduce reading
the partials the GEMM just wrote) and a stream-K route (hand-offs between CTA pairs), back to back
in one graph, replayed several times with the outputs cleared in between."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

# (M, N, K, output): 128x128 tiles; the CTA pair with a K split and its reduce; the CTA pair's
# stream-K tail (224 tiles on 74 pairs, 64 slabs each)
CASES = [(512, 768, 1408, "BF16"), (1024, 1024, 32768, "F16"), (4096, 3584, 8192, "BF16")]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def test_captured_chain_matches_eager_calls(lib):
    from gpu_helpers import TORCH_OUT, DeviceOperands
    from mxfp6_b200.synth import make_operands
    jobs = []
    for i, (M, N, K, out) in enumerate(CASES):
        ot = lib.OutType[out]
        dev = DeviceOperands(make_operands(M, N, K, kind="codes", seed=60 + i, exp_range=(109, 127)))
        o = dev.ops
        wsb = lib.gemm_workspace_size(o.M, o.N, o.Kp, ot)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
        D = torch.empty((o.M, o.N), dtype=TORCH_OUT[ot], device="cuda")
        jobs.append((ot, dev, ws, wsb, D))
    r = lib.route(lib.OutType.F16, 1024, 1024, 32768)
    assert r["splits"] > 1, r  # the chain covers a split-K route
    assert lib.route(lib.OutType.BF16, 4096, 3584, 8192)["stream_k"]

    stream = torch.cuda.Stream()

    def chain():
        for ot, dev, ws, wsb, D in jobs:
            o = dev.ops
            lib.gemm(ot, o.M, o.N, o.Kp, dev.A, dev.Bt, dev.sA, dev.sB, D, o.row_bytes, o.row_bytes,
                     ws if wsb else None, wsb, stream=stream)
            assert lib.last_error() == lib.OK, lib.last_error_string()

    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        chain()
    stream.synchronize()
    assert lib.device_status() == 0
    want = [_bits(D).clone() for *_, D in jobs]

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain()
    for rep in range(3):
        for *_, D in jobs:
            D.view(torch.uint8).fill_(0x5A + rep)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            g.replay()
        stream.synchronize()
        assert lib.device_status() == 0
        for (ot, dev, *_), D, w in zip(jobs, [j[4] for j in jobs], want):
            assert torch.equal(_bits(D), w), f"{dev.ops.M}x{dev.ops.N}x{dev.ops.Kp} replay {rep} differs"
    del g
