"""Re-entrancy of the drop-in entry (the reference's gemm() is pure and stream-ordered; this
library adds only a thread-local last error): several host threads issue GEMMs at once, each on
its own stream with its own output and workspace, on routes with and without split-K. Every
result must be bit-identical to the same call made alone, and a thread's rejected call must not
show up in the other threads' last_error()."""
from __future__ import annotations

import threading

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(512, 768, 1408), (256, 384, 32768), (2048, 2048, 1024), (1024, 512, 24576)]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def test_threads_on_their_own_streams(lib):
    from gpu_helpers import DeviceOperands, run_gemm
    from mxfp6_b200.synth import make_operands
    ot = lib.OutType.BF16
    jobs = []
    for i, (M, N, K) in enumerate(SHAPES):
        dev = DeviceOperands(make_operands(M, N, K, kind="codes", seed=40 + i))
        jobs.append((dev, _bits(run_gemm(dev, ot)).clone()))

    errors = []
    barrier = threading.Barrier(len(jobs) + 1)

    def worker(dev, want):
        try:
            o = dev.ops
            stream = torch.cuda.Stream()
            wsb = lib.gemm_workspace_size(o.M, o.N, o.Kp, ot)
            ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
            outs = [torch.empty((o.M, o.N), dtype=torch.bfloat16, device="cuda") for _ in range(4)]
            barrier.wait()
            for D in outs:
                lib.gemm(ot, o.M, o.N, o.Kp, dev.A, dev.Bt, dev.sA, dev.sB, D, o.row_bytes, o.row_bytes,
                         ws if wsb else None, wsb, stream=stream)
                if lib.last_error() != lib.OK:
                    errors.append(f"{o.M}x{o.N}x{o.Kp}: {lib.last_error_string()}")
                    return
                stream.synchronize()  # the workspace is reused by the next call on this stream
            for D in outs:
                if not torch.equal(_bits(D.cpu()), want):
                    errors.append(f"{o.M}x{o.N}x{o.Kp}: result differs from the call made alone")
                    return
        except Exception as e:  # reported through `errors`
            errors.append(repr(e))

    def rejecter():
        try:
            barrier.wait()
            dev = jobs[0][0]
            for _ in range(20):
                lib.gemm(ot, 100, 128, 128, dev.A, dev.Bt, dev.sA, dev.sB, dev.A, 96, 96)
                if lib.last_error() != lib.ERR_INVALID_SHAPE:
                    errors.append(f"rejecting thread saw {lib.last_error()}")
                    return
        except Exception as e:
            errors.append(repr(e))

    threads = [threading.Thread(target=worker, args=job) for job in jobs]
    threads.append(threading.Thread(target=rejecter))
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in threads), "a worker thread did not finish"
    assert not errors, errors
    torch.cuda.synchronize()
    assert lib.device_status() == 0


def test_repeated_and_alternating_calls_follow_their_buffers(lib, oracle):
    """Tensor maps are reused per thread when a call repeats its buffers and shape. Alternating two
    operand sets of one shape, refilling a buffer in place, and shrinking M on the same buffers
    must each give the result of a fresh call on the current contents."""
    from gpu_helpers import DeviceOperands, run_gemm
    from mxfp6_b200.synth import make_operands
    ot = lib.OutType.F16
    M, N, K = 1024, 768, 2048
    d1 = DeviceOperands(make_operands(M, N, K, kind="codes", seed=91))
    d2 = DeviceOperands(make_operands(M, N, K, kind="codes", seed=92))
    r1, r2 = _bits(run_gemm(d1, ot)).clone(), _bits(run_gemm(d2, ot)).clone()
    for _ in range(3):
        assert torch.equal(_bits(run_gemm(d1, ot)), r1)
        assert torch.equal(_bits(run_gemm(d2, ot)), r2)
    # new contents at the same addresses
    d1.A.copy_(d2.A)
    d1.Bt.copy_(d2.Bt)
    d1.sA.copy_(d2.sA)
    d1.sB.copy_(d2.sB)
    assert torch.equal(_bits(run_gemm(d1, ot)), r2)
    # the same buffers read as a smaller problem: the first 512 rows of A and 384 rows of B^T,
    # whose scale atoms are the leading atoms of the full buffers
    from gpu_helpers import check
    o = d2.ops
    m, n = 512, 384
    wsb = lib.gemm_workspace_size(m, n, o.Kp, ot)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
    D = torch.empty((m, n), dtype=torch.float16, device="cuda")
    lib.gemm(ot, m, n, o.Kp, d1.A, d1.Bt, d1.sA, d1.sB, D, o.row_bytes, o.row_bytes, ws if wsb else None, wsb)
    assert lib.last_error() == lib.OK
    torch.cuda.synchronize()
    check(D.cpu(), oracle.gemm(o.A[:m], o.sA[:m], o.Bt[:n], o.sB[:n], o.Kp), ot, oracle, label="prefix problem")
