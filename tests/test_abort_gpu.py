"""The kernels' bounded waits driven to expiry on the GPU, without faulting, trapping or hanging it.

mxfp6_set_wait_budget(1) gives every barrier wait inside the GEMM kernels launched by this
thread a budget of one clock cycle, far below the work: some role (TMA producer, MMA issuer or
epilogue) gives up, sets its MXFP6_DEV_* bit and raises the CTA's abort flag (the pair kernel
also raises its peer's); the other roles leave their loops; the CTA then waits, with the default
budget, for its loads and MMAs in flight, frees tensor memory and returns. The test checks that
the kernel returned (the device synchronises), that the status word reports the timeout, and
that the next call with the default budget on the same device is correct. The reference has no
equivalent (its kernels have no bounded waits and report nothing).
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT_BITS = 0x1 | 0x2 | 0x4  # producer, MMA issuer, epilogue (0x8: a drain that did not settle)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


@pytest.mark.parametrize("MT,NT", [(128, 128), (128, 256), (256, 256)])
def test_expired_waits_report_and_leave_the_device_usable(lib, oracle, MT, NT):
    from gpu_helpers import DeviceOperands, check, run_gemm
    from mxfp6_b200.synth import make_operands
    # 96 K slabs per tile: a tile takes tens of microseconds, so the epilogue's one-cycle wait for
    # its accumulator cannot be met. (K = 12288 also keeps an unsplit FP32 result within the
    # oracle's 1e-5 bound.)
    ops = make_operands(512, 512, 12288, kind="codes", seed=21, exp_range=(109, 127))
    dev = DeviceOperands(ops)
    before = run_gemm(dev, lib.OutType.F32, force=(MT, NT, 1))
    D = torch.zeros((ops.M, ops.N), dtype=torch.float32, device="cuda")
    assert lib.device_status() == 0
    prev = lib.set_wait_budget(1)
    try:
        lib.gemm_force_tile(lib.OutType.F32, ops.M, ops.N, ops.Kp, MT, NT, 1, dev.A, dev.Bt, dev.sA, dev.sB, D,
                            ops.row_bytes, ops.row_bytes)
        assert lib.last_error() == lib.OK  # the launch itself was accepted
        status = lib.device_status()       # synchronises: the kernel returned
    finally:
        assert lib.set_wait_budget(prev) == 1
    assert status != -1, "device synchronisation failed after the timed-out kernel"
    assert status & TIMEOUT_BITS, f"no timeout reported (status 0x{status:x})"
    assert lib.last_error() == lib.ERR_DEVICE_TIMEOUT
    # the same call with the default budget, on the same device, is right: bit for bit the result
    # of the call made before the timeout, and within tolerance of the oracle
    Dn = run_gemm(dev, lib.OutType.F32, force=(MT, NT, 1))
    assert torch.equal(Dn.view(torch.int32), before.view(torch.int32))
    check(Dn, oracle.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp), lib.OutType.F32, oracle,
          label=f"after timeout {MT}x{NT}")


def test_wait_budget_is_per_thread(lib):
    """The budget is a setting of the calling host thread: another thread keeps the default."""
    import threading
    prev = lib.set_wait_budget(12345)
    seen = {}

    def other():
        seen["v"] = lib.set_wait_budget(0)

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["v"] == 0
    assert lib.set_wait_budget(prev) == 12345
