"""Import of buffers laid out for the reference library (gfx950 preshuffle_B, tile_scale). The
golden fixtures hold the reference's own layouts for a K = 384 problem (tests/golden/make_golden.py);
importing them must give back exactly the B^T rows and raw scales they were made from."""
from __future__ import annotations

import numpy as np
import pytest


def test_import_preshuffled_B(lib, golden):
    Bt, Bsh = golden["imp_Bt"], golden["imp_Bsh"]
    N, Kp_ref = Bt.shape[0], Bt.shape[1] * 4 // 3
    out = lib.import_ref_B(Bsh, N, Kp_ref)
    assert out.shape == (N, lib.kpad(Kp_ref) * 3 // 4)
    assert np.array_equal(out[:, :Bt.shape[1]], Bt)
    assert not out[:, Bt.shape[1]:].any()


@pytest.mark.parametrize("which,dim,group", [("sB", 256, 2), ("sB", 256, 4), ("sA", 128, 2), ("sA", 128, 4)])
def test_import_tiled_scales(lib, golden, which, dim, group):
    raw = golden[f"imp_{which}"]
    Kp_ref = raw.shape[1] * 32
    tiled = golden[f"imp_{which}_tiled_g{group}"]
    out = lib.import_ref_scales(tiled, dim, Kp_ref, group, 3)
    assert np.array_equal(out[:, :raw.shape[1]], raw)
    assert (out[:, raw.shape[1]:] == 127).all()


def test_repad_rows(lib):
    src = np.arange(4 * 150, dtype=np.uint32).astype(np.uint8).reshape(4, 150)
    out = lib.repad_rows(src, 144, 192)
    assert np.array_equal(out[:, :144], src[:, :144]) and not out[:, 144:].any()


@pytest.mark.gpu
def test_gemm_on_imported_layouts(lib, golden, oracle):
    """A GEMM fed from imported reference buffers equals the oracle on the original operands."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gpu_helpers import check
    Bt, sB, A, sA = golden["imp_Bt"], golden["imp_sB"], golden["imp_A"], golden["imp_sA"]
    N, M, Kp_ref = Bt.shape[0], A.shape[0], Bt.shape[1] * 4 // 3
    Kp = lib.kpad(Kp_ref)
    Bt_i = lib.import_ref_B(golden["imp_Bsh"], N, Kp_ref)
    sB_i = lib.import_ref_scales(golden["imp_sB_tiled_g4"], N, Kp_ref, 4)
    sA_i = lib.import_ref_scales(golden["imp_sA_tiled_g4"], M, Kp_ref, 4)
    A_i = lib.repad_rows(A, Kp_ref * 3 // 4, Kp * 3 // 4)
    d = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    D = torch.empty((M, N), dtype=torch.float32, device="cuda")
    lib.gemm(lib.OutType.F32, M, N, Kp, d(A_i), d(Bt_i), d(lib.preprocess_scale(sA_i, M, Kp)),
             d(lib.preprocess_scale(sB_i, N, Kp)), D, Kp * 3 // 4, Kp * 3 // 4)
    assert lib.last_error() == lib.OK
    assert lib.device_status() == 0
    check(D.cpu(), oracle.gemm(A, sA, Bt, sB, Kp_ref), lib.OutType.F32, oracle, label="imported layouts")
