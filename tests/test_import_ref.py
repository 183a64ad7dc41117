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


# ---- forward layout generators (test inputs) against the reference's own layouts ----------------

def test_forward_preshuffle_matches_reference(golden):
    from ref_layouts import preshuffle_ref
    Bt = golden["imp_Bt"]
    assert np.array_equal(preshuffle_ref(Bt, Bt.shape[1] * 4 // 3), golden["imp_Bsh"])


@pytest.mark.parametrize("which,dim,group", [("sB", 256, 2), ("sB", 256, 4), ("sA", 128, 2), ("sA", 128, 4)])
def test_forward_tile_scales_matches_reference(golden, which, dim, group):
    from ref_layouts import tile_scales_ref
    raw = golden[f"imp_{which}"]
    assert np.array_equal(tile_scales_ref(raw, dim, raw.shape[1] * 32, group, 3),
                          golden[f"imp_{which}_tiled_g{group}"])


# ---- device import (mxfp6_import_ref_*_device) ----------------------------------------------------

def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.fixture
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.gpu
def test_device_import_B_golden(lib, golden, cuda):
    Bsh, Bt = golden["imp_Bsh"], golden["imp_Bt"]
    N, Kp_ref = Bt.shape[0], Bt.shape[1] * 4 // 3
    rb = lib.kpad(Kp_ref) * 3 // 4
    out = cuda.full((N, rb), 0xA5, dtype=cuda.uint8, device="cuda")
    assert lib.import_ref_B_device(_dev(Bsh), N, Kp_ref, out, rb) == lib.OK
    cuda.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), lib.import_ref_B(Bsh, N, Kp_ref))


# (N, K): the reference pads K to a multiple of 192 (Kp_ref), this library to a multiple of 128:
# 8192 -> 8256 vs 8192 (the reference's zero tail is dropped; 129 steps, a partial last block),
# 160 -> 192 vs 256 (this library's extra tail is zeroed), 4096 -> 4224 vs 4096.
@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(1024, 8192), (256, 160), (4096, 4096)])
def test_device_import_B_sizes(lib, cuda, N, K):
    from ref_layouts import preshuffle_ref
    Kp_ref = (K + 191) // 192 * 192
    rng = np.random.default_rng(N + K)
    Bt_ref = rng.integers(0, 256, (N, Kp_ref * 3 // 4), dtype=np.uint8)
    Bt_ref[:, K * 3 // 4:] = 0  # the reference's zero K padding
    rb = lib.kpad(K) * 3 // 4
    out = cuda.full((N, rb), 0xA5, dtype=cuda.uint8, device="cuda")
    assert lib.import_ref_B_device(_dev(preshuffle_ref(Bt_ref, Kp_ref)), N, Kp_ref, out, rb) == lib.OK
    cuda.cuda.synchronize()
    want = np.zeros((N, rb), np.uint8)
    n = min(rb, Bt_ref.shape[1])
    want[:, :n] = Bt_ref[:, :n]
    assert np.array_equal(out.cpu().numpy(), want)


@pytest.mark.gpu
@pytest.mark.parametrize("dim,K,group", [(256, 384, 4), (1024, 8192, 4), (256, 160, 2), (384, 4096, 3)])
def test_device_import_scales(lib, cuda, dim, K, group):
    from ref_layouts import tile_scales_ref
    Kp_ref = (K + 191) // 192 * 192
    Kp = lib.kpad(K)
    rng = np.random.default_rng(dim + K + group)
    raw = rng.integers(100, 150, (dim, Kp_ref // 32), dtype=np.uint8)
    ref_tiled = tile_scales_ref(raw, dim, Kp_ref, group, 3)
    out = cuda.full((lib.tiled_scale_bytes(dim, Kp),), 0xA5, dtype=cuda.uint8, device="cuda")
    assert lib.import_ref_scales_device(_dev(ref_tiled), dim, Kp_ref, group, 3, out, Kp) == lib.OK
    cuda.cuda.synchronize()
    want_raw = np.full((dim, Kp // 32), 127, np.uint8)
    n = min(Kp, Kp_ref) // 32
    want_raw[:, :n] = raw[:, :n]
    assert np.array_equal(out.cpu().numpy(), lib.preprocess_scale(want_raw, dim, Kp))


@pytest.mark.gpu
def test_gemm_on_device_imported_layouts(lib, golden, oracle, cuda):
    """The device import of the reference's buffers feeds the GEMM directly (no host step for B
    or the scales) and equals the oracle on the original operands."""
    from gpu_helpers import check
    Bt, sB, A, sA = golden["imp_Bt"], golden["imp_sB"], golden["imp_A"], golden["imp_sA"]
    N, M, Kp_ref = Bt.shape[0], A.shape[0], Bt.shape[1] * 4 // 3
    Kp = lib.kpad(Kp_ref)
    rb = Kp * 3 // 4
    dB = cuda.empty((N, rb), dtype=cuda.uint8, device="cuda")
    dsB = cuda.empty((lib.tiled_scale_bytes(N, Kp),), dtype=cuda.uint8, device="cuda")
    dsA = cuda.empty((lib.tiled_scale_bytes(M, Kp),), dtype=cuda.uint8, device="cuda")
    assert lib.import_ref_B_device(_dev(golden["imp_Bsh"]), N, Kp_ref, dB, rb) == lib.OK
    assert lib.import_ref_scales_device(_dev(golden["imp_sB_tiled_g4"]), N, Kp_ref, 4, 3, dsB, Kp) == lib.OK
    assert lib.import_ref_scales_device(_dev(golden["imp_sA_tiled_g4"]), M, Kp_ref, 4, 3, dsA, Kp) == lib.OK
    dA = cuda.empty((M, rb), dtype=cuda.uint8, device="cuda")
    assert lib.repad_rows_device(_dev(A), M, A.shape[1], A.shape[1], dA, rb) == lib.OK
    D = cuda.empty((M, N), dtype=cuda.float32, device="cuda")
    lib.gemm(lib.OutType.F32, M, N, Kp, dA, dB, dsA, dsB, D, rb, rb)
    assert lib.last_error() == lib.OK
    assert lib.device_status() == 0
    check(D.cpu(), oracle.gemm(A, sA, Bt, sB, Kp_ref), lib.OutType.F32, oracle, label="device-imported layouts")


@pytest.mark.gpu
@pytest.mark.parametrize("extra", [8, 24])
def test_device_import_B_odd_stride(lib, cuda, extra):
    """An output stride that is a multiple of 8 but not of 16 takes the 8-byte store path; the
    bytes past the reference's row are zeroed."""
    from ref_layouts import preshuffle_ref
    N, K = 512, 2048
    Kp_ref = (K + 191) // 192 * 192
    rng = np.random.default_rng(extra)
    Bt_ref = rng.integers(0, 256, (N, Kp_ref * 3 // 4), dtype=np.uint8)
    Bt_ref[:, K * 3 // 4:] = 0
    rb = Kp_ref * 3 // 4 + extra
    out = cuda.full((N, rb), 0xA5, dtype=cuda.uint8, device="cuda")
    assert lib.import_ref_B_device(_dev(preshuffle_ref(Bt_ref, Kp_ref)), N, Kp_ref, out, rb) == lib.OK
    cuda.cuda.synchronize()
    want = np.zeros((N, rb), np.uint8)
    want[:, :Bt_ref.shape[1]] = Bt_ref
    assert np.array_equal(out.cpu().numpy(), want)
