"""Device quantiser (mxfp6_quantize_device) against the host quantize_to_mxfp6, which the
reference's golden vectors pin: packed codes and scales must match byte for byte, including
NaN / Inf / zero / subnormal blocks, for both scale layouts."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _device_quantize(lib, mat, tiled):
    rows, cols = mat.shape
    d = torch.from_numpy(np.ascontiguousarray(mat, dtype=np.float32)).cuda()
    packed = torch.full((rows, cols * 3 // 4), 0xA5, dtype=torch.uint8, device="cuda")
    nsc = lib.tiled_scale_bytes(rows, cols) if tiled else rows * cols // 32
    scales = torch.full((nsc,), 0xA5, dtype=torch.uint8, device="cuda")
    assert lib.quantize_device(d, rows, cols, packed, scales, tiled) == lib.OK
    torch.cuda.synchronize()
    return packed.cpu().numpy(), scales.cpu().numpy()


def _special_matrix(rows, cols, seed):
    rng = np.random.default_rng(seed)
    m = (rng.standard_normal((rows, cols)) * np.exp(rng.uniform(-30, 30, (rows, 1)))).astype(np.float32)
    m[0] = 0.0
    m[1, 3] = np.nan
    m[2, :40] = np.inf
    m[3, 7] = -np.inf
    m[4] = np.float32(1e-41)                 # subnormal inputs
    m[5, ::5] = np.float32(7.5)
    m[6] *= np.float32(1e38)
    m[7, :32] = np.float32(-0.0)
    m[8, :32] = np.nan                       # an all-NaN block
    return m


def test_golden_quantisation(lib, golden):
    p, s = _device_quantize(lib, golden["quant_in"], tiled=False)
    assert np.array_equal(p, golden["quant_packed"])
    assert np.array_equal(s.reshape(golden["quant_scales"].shape), golden["quant_scales"])


@pytest.mark.parametrize("rows,cols", [(128, 128), (200, 96), (257, 4160), (4096, 8192)])
def test_matches_host_raw_scales(lib, rows, cols):
    m = _special_matrix(rows, cols, rows + cols)
    host = lib.quantize_to_mxfp6(m)
    p, s = _device_quantize(lib, m, tiled=False)
    assert np.array_equal(p, host.packed_data)
    assert np.array_equal(s.reshape(rows, cols // 32), host.scales)


@pytest.mark.parametrize("rows,cols", [(128, 256), (384, 1024), (256, 8192)])
def test_matches_host_tiled_scales(lib, rows, cols):
    m = _special_matrix(rows, cols, 7 * rows + cols)
    host = lib.quantize_to_mxfp6(m)
    p, s = _device_quantize(lib, m, tiled=True)
    assert np.array_equal(p, host.packed_data)
    assert np.array_equal(s, lib.preprocess_scale(host.scales, rows, cols))


def test_every_golden_encode_input(lib, golden):
    """Blocks whose max is exactly 7.5 get scale 2^0, so each code is the E2M3 conversion of the
    input itself: every golden encode input with |x| <= 7.5 (and NaN) goes through the device."""
    xs = golden["fp6_encode_in"]
    want = golden["fp6_encode_out"]
    keep = np.isnan(xs) | (np.abs(xs) <= 7.5)
    xs, want = xs[keep], want[keep]
    per = 31
    nblk = (len(xs) + per - 1) // per
    vals = np.zeros(nblk * per, np.float32)
    vals[:len(xs)] = xs
    blocks = np.concatenate([np.full((nblk, 1), 7.5, np.float32), vals.reshape(nblk, per)], axis=1)
    rows = (nblk + 3) // 4
    m = np.zeros((rows * 4, 32), np.float32)
    m[:nblk] = blocks
    m = m.reshape(rows, 128)
    p, s = _device_quantize(lib, m, tiled=False)
    assert (s[:nblk] == 127).all()
    codes = lib.unpack_codes(p).reshape(-1, 32)[:nblk, 1:].reshape(-1)[:len(xs)]
    bad = np.nonzero(codes != want)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first inputs {xs[bad[:5]]}"


@pytest.mark.parametrize("tiled", [False, True])
@pytest.mark.parametrize("rows,cols", [(128, 224), (256, 3808), (130, 160)])
def test_padded_output_rows(lib, rows, cols, tiled):
    """quantize_device_padded: rows of kpad(cols) codes with a zero tail, scales extended with
    code 127 (pad_scales_k), the first cols codes identical to the host quantiser."""
    if tiled and rows % 128:
        pytest.skip("tiled scales cover whole 128-row blocks")
    m = _special_matrix(rows, cols, 3 * rows + cols)
    host = lib.quantize_to_mxfp6(m)
    Kp = lib.kpad(cols)
    d = torch.from_numpy(m).cuda()
    packed = torch.full((rows, Kp * 3 // 4), 0xA5, dtype=torch.uint8, device="cuda")
    nsc = lib.tiled_scale_bytes(rows, Kp) if tiled else rows * Kp // 32
    scales = torch.full((nsc,), 0xA5, dtype=torch.uint8, device="cuda")
    assert lib.quantize_device_padded(d, rows, cols, Kp, packed, scales, tiled) == lib.OK
    torch.cuda.synchronize()
    p, s = packed.cpu().numpy(), scales.cpu().numpy()
    assert np.array_equal(p[:, :cols * 3 // 4], host.packed_data)
    assert not p[:, cols * 3 // 4:].any()
    want = lib.pad_scales_k(host.scales, rows, cols)
    if tiled:
        assert np.array_equal(s, lib.preprocess_scale(want, rows, Kp))
    else:
        assert np.array_equal(s.reshape(rows, Kp // 32), want)


@pytest.mark.parametrize("M,N,K", [(512, 768, 1952), (1024, 512, 8192)])
def test_activation_path_on_device(lib, oracle, M, N, K):
    """The FFN step on the device: FP32 activations -> quantize_device_padded (rows of kpad(K)
    codes, GEMM-tiled scales) -> GEMM, with no host round trip; equals the oracle GEMM of the
    host quantiser's output (A zero-padded to kpad(K))."""
    from gpu_helpers import check
    from mxfp6_b200.synth import make_operands
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    Kp = lib.kpad(K)
    b = make_operands(128, N, K, kind="normal", seed=5, sigma=(1.0, 0.02))
    d_x = torch.from_numpy(x).cuda()
    a_packed = torch.empty((M, Kp * 3 // 4), dtype=torch.uint8, device="cuda")
    a_scales = torch.empty(lib.tiled_scale_bytes(M, Kp), dtype=torch.uint8, device="cuda")
    assert lib.quantize_device_padded(d_x, M, K, Kp, a_packed, a_scales, True) == lib.OK
    Bt = torch.from_numpy(b.Bt).cuda()
    sB = torch.from_numpy(lib.preprocess_scale(b.sB, N, Kp)).cuda()
    D = torch.empty((M, N), dtype=torch.float32, device="cuda")
    wsb = lib.gemm_workspace_size(M, N, Kp, lib.OutType.F32)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda") if wsb else None
    lib.gemm(lib.OutType.F32, M, N, Kp, a_packed, Bt, a_scales, sB, D, Kp * 3 // 4, Kp * 3 // 4, ws, wsb)
    assert lib.last_error() == lib.OK
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    host = lib.quantize_to_mxfp6(x)
    A_pad = np.zeros((M, Kp * 3 // 4), np.uint8)
    A_pad[:, :K * 3 // 4] = host.packed_data
    sA_pad = lib.pad_scales_k(host.scales, M, K)
    assert np.array_equal(a_packed.cpu().numpy(), A_pad)
    check(D.cpu(), oracle.gemm(A_pad, sA_pad, b.Bt, b.sB, Kp), lib.OutType.F32, oracle, label=f"ffn {M}x{N}x{K}")
