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
