"""GPU parity: the sm_100a kernels through the C ABI against the CPU oracle.

Cases mirror the reference's correctness list (tests/test_gemm.cpp:402-442 of eeezio/mxfp6-gemm)
re-expressed for the B200 routes, for every output type, plus the BASELINE configurations
(full-size, checked on 256 sampled full rows, all of K and N), the column shards of config 5
against the unsplit result, determinism, poisoned outputs and
the split-K workspace contract.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

OUTS = ["F32", "F16", "BF16"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def _setup(M, N, K, kind="uniform", seed=None, **kw):
    from mxfp6_b200.synth import make_operands
    from gpu_helpers import DeviceOperands
    seed = seed if seed is not None else M * 3 + N * 7 + K
    ops = make_operands(M, N, K, kind=kind, seed=seed, **kw)
    return ops, DeviceOperands(ops)


def _ref(oracle, ops, rows=None):
    return oracle.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp, rows=rows)


def test_probe_tma_fp6_unpack_layout():
    """Pins the 16U6 unpack: 16 packed codes (12 bytes) per 16-byte shared-memory slot, in the
    reference's packing order, 128-byte swizzle by row, and the byte count the load reports
    (96 per 128-code row: the mbarrier armed with exactly that count completes). The probe is a
    test-only library (tests/probe), not part of libmxfp6gemm.so."""
    import ctypes
    import os
    so = os.path.join(os.path.dirname(os.path.abspath(__file__)), "probe", "libmxfp6probe.so")
    if not os.path.exists(so):
        raise FileNotFoundError(f"{so} missing: run `make -C tests/probe` (or __graft_entry__.build())")
    probe = ctypes.CDLL(so).mxfp6_probe_tma_fp6
    probe.restype = ctypes.c_int
    probe.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    rows, Kp = 128, 128
    rng = np.random.default_rng(5)
    src = rng.integers(0, 256, (rows, 96), dtype=np.uint8)
    dsrc = torch.from_numpy(src).cuda()
    for swz in (0, 1):
        out = torch.zeros(rows * 128 + 16, dtype=torch.uint8, device="cuda")
        assert probe(dsrc.data_ptr(), rows, Kp, 96, swz, out.data_ptr()) == 0
        torch.cuda.synchronize()
        o = out.cpu().numpy()
        flag = int(o[rows * 128:rows * 128 + 4].view(np.int32)[0])
        assert flag == 1, f"swizzle={swz}: the barrier armed with {rows * 96} bytes did not complete"
        dump = o[:rows * 128].reshape(rows, 128)
        for r in range(rows):
            for j in range(8):
                pos = (j ^ (r % 8)) if swz else j
                slot = dump[r, 16 * pos:16 * pos + 12]
                assert np.array_equal(slot, src[r, 12 * j:12 * j + 12]), f"swizzle={swz} row {r} slot {j}"


def test_cfg1_256x256x512_fp32(lib, oracle):
    """uniform codes over all 64 E2M3 values, exponents in [120, 134]."""
    from gpu_helpers import check, run_gemm
    ops, dev = _setup(256, 256, 512, kind="codes", seed=1, exp_range=(120, 134))
    D = run_gemm(dev, lib.OutType.F32)
    check(D, _ref(oracle, ops), lib.OutType.F32, oracle, label="cfg1")


@pytest.mark.parametrize("ot", OUTS)
@pytest.mark.parametrize("M,N,K", [(512, 512, 768), (768, 1280, 960), (4096, 4096, 768)])
def test_reference_verify_cases(lib, oracle, ot, M, N, K):
    from gpu_helpers import check, run_gemm
    ops, dev = _setup(M, N, K)
    D = run_gemm(dev, lib.OutType[ot])
    check(D, _ref(oracle, ops), lib.OutType[ot], oracle, label=f"{M}x{N}x{K}")


@pytest.mark.parametrize("ot", OUTS)
@pytest.mark.parametrize("M,N,K,MT,NT", [
    (256, 256, 768, 128, 128), (384, 512, 1536, 128, 128), (256, 384, 768, 128, 256), (384, 768, 960, 128, 256),
    (1280, 1152, 384, 128, 256), (128, 128, 128, 128, 128), (128, 256, 128, 128, 256),
    (256, 256, 768, 256, 256), (512, 512, 1536, 256, 256), (384, 640, 960, 256, 256), (128, 128, 128, 256, 256),
    (1280, 1152, 384, 256, 256), (2304, 2560, 1024, 256, 256)])
def test_forced_tiles(lib, oracle, ot, M, N, K, MT, NT):
    """Every tile on small shapes (reference: verify_128x128 / verify_128x384), including
    partial tiles (M % 256 == 128 or N % 256 == 128: zero-filled loads, masked stores), a single
    K slab, and more tiles than CTA pairs (persistent loop with both accumulator buffers)."""
    from gpu_helpers import check, run_gemm
    ops, dev = _setup(M, N, K)
    D = run_gemm(dev, lib.OutType[ot], force=(MT, NT, 1))
    check(D, _ref(oracle, ops), lib.OutType[ot], oracle, label=f"{M}x{N}x{K} {MT}x{NT}")


@pytest.mark.parametrize("ot", OUTS)
@pytest.mark.parametrize("M,N,K,MT,NT,S", [(2048, 1024, 12288, 128, 256, 4), (2048, 1024, 3808, 128, 256, 2),
                                           (2048, 1024, 6400, 128, 256, 3), (256, 384, 4096, 128, 128, 5),
                                           (512, 640, 1920, 128, 256, 7), (2048, 1024, 12288, 256, 256, 4),
                                           (2048, 1024, 6400, 256, 256, 3), (384, 640, 4096, 256, 256, 5)])
def test_forced_splits(lib, oracle, ot, M, N, K, MT, NT, S):
    """Split-K with even and uneven segments (reference: verify_compact split cases) and the
    deterministic FP32 reduce, for every output type."""
    from gpu_helpers import check, run_gemm, sample_rows
    ops, dev = _setup(M, N, K)
    D = run_gemm(dev, lib.OutType[ot], force=(MT, NT, S))
    rows = sample_rows(M, 96) if M * N * ops.Kp > 2**31 else None
    check(D, _ref(oracle, ops, rows), lib.OutType[ot], oracle, rows=rows, label=f"{M}x{N}x{K} S={S}")


@pytest.mark.parametrize("ot", OUTS)
@pytest.mark.parametrize("M,N,K", [(2304, 2560, 1024), (2432, 2688, 256), (4096, 3584, 1024), (2432, 2688, 2048),
                                   (18944, 256, 512)])
def test_forced_stream_k(lib, oracle, ot, M, N, K):
    """The CTA pair's stream-K tail: 90, 110 and 224 tiles on 74 pairs, so each pair's K-slab
    range starts and ends inside tiles and hands accumulators on (at K = 256, every two or three
    slabs), partial M and N edge tiles, and 74 tiles (whole waves: no stream-K). Results match
    the oracle and are bit for bit those of the whole-tile schedule."""
    from gpu_helpers import check, run_gemm, sample_rows
    ops, dev = _setup(M, N, K)
    o = lib.OutType[ot]
    whole = run_gemm(dev, o, force=(256, 256, 1))
    D = run_gemm(dev, o, force=(256, 256, 1, 1))
    bits = torch.int32 if o == lib.OutType.F32 else torch.int16
    assert torch.equal(D.view(bits), whole.view(bits))
    rows = sample_rows(M, 128) if M * N * ops.Kp > 2**31 else None
    check(D, _ref(oracle, ops, rows), o, oracle, rows=rows, label=f"{M}x{N}x{K} stream-K")


@pytest.mark.parametrize("M,N,K,n,ot", [(2048, 1024, 24576, 1, "F16"), (2048, 1024, 24576, 3, "BF16"),
                                         (1024, 1024, 32768, 2, "F16"), (768, 1280, 12288, 1, "F32"),
                                         (2304, 1152, 8192, 2, "BF16"), (2304, 1152, 8192, 3, "F32")])
def test_forced_banded_split(lib, oracle, M, N, K, n, ot):
    """The CTA pair's banded split: fewer tiles than pairs (32, 16, 15 and 45; L = 2, 4, 4 and 1
    long bands per tile, partial M and N edge tiles), the first pairs take one long K band each
    and the rest share `n` short bands; the partials are reduced in band order. Matches the
    oracle and is bitwise repeatable."""
    from gpu_helpers import check, run_gemm, sample_rows
    ops, dev = _setup(M, N, K)
    o = lib.OutType[ot]
    D = run_gemm(dev, o, force=(256, 256, n, 2))
    again = run_gemm(dev, o, force=(256, 256, n, 2))
    bits = torch.int32 if o == lib.OutType.F32 else torch.int16
    assert torch.equal(D.view(bits), again.view(bits))
    rows = sample_rows(M, 96) if M * N * ops.Kp > 2**31 else None
    check(D, _ref(oracle, ops, rows), o, oracle, rows=rows, label=f"{M}x{N}x{K} banded n={n}")


def test_stream_k_repeated_launches_use_fresh_flags(lib):
    """Hand-off flags are tagged per launch and never cleared: back-to-back launches on one
    workspace, and a launch after the workspace was filled with stale data, stay bit-identical."""
    from gpu_helpers import TORCH_OUT
    ops, dev = _setup(2304, 2560, 512, kind="codes", seed=3)
    o = lib.OutType.BF16
    wsb = lib.stream_k_bytes()
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    outs = []
    for fill in (None, None, 0xFF, 0x00):
        if fill is not None:
            ws.fill_(fill)
        D = torch.empty((ops.M, ops.N), dtype=TORCH_OUT[o], device="cuda")
        lib.gemm_force_route(o, ops.M, ops.N, ops.Kp, 256, 256, 1, 1, dev.A, dev.Bt, dev.sA, dev.sB, D,
                             ops.row_bytes, ops.row_bytes, ws, wsb)
        assert lib.last_error() == lib.OK
        outs.append(D)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    for D in outs[1:]:
        assert torch.equal(D.view(torch.int16), outs[0].view(torch.int16))


@pytest.mark.parametrize("M,N,K", [(128, 384, 3072), (256, 384, 32768), (512, 640, 960), (256, 1408, 384),
                                   (2048, 1024, 12288)])
def test_routed_shapes(lib, oracle, M, N, K):
    """Routed (not forced) shapes from the reference's list, with and without a workspace."""
    from gpu_helpers import check, run_gemm, sample_rows
    ops, dev = _setup(M, N, K)
    rows = sample_rows(M, 64) if M * N * ops.Kp > 2**31 else None
    ref = _ref(oracle, ops, rows)
    for ws_mode in ("sized", "none"):
        D = run_gemm(dev, lib.OutType.F32, ws_mode=ws_mode)
        check(D, ref, lib.OutType.F32, oracle, rows=rows, label=f"{M}x{N}x{K} ws={ws_mode}")


def test_deterministic_and_split_invariant_bits(lib):
    """Two runs give identical bits, with and without split-K."""
    from gpu_helpers import run_gemm
    ops, dev = _setup(1024, 768, 4096, kind="codes", seed=9)
    for force in ((128, 256, 1), (128, 256, 3), (128, 128, 4), (256, 256, 1), (256, 256, 3)):
        a = run_gemm(dev, lib.OutType.F32, force=force)
        b = run_gemm(dev, lib.OutType.F32, force=force)
        assert torch.equal(a.view(torch.int32), b.view(torch.int32)), force


def test_special_scales(lib, oracle):
    """Scale code 255 (NaN) poisons exactly its rows / columns; code 0 (2^-127) and large codes stay finite."""
    from gpu_helpers import DeviceOperands, check, run_gemm
    from mxfp6_b200.synth import make_operands
    ops = make_operands(256, 256, 512, kind="codes", seed=4, exp_range=(120, 134))
    ops.sA[3, 2] = 255
    ops.sB[17, 0] = 255
    ops.sA[10, :] = 0
    ops.sB[40, :] = 160
    D = run_gemm(DeviceOperands(ops), lib.OutType.F32)
    ref = _ref(oracle, ops)
    check(D, ref, lib.OutType.F32, oracle, label="special scales")
    g = D.numpy()
    assert np.isnan(g[3]).all() and np.isnan(g[:, 17]).all()


def test_row_permutation_and_scale_doubling(lib):
    """Size-independent properties on a full-size shape: bumping every A scale exponent by one
    doubles D exactly, and permuting A's rows permutes D's rows bit for bit."""
    from gpu_helpers import DeviceOperands, run_gemm
    from mxfp6_b200.synth import make_operands
    ops = make_operands(2048, 2048, 4096, kind="codes", seed=12, exp_range=(118, 126))
    D0 = run_gemm(DeviceOperands(ops), lib.OutType.F32)
    ops.sA = ops.sA + 1
    D1 = run_gemm(DeviceOperands(ops), lib.OutType.F32)
    assert torch.equal(D1, D0 * 2)
    ops.sA = ops.sA - 1
    perm = np.random.default_rng(1).permutation(2048)
    ops.A, ops.sA = ops.A[perm].copy(), ops.sA[perm].copy()
    D2 = run_gemm(DeviceOperands(ops), lib.OutType.F32)
    assert torch.equal(D2.view(torch.int32), D0[torch.from_numpy(perm)].view(torch.int32))


# Rows of the full-size configs compared with the oracle (all of N, all of K): the bar is the
# full matrix or a fixed subset of at least 256 full rows, including both ends and tile edges.
PARITY_ROWS = 256

_CFG5 = {}


def _cfg5_operands():
    """BASELINE config 5 (seeded, quantised on the host), shared by the tests that need it."""
    if "ops" not in _CFG5:
        _CFG5["ops"], _CFG5["dev"] = _setup(4096, 28672, 8192, kind="normal", seed=2026)
    return _CFG5["ops"], _CFG5["dev"]


@pytest.mark.parametrize("cfg", ["cfg2_square_f16_inrange", "cfg2_square_f16_overflow", "cfg3_narrow_deepk_f16",
                                 "cfg3_narrow_deepk_f16_overflow", "cfg4_wide_bf16", "cfg5_ffn_bf16"])
def test_baseline_configs_sampled(lib, oracle, cfg):
    """BASELINE configs 2-5 at full size; the oracle runs the full K and N on 256 sampled rows.
    The "overflow" cases keep BASELINE's exponent range [118, 136], where most FP16 outputs
    overflow: infinities must match the oracle's in sign (the in-range companions shift the
    exponents by -9 so that the ulp check has finite values to bite on)."""
    from gpu_helpers import check, run_gemm, sample_rows
    spec = {
        "cfg2_square_f16_inrange": (8192, 8192, 8192, "codes", (109, 127), lib.OutType.F16),
        "cfg2_square_f16_overflow": (8192, 8192, 8192, "codes", (118, 136), lib.OutType.F16),
        "cfg3_narrow_deepk_f16": (2048, 1024, 105728, "codes", (109, 127), lib.OutType.F16),
        "cfg3_narrow_deepk_f16_overflow": (2048, 1024, 105728, "codes", (118, 136), lib.OutType.F16),
        "cfg4_wide_bf16": (2048, 6144, 16128, "codes", (118, 136), lib.OutType.BF16),
        "cfg5_ffn_bf16": (4096, 28672, 8192, "normal", None, lib.OutType.BF16),
    }[cfg]
    M, N, K, kind, er, ot = spec
    kw = {"exp_range": er} if er else {}
    ops, dev = _cfg5_operands() if cfg.startswith("cfg5") else _setup(M, N, K, kind=kind, seed=2026, **kw)
    rows = sample_rows(M, PARITY_ROWS)
    D = run_gemm(dev, ot)
    ref = _ref(oracle, ops, rows)
    check(D, ref, ot, oracle, rows=rows, label=cfg)
    if cfg.endswith("overflow"):
        assert (np.abs(ref) > 65504.0).mean() > 0.5  # most outputs do overflow FP16


@pytest.mark.parametrize("g", [2, 4, 8])
def test_cfg5_column_shards_equal_unsplit_D(lib, g):
    """Column-parallel sharding of BASELINE config 5 over g GPUs, run shard by shard on one
    device: shard r holds all of A and B^T rows [r*N/g, (r+1)*N/g) with their scale atoms, and
    the concatenation of the shards' D is the unsplit D bit for bit (no K split on either side,
    so every element sums the same products in the same order)."""
    ops, dev = _cfg5_operands()
    M, N, Kp, rb = ops.M, ops.N, ops.Kp, ops.row_bytes
    full_route = lib.route(lib.OutType.BF16, M, N, Kp)
    D_full = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    lib.gemm(lib.OutType.BF16, M, N, Kp, dev.A, dev.Bt, dev.sA, dev.sB, D_full, rb, rb)
    assert lib.last_error() == lib.OK
    Ng = N // g
    atoms = Kp // 128 * 512  # tiled scale bytes per 128 rows of B^T
    D_cat = torch.empty_like(D_full)
    for r in range(g):
        route = lib.route(lib.OutType.BF16, M, Ng, Kp)
        assert route["splits"] == 1 and full_route["splits"] == 1, (route, full_route)
        D_r = torch.full((M, Ng), float("nan"), dtype=torch.bfloat16, device="cuda")
        lib.gemm(lib.OutType.BF16, M, Ng, Kp, dev.A, dev.Bt[r * Ng:(r + 1) * Ng], dev.sA,
                 dev.sB[r * Ng // 128 * atoms:(r + 1) * Ng // 128 * atoms], D_r, rb, rb)
        assert lib.last_error() == lib.OK
        D_cat[:, r * Ng:(r + 1) * Ng] = D_r
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    assert torch.equal(D_cat.view(torch.int16), D_full.view(torch.int16))


@pytest.mark.parametrize("M,N,K", [(2048, 1024, 105728), (1024, 512, 105728), (256, 384, 32768)])
def test_long_k_fp32_within_tolerance(lib, oracle, M, N, K):
    """FP32 output at long K: the route keeps split segments short enough (FP32_SEGMENT_K) that
    the result stays within 1e-5 (norm-wise) of the sequential FP32 oracle."""
    from gpu_helpers import check, run_gemm, sample_rows
    ops, dev = _setup(M, N, K, kind="codes", seed=5, exp_range=(109, 127))
    rows = sample_rows(M, PARITY_ROWS)
    D = run_gemm(dev, lib.OutType.F32)
    check(D, _ref(oracle, ops, rows), lib.OutType.F32, oracle, rows=rows, label=f"{M}x{N}x{K} fp32")


def test_small_workspace_falls_back_unsplit(lib, oracle, capfd):
    """A shape that wants split-K but gets too small a workspace runs unsplit, warns, and is right."""
    from gpu_helpers import check, run_gemm, sample_rows
    M, N, K = 2048, 1024, 105728
    assert lib.gemm_workspace_size(M, N, K) > 0
    ops, dev = _setup(M, N, K)
    D = run_gemm(dev, lib.OutType.F32, ws_mode="none")
    assert "split-K skipped" in capfd.readouterr().err
    rows = sample_rows(M, 32)
    check(D, _ref(oracle, ops, rows), lib.OutType.F32, oracle, rows=rows, label="ws fallback")


def test_launch_counter_and_stream(lib, oracle):
    from gpu_helpers import check, run_gemm
    ops, dev = _setup(256, 512, 1024)
    n0 = lib.launch_count()
    s = torch.cuda.Stream()
    D = run_gemm(dev, lib.OutType.F16, stream=s)
    assert lib.launch_count() > n0
    check(D, _ref(oracle, ops), lib.OutType.F16, oracle, label="stream")


@pytest.mark.parametrize("MT,NT", [(256, 256), (128, 256)])
def test_output_only_16_byte_aligned(lib, oracle, MT, NT):
    """D at a 16-byte (not 32-byte) aligned address takes the 128-bit store path."""
    from gpu_helpers import check
    ops, dev = _setup(256, 512, 1024)
    o = ops
    raw = torch.full((o.M * o.N * 2 + 64,), 0x5A, dtype=torch.uint8, device="cuda")
    base = raw.data_ptr()
    off = (32 - base % 32) % 32 + 16
    D = raw[off:off + o.M * o.N * 2].view(torch.float16).view(o.M, o.N)
    assert D.data_ptr() % 32 == 16
    lib.gemm_force_tile(lib.OutType.F16, o.M, o.N, o.Kp, MT, NT, 1, dev.A, dev.Bt, dev.sA, dev.sB, D, o.row_bytes,
                        o.row_bytes)
    assert lib.last_error() == lib.OK
    assert lib.device_status() == 0
    check(D.cpu(), _ref(oracle, ops), lib.OutType.F16, oracle, label="16-byte aligned D")
