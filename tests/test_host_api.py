"""Host-side checks that need no GPU: the C-ABI library loads and exports what include/*.h
declares, the host layout producers match the oracle and the reference's golden vectors, the
route table keeps the reference's coverage and workspace properties (tests/test_gemm.cpp:256-367
of eeezio/mxfp6-gemm), and invalid calls are rejected before any device work."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(mxfp6_\w+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 15
    so = ctypes.CDLL(lib.LIB_PATH)
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing


def test_k_tile_and_kpad(lib):
    assert lib.K_TILE == 128
    assert [lib.kpad(k) for k in (1, 128, 129, 224, 16128, 105728)] == [128, 128, 256, 256, 16128, 105728]


def test_quantize_matches_golden_and_oracle(lib, golden, oracle):
    q = lib.quantize_to_mxfp6(golden["quant_in"])
    assert np.array_equal(q.scales, golden["quant_scales"])
    assert np.array_equal(q.packed_data, golden["quant_packed"])
    rng = np.random.default_rng(2)
    m = (rng.standard_normal((333, 640)) * np.exp(rng.uniform(-20, 20, (333, 1)))).astype(np.float32)
    for threads in (1, 4, 0):
        q = lib.quantize_to_mxfp6(m, threads)
        p, s = oracle.quantize(m)
        assert np.array_equal(q.packed_data, p) and np.array_equal(q.scales, s)


def test_dequantize_matches_oracle(lib, oracle):
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, (64, 96), dtype=np.uint8)
    scales = rng.integers(100, 150, (64, 4), dtype=np.uint8)
    scales[0, 0] = 255
    q = lib.QuantizedMatrix(packed, scales, 64, 128)
    a = lib.dequantize_mxfp6(q)
    b = oracle.dequantize(packed, scales, 128)
    assert np.array_equal(np.isnan(a), np.isnan(b))
    assert np.array_equal(np.nan_to_num(a), np.nan_to_num(b))


def test_pack_unpack_roundtrip(lib):
    rng = np.random.default_rng(4)
    codes = rng.integers(0, 64, (7, 256), dtype=np.uint8)
    assert np.array_equal(lib.unpack_codes(lib.pack_codes(codes)), codes)


@pytest.mark.parametrize("rows,K", [(128, 128), (256, 512), (200, 384), (1, 128), (384, 1024)])
def test_scale_atom_layout(lib, rows, K):
    """Atom layout: raw (r, j) at atom (r/128)*(K/128) + j/4, byte (r%32)*16 + ((r%128)/32)*4 + j%4;
    rows past `rows` are filled with the finite code 127; untile inverts tile."""
    rng = np.random.default_rng(rows + K)
    raw = rng.integers(0, 256, (rows, K // 32), dtype=np.uint8)
    t = lib.preprocess_scale(raw, rows, K)
    assert t.size == lib.tiled_scale_bytes(rows, K) == ((rows + 127) // 128) * (K // 128) * 512
    for r in range(rows):
        for j in range(K // 32):
            off = ((r // 128) * (K // 128) + j // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + j % 4
            assert t[off] == raw[r, j]
    assert np.array_equal(lib.untile_scales(t, rows, K), raw)
    if rows % 128:
        filled = np.zeros(t.size, bool)
        for r in range(rows):
            for j in range(K // 32):
                filled[((r // 128) * (K // 128) + j // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + j % 4] = True
        assert (t[~filled] == 127).all()
    assert lib.tile_scale(t, 4, 2) is t


def test_preshuffle_is_identity(lib):
    rng = np.random.default_rng(5)
    q = lib.preprocess_B(rng.uniform(-1, 1, (256, 128)).astype(np.float32))
    assert q.rows == 128 and q.cols == 256
    assert lib.preshuffle_B(q) is q.packed_data


# ---- routing properties (reference: tests/test_gemm.cpp:319-365) ---------------------------------

SWEEP_K = [512, 4096, 16128, 32768, 40000, 105728]


def test_route_covers_every_shape(lib):
    """Every M, N multiple of 128 up to 16384 x 24576 routes to a tile that covers the output
    (the 256-wide tile covers N % 256 == 128 with a masked half tile); splits stay within K."""
    for K in SWEEP_K:
        Kp = lib.kpad(K)
        for M in range(128, 16385, 1024):
            for N in range(128, 24577, 640):
                t = lib.choose_tile(M, N, Kp)
                assert (t.MT, t.NT) in ((256, 256), (128, 256), (128, 128))
                assert M % 128 == 0 and N % 128 == 0  # every tile covers the rest by masking
                assert (t.MPW, t.NPW) == (t.MT // 32, t.NT // 32)
                ws = lib.gemm_workspace_size(M, N, Kp)
                need = 0
                for ot in (lib.OutType.F16, lib.OutType.F32):
                    r = lib.route(ot, M, N, Kp)
                    if ot == lib.OutType.F16:  # choose_tile reports the FP16/BF16 route
                        assert r["MT"] == t.MT and r["NT"] == t.NT
                    assert 1 <= r["splits"] <= Kp // 128
                    # the stream-K tail belongs to the CTA pair without a K split, on tiles that do
                    # not fill whole waves of 74 pairs (and fill at least one), where the idle part
                    # of the last wave is at least 35 slabs deep
                    tiles = -(-M // 256) * -(-N // 256)
                    assert r["stream_k"] == (r["MT"] == 256 and r["splits"] == 1 and tiles >= 74 and tiles % 74 != 0
                                             and (74 - tiles % 74) * (Kp // 128) >= 35 * 74)
                    b = (r["splits"] * M * N * 4 if r["splits"] > 1 else 0) + (lib.stream_k_bytes() if r["stream_k"] else 0)
                    need = max(need, b)
                assert ws == need


def test_route_examples(lib):
    # BASELINE shapes: the square and FFN shapes fill the machine unsplit; the FFN shape and its
    # column shards (1792 / 224 / 448 tiles on 74 pairs) and the wide shape run a stream-K tail,
    # whose hand-off area is their whole workspace; the narrow deep-K shape splits; tiny shapes
    # never split.
    assert lib.gemm_workspace_size(8192, 8192, 8192) == 0  # 1024 tiles: the last wave 62/74 full
    assert lib.gemm_workspace_size(4096, 28672, 8192) == lib.stream_k_bytes() == 74 * (256 * 256 * 4 + 16)
    for shape in [(4096, 28672, 8192), (4096, 3584, 8192), (4096, 7168, 8192), (2048, 6144, 16128)]:
        assert lib.route(lib.OutType.BF16, *shape)["stream_k"], shape
    assert not lib.route(lib.OutType.F16, 8192, 8192, 8192)["stream_k"]
    assert not lib.route(lib.OutType.F16, 2048, 1024, 105728)["stream_k"]  # split-K instead
    # 32 tiles on 74 CTA pairs with a deep K: two long bands per tile on 64 pairs, the rest of K on
    # the other 10 (FP32 keeps its short equal segments)
    r = lib.route(lib.OutType.F16, 2048, 1024, 105728)
    assert r["banded"] and r["MT"] == 256 and r["splits"] >= 3
    assert lib.gemm_workspace_size(2048, 1024, 105728, lib.OutType.F16) == r["splits"] * 2048 * 1024 * 4
    assert not lib.route(lib.OutType.F32, 2048, 1024, 105728)["banded"]
    # a shallow K: the tail would cost more than the last wave's idle slabs (4096^3: 32 slabs, 34/74)
    assert not lib.route(lib.OutType.F16, 4096, 4096, 4096)["stream_k"]
    assert lib.gemm_workspace_size(2048, 1024, 105728) > 0
    assert lib.gemm_workspace_size(256, 256, 512) == 0
    assert lib.gemm_workspace_size(128, 128, 128) == 0
    assert lib.choose_tile(8192, 8192, 8192).MT == 256  # CTA-pair tile on machine-filling shapes
    for shape in [(2048, 1024, 105728), (2048, 6144, 16128), (4096, 28672, 8192), (4096, 3584, 8192)]:
        assert lib.choose_tile(*shape).MT == 256, shape


@pytest.mark.parametrize("M,N,K,MT,NT,splits", [(2048, 1024, 12288, 256, 256, 2), (2048, 256, 4096, 128, 128, 3),
                                                 (2048, 256, 16128, 128, 256, 6), (2048, 512, 6144, 128, 128, 2)])
def test_deep_k_one_wave_shapes_split(lib, M, N, K, MT, NT, splits):
    """One wave of 128x128 tiles with a deep K runs faster split (measured back to back on B200:
    2048x1024x12288 39.1 us on one 128x128 wave, 31.9 us as a 2-way split on the CTA pair)."""
    r = lib.route(lib.OutType.F16, M, N, lib.kpad(K))
    assert (r["MT"], r["NT"], r["splits"]) == (MT, NT, splits), r
    assert lib.gemm_workspace_size(M, N, lib.kpad(K), lib.OutType.F16) == splits * M * N * 4


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 256, 512), (512, 512, 1024), (512, 256, 2048),
                                   (1024, 2048, 8192)])
def test_small_shapes_take_the_single_cta_kernel_unsplit(lib, M, N, K):
    """Where a launch's fixed cost dominates, the route avoids the CTA pair's start-up and the
    split-K reduce's extra launch (both measured slower on these shapes)."""
    t = lib.choose_tile(M, N, K)
    assert (t.MT, t.NT) == (128, 128)
    assert lib.gemm_workspace_size(M, N, K) == 0


def test_workspace_query_per_output_type(lib):
    """The type-free query covers every output type; FP32 splits long K into short segments."""
    for M, N, K in [(2048, 1024, 105728), (256, 384, 32768), (8192, 8192, 8192), (1024, 512, 105728)]:
        per = [lib.gemm_workspace_size(M, N, K, ot) for ot in lib.OutType]
        assert lib.gemm_workspace_size(M, N, K) == max(per)
    assert lib.gemm_workspace_size(2048, 1024, 105728, lib.OutType.F32) == 9 * 2048 * 1024 * 4
    assert lib.gemm_workspace_size(2048, 1024, 105728, lib.OutType.F16) < 9 * 2048 * 1024 * 4


def test_workspace_query_on_degenerate_shapes(lib):
    """Sub-tile shapes must not crash the query (reference: tests/test_gemm.cpp:362-365)."""
    for M, N, K in [(192, 256, 32832), (256, 192, 3072), (64, 64, 3072), (0, 128, 128), (128, 128, 0)]:
        lib.gemm_workspace_size(M, N, lib.kpad(K) if K else 0)
        lib.choose_tile(M, N, lib.kpad(K) if K else 0)


# ---- argument validation (no device work happens) --------------------------------------------------

@pytest.mark.parametrize("args,code", [
    (dict(M=100), "ERR_INVALID_SHAPE"),
    (dict(N=200), "ERR_INVALID_SHAPE"),
    (dict(Kp=192), "ERR_INVALID_SHAPE"),
    (dict(Kp=0), "ERR_INVALID_SHAPE"),
    (dict(Ar=90), "ERR_INVALID_STRIDE"),
    (dict(Br=112), "ERR_INVALID_STRIDE"),
    (dict(dA=0), "ERR_NULL_POINTER"),
    (dict(dD=0), "ERR_NULL_POINTER"),
    (dict(dA=0x1002), "ERR_MISALIGNED"),
    (dict(Kp=256, Ar=96, Br=192), "ERR_INVALID_STRIDE"),   # compact stride of K=128 < kpad^-1(256)
    (dict(Kp=256, Ar=190, Br=192), "ERR_INVALID_STRIDE"),  # not a multiple of 4
    (dict(dsB=0x1008), "ERR_MISALIGNED"),
    (dict(ot=7), "ERR_INVALID_OUT_TYPE"),
])
def test_invalid_arguments_rejected(lib, capfd, args, code):
    base = dict(ot=0, M=128, N=128, Kp=128, dA=0x1000, dB=0x2000, dsA=0x3000, dsB=0x4000, dD=0x5000,
                Ar=96, Br=96)
    base.update(args)
    lib.gemm(base["ot"], base["M"], base["N"], base["Kp"], base["dA"], base["dB"], base["dsA"], base["dsB"],
             base["dD"], base["Ar"], base["Br"])
    assert lib.last_error() == getattr(lib, code)
    assert "[mxfp6]" in capfd.readouterr().err


def test_forced_route_validation(lib, capfd):
    lib.gemm_force_tile(0, 128, 128, 128, 128, 192, 1, 0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 96, 96)
    assert lib.last_error() == lib.ERR_UNSUPPORTED
    lib.gemm_force_tile(0, 128, 128, 128, 256, 128, 1, 0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 96, 96)
    assert lib.last_error() == lib.ERR_UNSUPPORTED
    lib.gemm_force_tile(0, 128, 128, 512, 128, 128, 2, 0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 384, 384, None, 0)
    assert lib.last_error() == lib.ERR_WORKSPACE


def test_gather_validation(lib, capfd):
    """mxfp6_gemm_gather rejects bad destination lists before any device work."""
    args = dict(ot=1, M=128, N=128, Kp=128, dA=0x1000, dB=0x2000, dsA=0x3000, dsB=0x4000, Ar=96, Br=96)
    base = (args["ot"], args["M"], args["N"], args["Kp"], args["dA"], args["dB"], args["dsA"], args["dsB"])
    lib.gemm_gather(*base, [], 256, 0, 96, 96)
    assert lib.last_error() == lib.ERR_NULL_POINTER
    lib.gemm_gather(*base, [0x5000] * 9, 256, 0, 96, 96)
    assert lib.last_error() == lib.ERR_NULL_POINTER
    lib.gemm_gather(*base, [0x5000], 200, 128, 96, 96)          # ldd < col0 + N
    assert lib.last_error() == lib.ERR_INVALID_STRIDE
    lib.gemm_gather(*base, [0x5000], 260, 4, 96, 96)            # col0 * 2 bytes not 16-aligned
    assert lib.last_error() == lib.ERR_INVALID_STRIDE
    lib.gemm_gather(*base, [0x5000, 0x5008], 256, 0, 96, 96)    # second destination misaligned
    assert lib.last_error() == lib.ERR_MISALIGNED
    assert "[mxfp6]" in capfd.readouterr().err
