"""Compact A on the GPU: the reference's "pad-B-only / compact-A" recipe
(tests/test_gemm.cpp:131-201 and include/mxfp6/preprocess.hpp:12-38 of eeezio/mxfp6-gemm).

A keeps its natural row stride 3K/4 with K % 128 != 0; B and both scale sets are padded to
Kp = kpad(K), A's scale tail with the finite code 127 (pad_scales_k). The tensor-memory
accelerator cannot address such a stride. gemm() either re-pads A first (into the caller's
workspace when it was sized for that, else into the library's re-pad scratch) and runs the
tensor-load kernel, or, with the scratch switched off, the kernels load A with their loader
warps. Checked against the oracle on the zero-padded A (the reference's own comparison), and
bit for bit against the tensor-load path on the padded A: every way feeds the tensor cores the
same shared-memory image, so the sums must agree exactly.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def _compact_buffer(ops, poison=0x5A, offset=0, stride=None):
    """A rows of 3K/4 bytes (or `stride`) in a poisoned buffer with the reference's end pad,
    starting `offset` bytes into the allocation. Returns (tensor view, stride)."""
    import mxfp6_b200 as lib
    stride = stride or ops.K * 3 // 4
    total = offset + ops.M * stride + lib.a_compact_end_pad(ops.K)
    buf = torch.full((total,), poison, dtype=torch.uint8, device="cuda")
    rows = np.full((ops.M, stride), poison, np.uint8)
    keep = min(stride, ops.row_bytes)  # the compact row, or the padded row with its zero K tail
    rows[:, :keep] = ops.A[:, :keep]
    buf[offset:offset + ops.M * stride] = torch.from_numpy(rows.reshape(-1)).cuda()
    return buf[offset:], stride


def _run(lib, ops, dA, a_stride, ot, dev, force=None, scratch=True):
    """One call with the workspace the reference's three-argument query gives (or a forced
    route); `scratch` False keeps the library from re-padding A into its own scratch, so the
    loader warps read it in place."""
    prev = lib.set_repad_scratch(1 if scratch else 0)
    try:
        return _run_once(lib, ops, dA, a_stride, ot, dev, force)
    finally:
        lib.set_repad_scratch(prev)


def _run_once(lib, ops, dA, a_stride, ot, dev, force):
    D = torch.empty((ops.M, ops.N), dtype={0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[int(ot)],
                    device="cuda")
    D.view(torch.uint8).fill_(0x5A)
    if force is None:
        wsb = lib.gemm_workspace_size(ops.M, ops.N, ops.Kp)
    else:
        wsb = force[2] * ops.M * ops.N * 4 if force[2] > 1 else 0
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda") if wsb else None
    if force is None:
        lib.gemm(ot, ops.M, ops.N, ops.Kp, dA, dev.Bt, dev.sA, dev.sB, D, a_stride, ops.row_bytes, ws, wsb)
    else:
        lib.gemm_force_tile(ot, ops.M, ops.N, ops.Kp, force[0], force[1], force[2], dA, dev.Bt, dev.sA, dev.sB,
                            D, a_stride, ops.row_bytes, ws, wsb)
    assert lib.last_error() == lib.OK, lib.last_error_string()
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    return D.cpu()


def _setup(M, N, K, kind="uniform"):
    from mxfp6_b200.synth import make_operands
    from gpu_helpers import DeviceOperands
    ops = make_operands(M, N, K, kind=kind, seed=M * 5 + N * 11 + K * 2)
    return ops, DeviceOperands(ops)


# The reference's verify_compact list (tests/test_gemm.cpp:405-413), FP32 output, routed.
@pytest.mark.parametrize("M,N,K", [(4096, 4096, 224), (768, 1280, 224), (512, 512, 160), (2048, 1024, 12288),
                                   (2048, 1024, 3808), (2048, 1024, 6304)])
def test_reference_compact_cases(lib, oracle, M, N, K):
    from gpu_helpers import check, sample_rows
    ops, dev = _setup(M, N, K)
    dA, stride = _compact_buffer(ops)
    D = _run(lib, ops, dA, stride, lib.OutType.F32, dev)
    assert not torch.isnan(D).any()
    assert torch.equal(D, _run(lib, ops, dA, stride, lib.OutType.F32, dev, scratch=False))
    rows = sample_rows(M, 96) if M * N * ops.Kp > 2**31 else None
    ref = oracle.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp, rows=rows)
    check(D, ref, lib.OutType.F32, oracle, rows=rows, label=f"compact {M}x{N}x{K}")


@pytest.mark.parametrize("ot", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("MT,NT,S", [(128, 128, 1), (128, 256, 1), (128, 256, 3), (256, 256, 1), (256, 256, 4)])
def test_compact_every_route_bitwise(lib, oracle, ot, MT, NT, S):
    """Every tile and split on compact A, 1152 rows (a half-empty last CTA pair): equal to the
    oracle within tolerance and bit-identical to the same route on the padded A."""
    from gpu_helpers import check
    M, N, K = 1152, 1280, 2144
    ops, dev = _setup(M, N, K, kind="codes")
    dA, stride = _compact_buffer(ops)
    D = _run(lib, ops, dA, stride, lib.OutType[ot], dev, force=(MT, NT, S))
    D_pad = _run(lib, ops, dev.A, ops.row_bytes, lib.OutType[ot], dev, force=(MT, NT, S))
    assert torch.equal(D.view(torch.uint8), D_pad.view(torch.uint8))
    check(D, oracle.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp), lib.OutType[ot], oracle,
          label=f"compact {MT}x{NT} S={S}")


@pytest.mark.parametrize("MT,NT,S", [(128, 128, 1), (128, 256, 3), (256, 256, 1), (256, 256, 4)])
def test_unaligned_base_every_route_bitwise(lib, MT, NT, S):
    """A base only 4-byte aligned (the loader warps' copies need nothing more) must match the
    tensor-load path bit for bit on every tile."""
    M, N, K = 1152, 1280, 2144
    ops, dev = _setup(M, N, K, kind="codes")
    dA, stride = _compact_buffer(ops, offset=4)
    D = _run(lib, ops, dA, stride, lib.OutType.F32, dev, force=(MT, NT, S))
    D_pad = _run(lib, ops, dev.A, ops.row_bytes, lib.OutType.F32, dev, force=(MT, NT, S))
    assert torch.equal(D, D_pad)


@pytest.mark.parametrize("offset,extra", [(4, 0), (0, 8), (12, 4), (0, 4), (8, 0), (0, 16)])
def test_unaligned_base_and_stride(lib, oracle, offset, extra):
    """Bases and strides off the tensor-load path's 32-byte rules: compact or padded strides that
    are multiples of 8 or only of 4, and bases 4, 8 or 12 bytes past a 16-byte boundary. All
    are re-padded by the library (M*N*Kp is above its scratch threshold) or, with the scratch
    off, read by the loader warps, and must equal the tensor-load path on the padded A."""
    M, N, K = 1024, 1280, 1952
    ops, dev = _setup(M, N, K, kind="codes")
    stride = ops.row_bytes + extra if extra else ops.K * 3 // 4
    dA, stride = _compact_buffer(ops, offset=offset, stride=stride)
    D = _run(lib, ops, dA, stride, lib.OutType.F32, dev)
    D_in_place = _run(lib, ops, dA, stride, lib.OutType.F32, dev, scratch=False)
    D_pad = _run(lib, ops, dev.A, ops.row_bytes, lib.OutType.F32, dev)
    assert torch.equal(D, D_pad) and torch.equal(D_in_place, D_pad)


def test_compact_large_bitwise(lib):
    """Full-size compact A (8192 x 8192 x 8160, K % 128 = 96) on the pair route with its stream-K
    tail: bit-identical to the padded tensor-load path (a size-independent check; the oracle is
    too slow here)."""
    M, N, K = 8192, 8192, 8160
    ops, dev = _setup(M, N, K, kind="codes")
    dA, stride = _compact_buffer(ops)
    D = _run(lib, ops, dA, stride, lib.OutType.F16, dev)
    D_in_place = _run(lib, ops, dA, stride, lib.OutType.F16, dev, scratch=False)
    D_pad = _run(lib, ops, dev.A, ops.row_bytes, lib.OutType.F16, dev)
    assert torch.equal(D.view(torch.int16), D_pad.view(torch.int16))
    assert torch.equal(D_in_place.view(torch.int16), D_pad.view(torch.int16))


def test_device_repad_then_tensor_path(lib):
    """repad_rows_device turns compact rows into padded ones on the device (zero tail); the GEMM
    on the result takes the tensor-load path and equals the compact-A GEMM bit for bit."""
    M, N, K = 1024, 768, 1952
    ops, dev = _setup(M, N, K, kind="codes")
    dA, stride = _compact_buffer(ops)
    padded = torch.full((M, ops.row_bytes), 0x77, dtype=torch.uint8, device="cuda")
    assert lib.repad_rows_device(dA, M, stride, stride, padded, ops.row_bytes) == lib.OK
    torch.cuda.synchronize()
    assert torch.equal(padded.cpu(), torch.from_numpy(ops.A))
    D_c = _run(lib, ops, dA, stride, lib.OutType.BF16, dev)
    D_p = _run(lib, ops, padded, ops.row_bytes, lib.OutType.BF16, dev)
    assert torch.equal(D_c.view(torch.int16), D_p.view(torch.int16))


@pytest.mark.parametrize("ot", ["F32", "BF16"])
@pytest.mark.parametrize("M,N,K", [(4096, 4096, 224), (2048, 1024, 3808), (1152, 1280, 2144)])
def test_compact_with_a_aware_workspace(lib, ot, M, N, K):
    """With a workspace sized by gemm_workspace_size(M, N, Kp, A_row_bytes), gemm() re-pads the
    compact A into the workspace (one extra launch) and runs the tensor-load kernel: the result
    is bit-identical to the in-place loader path and to the padded A, and A is left untouched."""
    ops, dev = _setup(M, N, K, kind="codes")
    dA, stride = _compact_buffer(ops)
    before = dA.clone()
    o = lib.OutType[ot]
    wsb = lib.gemm_workspace_size_a(M, N, ops.Kp, stride)
    assert wsb >= M * ops.row_bytes
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    D = torch.empty((M, N), dtype={0: torch.float32, 2: torch.bfloat16}[int(o)], device="cuda")
    n0 = lib.launch_count()
    lib.gemm(o, M, N, ops.Kp, dA, dev.Bt, dev.sA, dev.sB, D, stride, ops.row_bytes, ws, wsb)
    assert lib.last_error() == lib.OK, lib.last_error_string()
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    n_repad = lib.launch_count() - n0
    # workspace from the 3-argument query, scratch off: the loader warps
    D_in_place = _run(lib, ops, dA, stride, o, dev, scratch=False)
    n1 = lib.launch_count()
    _run(lib, ops, dA, stride, o, dev, scratch=False)
    n_in_place = lib.launch_count() - n1
    # the same workspace with the library's scratch: re-pad, then the tensor load
    n2 = lib.launch_count()
    D_scratch = _run(lib, ops, dA, stride, o, dev)
    n_scratch = lib.launch_count() - n2
    D_pad = _run(lib, ops, dev.A, ops.row_bytes, o, dev)
    assert n_repad == n_in_place + 1 and n_scratch == n_repad
    bits = (lambda t: t.view(torch.int32)) if o == lib.OutType.F32 else (lambda t: t.view(torch.int16))
    assert torch.equal(bits(D.cpu()), bits(D_pad)) and torch.equal(bits(D_in_place), bits(D_pad))
    assert torch.equal(bits(D_scratch), bits(D_pad))
    assert torch.equal(dA, before)


def test_repad_scratch_pool(lib):
    """The library's re-pad scratch: a compact A with the reference-sized workspace (none, for this
    unsplit shape) is re-padded into memory the library takes from its own pool in stream order,
    which keeps it for later calls; calls on two streams at once each get their own; a call
    captured in a CUDA graph takes no scratch (it reads A in place) and replays to the same bits;
    releasing the pool returns its memory."""
    M, N, K = 1024, 1536, 3040
    ops, dev = _setup(M, N, K, kind="codes")
    dA, stride = _compact_buffer(ops)
    o = lib.OutType.BF16
    assert lib.gemm_workspace_size(M, N, ops.Kp) == 0 and lib.route(int(o), M, N, ops.Kp)["splits"] == 1
    assert lib.set_repad_scratch(1) == 1  # on by default
    assert lib.release_repad_scratch() == lib.OK
    D_pad = _run(lib, ops, dev.A, ops.row_bytes, o, dev)
    want = D_pad.view(torch.int16)

    def call(D, stream=None):
        lib.gemm(o, M, N, ops.Kp, dA, dev.Bt, dev.sA, dev.sB, D, stride, ops.row_bytes, None, 0, stream=stream)
        assert lib.last_error() == lib.OK, lib.last_error_string()

    D = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    n0 = lib.launch_count()
    call(D)
    n_scratch = lib.launch_count() - n0
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    assert torch.equal(D.cpu().view(torch.int16), want)
    held = lib.repad_scratch_bytes()
    assert held >= M * ops.row_bytes, held

    # two streams at once, several calls each
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = [torch.empty((M, N), dtype=torch.bfloat16, device="cuda") for _ in range(4)]
    s1.wait_stream(torch.cuda.current_stream())
    s2.wait_stream(torch.cuda.current_stream())
    for i, Dk in enumerate(outs):
        st = s1 if i % 2 == 0 else s2
        with torch.cuda.stream(st):
            call(Dk, stream=st)
    torch.cuda.synchronize()
    assert lib.device_status() == 0
    for Dk in outs:
        assert torch.equal(Dk.cpu().view(torch.int16), want)

    # captured: no scratch, one launch fewer (no re-pad), same bits on replay
    gs = torch.cuda.Stream()
    Dg = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    gs.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    n1 = lib.launch_count()
    with torch.cuda.graph(g, stream=gs):
        call(Dg, stream=gs)
    assert lib.launch_count() - n1 == n_scratch - 1
    Dg.view(torch.uint8).fill_(0x5A)
    torch.cuda.synchronize()
    with torch.cuda.stream(gs):
        g.replay()
    gs.synchronize()
    assert lib.device_status() == 0
    assert torch.equal(Dg.cpu().view(torch.int16), want)
    del g

    assert lib.release_repad_scratch() == lib.OK
    assert lib.repad_scratch_bytes() == 0

    # below the scratch threshold (M*N*Kp < 2^31) the loader warps read A in place: no re-pad
    small, sdev = _setup(256, 256, 480, kind="codes")
    sA_c, sstride = _compact_buffer(small)
    counts = []
    for on in (True, False):
        n = lib.launch_count()
        Ds = _run(lib, small, sA_c, sstride, o, sdev, scratch=on)
        counts.append(lib.launch_count() - n)
    assert counts[0] == counts[1] and lib.repad_scratch_bytes() == 0
    assert torch.equal(Ds.view(torch.int16), _run(lib, small, sdev.A, small.row_bytes, o, sdev).view(torch.int16))
