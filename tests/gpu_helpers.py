"""Device-side helpers for the GPU parity tests: upload synthetic operands, call the library
through its C ABI, and compare with the CPU oracle under the stated tolerances:

  FP32 out:       max|D - Dref| / max|Dref| <= 1e-5   (norm-wise: the reference's own sequential
                  FP32 sum differs from an exact sum by more than 1e-5 element-wise at large K)
  FP16/BF16 out:  every element within 1 ulp of round-to-nearest-even(Dref), or within the FP32
                  norm-wise bound plus one ulp (cancellation); infinities match in sign.
"""
from __future__ import annotations

import numpy as np
import torch

import mxfp6_b200 as lib
from mxfp6_b200.synth import Operands

FP32_TOL = 1e-5
TORCH_OUT = {lib.OutType.F32: torch.float32, lib.OutType.F16: torch.float16,
             lib.OutType.BF16: torch.bfloat16}


class DeviceOperands:
    def __init__(self, ops: Operands, device="cuda"):
        self.ops = ops
        self.A = torch.from_numpy(ops.A).to(device)
        self.Bt = torch.from_numpy(ops.Bt).to(device)
        self.sA = torch.from_numpy(lib.preprocess_scale(ops.sA, ops.M, ops.Kp)).to(device)
        self.sB = torch.from_numpy(lib.preprocess_scale(ops.sB, ops.N, ops.Kp)).to(device)


def run_gemm(dev: DeviceOperands, ot, ws_mode="sized", force=None, poison=True, stream=None):
    """Run the routed GEMM (or a forced route (MT, NT, splits[, stream_k])); returns D as a torch
    CPU tensor."""
    o = dev.ops
    D = torch.empty((o.M, o.N), dtype=TORCH_OUT[ot], device=dev.A.device)
    if poison:
        D.view(torch.uint8).fill_(0x5A)
    ws, wsb = None, 0
    if force is not None:
        MT, NT, S = force[:3]
        if S > 1:
            wsb = S * o.M * o.N * 4
        if len(force) > 3 and force[3] == 1:  # stream-K tail
            wsb = max(wsb, lib.stream_k_bytes())
        if len(force) > 3 and force[3] == 2:  # banded split: long bands plus `S` short bands
            wsb = max(wsb, (74 // max(1, (-(-o.M // 256)) * (-(-o.N // 256))) + S) * o.M * o.N * 4)
    elif ws_mode == "sized":
        wsb = lib.gemm_workspace_size(o.M, o.N, o.Kp)
    elif ws_mode == "none":
        wsb = 0
    if wsb:
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev.A.device)
        if poison:
            ws.fill_(0x5A)
    if force is None:
        lib.gemm(ot, o.M, o.N, o.Kp, dev.A, dev.Bt, dev.sA, dev.sB, D, o.row_bytes, o.row_bytes, ws, wsb,
                 stream=stream)
    elif len(force) == 3:
        lib.gemm_force_tile(ot, o.M, o.N, o.Kp, force[0], force[1], force[2], dev.A, dev.Bt, dev.sA, dev.sB, D,
                            o.row_bytes, o.row_bytes, ws, wsb, stream=stream)
    else:  # (MT, NT, splits, stream_k)
        lib.gemm_force_route(ot, o.M, o.N, o.Kp, force[0], force[1], force[2], force[3], dev.A, dev.Bt, dev.sA,
                             dev.sB, D, o.row_bytes, o.row_bytes, ws, wsb, stream=stream)
    err = lib.last_error()
    assert err == lib.OK, f"gemm rejected the call: {err} {lib.last_error_string()}"
    torch.cuda.synchronize()
    st = lib.device_status()
    assert st == 0, f"kernel status bits 0x{st:x} (bounded wait expired)"
    return D.cpu()


def ulp_distance16(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    def ordered(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x)
    return np.abs(ordered(a_bits) - ordered(b_bits))


def check(D: torch.Tensor, ref32: np.ndarray, ot, oracle, rows=None, label=""):
    """Compare GPU output rows (all or the given subset) with the oracle's FP32 result."""
    got = D if rows is None else D[torch.as_tensor(rows)]
    ref = np.asarray(ref32, np.float32)
    finite = np.isfinite(ref)
    scale = float(np.max(np.abs(ref[finite]))) if finite.any() else 1.0
    if ot == lib.OutType.F32:
        g = got.numpy()
        assert np.array_equal(np.isnan(g), np.isnan(ref)), f"{label}: NaN pattern differs"
        m = finite
        err = float(np.max(np.abs(g[m] - ref[m]))) / max(scale, 1e-30) if m.any() else 0.0
        assert err <= FP32_TOL, f"{label}: norm-wise rel err {err:.3e} > {FP32_TOL}"
        return err
    bits = got.view(torch.int16).numpy().view(np.uint16)
    ref_bits = oracle.round_f16_bits(ref) if ot == lib.OutType.F16 else oracle.round_bf16_bits(ref)
    d = ulp_distance16(bits, ref_bits)
    gf = got.float().numpy()
    ref_r = (ref_bits.view(np.float16).astype(np.float32) if ot == lib.OutType.F16
             else (ref_bits.astype(np.uint32) << 16).view(np.float32))
    ulp = np.abs(np.spacing(ref_r.astype(np.float16 if ot == lib.OutType.F16 else np.float32)))
    if ot == lib.OutType.BF16:
        ulp = np.abs(ref_r) * 2.0 ** -7 + 1e-38
    ok = (d <= 1) | (np.isfinite(gf) & np.isfinite(ref) & (np.abs(gf - ref) <= FP32_TOL * scale + ulp))
    inf_ref = np.isinf(ref_r)
    ok &= ~inf_ref | (np.sign(gf) == np.sign(ref_r))
    bad = np.argwhere(~ok)
    assert bad.size == 0, (f"{label}: {len(bad)} elements beyond 1 ulp, first {bad[:3].tolist()} "
                           f"got {gf[tuple(bad[0])]} ref {ref[tuple(bad[0])]}")
    return int(d.max()) if d.size else 0


def sample_rows(M: int, n: int, seed: int = 7) -> np.ndarray:
    """n distinct rows spread over [0, M): both ends, tile boundaries and random rows."""
    rng = np.random.default_rng(seed)
    fixed = [0, 1, 31, 32, 127, 128, M // 2, M - 129, M - 128, M - 1]
    rows = set(r for r in fixed if 0 <= r < M)
    while len(rows) < min(n, M):
        rows.add(int(rng.integers(0, M)))
    return np.array(sorted(rows), np.int32)
