"""ctypes face of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Loaded only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as the checker
or the timed baseline; the product path never imports it.

  Oracle      oracle/liboracle.so, the plain-C restatement (oracle/mxfp6_oracle.c).
  Reference   oracle/_ref/libmxfp6ref.so, the reference's own CPU functions compiled from its
              sources (oracle/ref_shim.cpp); present only where it was built.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmxfp6ref.so")

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def _bind(lib, name, res, args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = args
    return f


class Oracle:
    """The C restatement of the reference's CPU path."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle` (or __graft_entry__.build())")
        lib = C.CDLL(path)
        self.lib = lib
        self.fp6_to_float = _bind(lib, "oracle_fp6_to_float", C.c_float, [C.c_uint8])
        self.float_to_fp6 = _bind(lib, "oracle_float_to_fp6", C.c_uint8, [C.c_float])
        self.e8m0_to_float = _bind(lib, "oracle_e8m0_to_float", C.c_float, [C.c_uint8])
        self.float_to_e8m0 = _bind(lib, "oracle_float_to_e8m0", C.c_uint8, [C.c_float])
        self._quantize = _bind(lib, "oracle_quantize", None, [_f32p, C.c_int, C.c_int, _u8p, _u8p])
        self._dequantize = _bind(lib, "oracle_dequantize", None,
                                 [_u8p, C.c_int, _u8p, C.c_int, C.c_int, _f32p])
        self._gemm_rows = _bind(lib, "oracle_gemm_rows", C.c_int,
                                [_u8p, C.c_int, _u8p, _u8p, C.c_int, _u8p, C.c_int, C.c_int,
                                 C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int])
        self._round_f16 = _bind(lib, "oracle_round_f16", None, [_f32p, _u16p, C.c_longlong])
        self._round_bf16 = _bind(lib, "oracle_round_bf16", None, [_f32p, _u16p, C.c_longlong])

    def quantize(self, mat: np.ndarray):
        mat = np.ascontiguousarray(mat, dtype=np.float32)
        rows, cols = mat.shape
        packed = np.empty((rows, cols * 3 // 4), np.uint8)
        scales = np.empty((rows, cols // 32), np.uint8)
        self._quantize(mat, rows, cols, packed, scales)
        return packed, scales

    def dequantize(self, packed: np.ndarray, scales: np.ndarray, cols: int):
        packed = np.ascontiguousarray(packed)
        rows = packed.shape[0]
        out = np.empty((rows, cols), np.float32)
        self._dequantize(packed, packed.shape[1], np.ascontiguousarray(scales), rows, cols, out)
        return out

    def gemm(self, A, sA, Bt, sB, K, rows=None, f64=False, threads=None):
        """D rows = dequant(A)[rows] @ dequant(Bt)^T in the reference's sequential FP32 order
        (or FP64 with f64=True). A/Bt: packed uint8 [rows][row_bytes]; sA/sB: raw scales."""
        A = np.ascontiguousarray(A)
        Bt = np.ascontiguousarray(Bt)
        N = Bt.shape[0]
        if rows is None:
            nrows, rows_ptr, keep = A.shape[0], None, None
        else:
            keep = np.ascontiguousarray(rows, dtype=np.int32)
            nrows, rows_ptr = len(keep), keep.ctypes.data
        threads = threads or min(os.cpu_count() or 1, max(1, nrows))
        if f64:
            out = np.empty((nrows, N), np.float64)
            p32, p64 = None, out.ctypes.data
        else:
            out = np.empty((nrows, N), np.float32)
            p32, p64 = out.ctypes.data, None
        rc = self._gemm_rows(A, A.shape[1], np.ascontiguousarray(sA), Bt, Bt.shape[1],
                             np.ascontiguousarray(sB), N, K, rows_ptr, nrows, p32, p64, threads)
        if rc != 0:
            raise MemoryError("oracle_gemm_rows allocation failed")
        del keep
        return out

    def round_f16_bits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint16)
        self._round_f16(x.reshape(-1), out.reshape(-1), x.size)
        return out

    def round_bf16_bits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint16)
        self._round_bf16(x.reshape(-1), out.reshape(-1), x.size)
        return out


class Reference:
    """The reference's own CPU functions (compiled from its sources into oracle/_ref/)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle` where the reference sources exist")
        lib = C.CDLL(path)
        self.lib = lib
        self.fp6_to_float = _bind(lib, "ref_fp6_to_float", C.c_float, [C.c_uint8])
        self.float_to_fp6 = _bind(lib, "ref_float_to_fp6", C.c_uint8, [C.c_float])
        self.e8m0_to_float = _bind(lib, "ref_e8m0_to_float", C.c_float, [C.c_uint8])
        self.float_to_e8m0 = _bind(lib, "ref_float_to_e8m0", C.c_uint8, [C.c_float])
        self._pack = _bind(lib, "ref_pack_fp6", None, [_u8p, C.c_int, _u8p])
        self._unpack = _bind(lib, "ref_unpack_fp6", None, [_u8p, C.c_int, _u8p])
        self._quantize = _bind(lib, "ref_quantize", None, [_f32p, C.c_int, C.c_int, _u8p, _u8p])
        self._gemm = _bind(lib, "ref_gemm", None, [_u8p, _u8p, _u8p, _u8p, C.c_int, C.c_int, C.c_int, _f32p])
        self._gemm_mt = _bind(lib, "ref_gemm_rows_mt", None,
                              [_u8p, _u8p, _u8p, _u8p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int])

    def preshuffle_B(self, Bt, sB, K):
        Bt = np.ascontiguousarray(Bt)
        N = Bt.shape[0]
        out = np.empty(N // 32 * (K // 64) * 1536, np.uint8)
        f = _bind(self.lib, "ref_preshuffle_B", None, [_u8p, _u8p, C.c_int, C.c_int, _u8p])
        f(Bt, np.ascontiguousarray(sB), N, K, out)
        return out

    def tile_scales(self, raw, dim, K, group, subs):
        q = _bind(self.lib, "ref_tiled_scale_bytes", C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int])
        out = np.empty(q(dim, K, group, subs), np.uint8)
        f = _bind(self.lib, "ref_tile_scales", None, [_u8p, C.c_int, C.c_int, C.c_int, C.c_int, _u8p])
        f(np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1), dim, K, group, subs, out)
        return out

    def pack(self, codes: np.ndarray) -> np.ndarray:
        codes = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
        out = np.empty(codes.size * 3 // 4, np.uint8)
        self._pack(codes, codes.size, out)
        return out

    def unpack(self, packed: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.uint8)
        self._unpack(np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1), n, out)
        return out

    def quantize(self, mat: np.ndarray):
        mat = np.ascontiguousarray(mat, dtype=np.float32)
        rows, cols = mat.shape
        packed = np.empty((rows, cols * 3 // 4), np.uint8)
        scales = np.empty((rows, cols // 32), np.uint8)
        self._quantize(mat, rows, cols, packed, scales)
        return packed, scales

    def gemm(self, A, sA, Bt, sB, K, threads=1):
        """mxfp6_gemm_ref on compact (row stride 3K/4) operands; threads > 1 splits rows."""
        A = np.ascontiguousarray(A)
        Bt = np.ascontiguousarray(Bt)
        M, N = A.shape[0], Bt.shape[0]
        D = np.empty((M, N), np.float32)
        if threads <= 1:
            self._gemm(A, np.ascontiguousarray(sA), Bt, np.ascontiguousarray(sB), M, N, K, D)
        else:
            self._gemm_mt(A, np.ascontiguousarray(sA), Bt, np.ascontiguousarray(sB), M, N, K, D, threads)
        return D


def reference_available() -> bool:
    return os.path.exists(REF_SO)
