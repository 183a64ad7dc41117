"""Python binding of libmxfp6gemm (B200 MXFP6 GEMM) over its C ABI (include/mxfp6_gemm.h).

Mirrors the reference library's public interface (eeezio/mxfp6-gemm include/mxfp6/gemm.hpp and
include/mxfp6/preprocess.hpp): OutType, K_TILE, kpad, choose_tile, gemm_workspace_size, gemm,
and the host layout producers quantize_to_mxfp6 / preprocess_B / preprocess_scale /
preshuffle_B / tile_scale. Device buffers are passed as raw addresses (ints) or as objects with
a data_ptr() method (torch tensors); the binding itself has no torch dependency.

There is no CPU fallback: importing this module loads the compiled library and raises if it
is missing, and every GEMM runs the sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libmxfp6gemm.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR}` "
                      "(or python -c 'import __graft_entry__; __graft_entry__.build()')")

_lib = C.CDLL(LIB_PATH)

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")


def _fn(name, res, args):
    f = getattr(_lib, name)
    f.restype = res
    f.argtypes = args
    return f


_gemm = _fn("mxfp6_gemm", None, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                 C.c_size_t])
_gemm_stream = _fn("mxfp6_gemm_stream", None,
                   [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                    C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p])
_force = _fn("mxfp6_gemm_force_tile", None,
             [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
              C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
              C.c_void_p])
_force_route = _fn("mxfp6_gemm_force_route", None,
                   [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                    C.c_void_p])
_route_sk = _fn("mxfp6_route_stream_k", C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int])
_route_band = _fn("mxfp6_route_banded", C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int])
_sk_bytes = _fn("mxfp6_stream_k_workspace_bytes", C.c_size_t, [])
_static_ws_gemm = _fn("mxfp6_gemm_static_workspace", None,
                      [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                       C.c_void_p, C.c_int, C.c_int, C.c_void_p])
static_workspace_bytes = _fn("mxfp6_static_workspace_bytes", C.c_size_t, [])
set_repad_scratch = _fn("mxfp6_set_repad_scratch", C.c_int, [C.c_int])  # returns the previous setting
repad_scratch_bytes = _fn("mxfp6_repad_scratch_bytes", C.c_size_t, [])
release_repad_scratch = _fn("mxfp6_release_repad_scratch", C.c_int, [])
_gather = _fn("mxfp6_gemm_gather", None,
              [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
               C.POINTER(C.c_void_p), C.c_int, C.c_longlong, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
               C.c_void_p])
_ipc_export = _fn("mxfp6_ipc_export", C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_size_t)])
_ipc_import = _fn("mxfp6_ipc_import", C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p),
                                               C.POINTER(C.c_void_p)])
_ipc_close = _fn("mxfp6_ipc_close", C.c_int, [C.c_void_p])

_ws = _fn("mxfp6_gemm_workspace_size", C.c_size_t, [C.c_int, C.c_int, C.c_int])
_ws_out = _fn("mxfp6_gemm_workspace_size_out", C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int])
_ws_a = _fn("mxfp6_gemm_workspace_size_a", C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int])
_choose = _fn("mxfp6_choose_tile", None, [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)])
_route = _fn("mxfp6_route", None, [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)])
_k_tile = _fn("mxfp6_k_tile", C.c_int, [])
_kpad = _fn("mxfp6_kpad", C.c_int, [C.c_int])
last_error = _fn("mxfp6_last_error", C.c_int, [])
_last_error_string = _fn("mxfp6_last_error_string", C.c_char_p, [])
_device_status = _fn("mxfp6_device_status", C.c_int, [])
launch_count = _fn("mxfp6_launch_count", C.c_uint64, [])
set_wait_budget = _fn("mxfp6_set_wait_budget", C.c_longlong, [C.c_longlong])  # this thread's kernels; <= 0: default
_quantize = _fn("mxfp6_quantize", None, [_f32p, C.c_int, C.c_int, _u8p, _u8p, C.c_int])
_quantize_dev = _fn("mxfp6_quantize_device", C.c_int,
                    [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p])
_quantize_dev_p = _fn("mxfp6_quantize_device_padded", C.c_int,
                      [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p])
_imp_B_dev = _fn("mxfp6_import_ref_B_device", C.c_int,
                 [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p])
_imp_sc_dev = _fn("mxfp6_import_ref_scales_device", C.c_int,
                  [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p])
_repad_dev = _fn("mxfp6_repad_rows_device", C.c_int,
                 [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p])
_dequantize = _fn("mxfp6_dequantize", None, [_u8p, _u8p, C.c_int, C.c_int, _f32p])
_tiled_bytes = _fn("mxfp6_tiled_scale_bytes", C.c_size_t, [C.c_int, C.c_int])
_tile = _fn("mxfp6_tile_scales", None, [_u8p, C.c_int, C.c_int, _u8p])
_untile = _fn("mxfp6_untile_scales", None, [_u8p, C.c_int, C.c_int, _u8p])
_imp_B = _fn("mxfp6_import_ref_B", C.c_int, [_u8p, C.c_int, C.c_int, _u8p, C.c_int])
_imp_sc = _fn("mxfp6_import_ref_scales", C.c_int, [_u8p, C.c_int, C.c_int, C.c_int, C.c_int, _u8p])
_repad = _fn("mxfp6_repad_rows", C.c_int, [_u8p, C.c_int, C.c_int, C.c_int, _u8p, C.c_int])

# status codes (enum mxfp6_status)
OK, ERR_INVALID_SHAPE, ERR_INVALID_STRIDE, ERR_MISALIGNED, ERR_NULL_POINTER = 0, 1, 2, 3, 4
ERR_INVALID_OUT_TYPE, ERR_CUDA, ERR_DEVICE_TIMEOUT, ERR_WORKSPACE, ERR_UNSUPPORTED = 5, 6, 7, 8, 9


class OutType(enum.IntEnum):
    F32 = 0
    F16 = 1
    BF16 = 2


K_TILE = _k_tile()


def kpad(K: int) -> int:
    return _kpad(K)


def a_compact_end_pad(K: int) -> int:
    """Spare bytes the reference asks for after a compact A buffer (never read here)."""
    return kpad(K) * 3 // 4 - K * 3 // 4


def pad_scales_k(scales: np.ndarray, dim: int, K: int) -> np.ndarray:
    """Raw scales [dim][K/32] -> [dim][kpad(K)/32], tail blocks code 127 (finite, 2^0)."""
    out = np.full((dim, kpad(K) // 32), 127, np.uint8)
    out[:, :K // 32] = np.asarray(scales, np.uint8).reshape(dim, K // 32)
    return out


@dataclass(frozen=True)
class TileChoice:
    MT: int
    NT: int
    MPW: int
    NPW: int


def choose_tile(M: int, N: int, Kp: int) -> TileChoice:
    out = (C.c_int * 4)()
    _choose(M, N, Kp, out)
    return TileChoice(*out)


def route(ot, M: int, N: int, Kp: int) -> dict:
    """The route gemm() takes for output type ot: tile, K splits (mxfp6_route), whether the CTA
    pair runs a stream-K tail (mxfp6_route_stream_k) and whether its split is banded
    (mxfp6_route_banded)."""
    out = (C.c_int * 3)()
    _route(int(ot), M, N, Kp, out)
    return {"MT": out[0], "NT": out[1], "splits": out[2], "stream_k": bool(_route_sk(int(ot), M, N, Kp)),
            "banded": bool(_route_band(int(ot), M, N, Kp))}


def gemm_workspace_size(M: int, N: int, Kp: int, ot=None) -> int:
    """Split-K workspace bytes: for every output type (as the reference's query), or for `ot`."""
    return _ws(M, N, Kp) if ot is None else _ws_out(int(ot), M, N, Kp)


def gemm_workspace_size_a(M: int, N: int, Kp: int, a_row_bytes: int) -> int:
    """Workspace that also holds a padded copy of an A the tensor load cannot address."""
    return _ws_a(M, N, Kp, a_row_bytes)


def _addr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def gemm(ot, M, N, Kp, dA, dBsh, dsA, dsB, dD, A_row_bytes, B_row_bytes, ws=None, ws_bytes=0,
         stream=None):
    """D[M,N] = A[M,K]·B[K,N] (mxfp6::gemm). Asynchronous; check last_error() after the call."""
    args = (int(ot), M, N, Kp, _addr(dA), _addr(dBsh), _addr(dsA), _addr(dsB), _addr(dD),
            A_row_bytes, B_row_bytes, _addr(ws), ws_bytes)
    if stream is None:
        _gemm(*args)
    else:
        _gemm_stream(*args, _addr(stream) if not hasattr(stream, "cuda_stream") else stream.cuda_stream)


def gemm_force_tile(ot, M, N, Kp, MT, NT, splits, dA, dBsh, dsA, dsB, dD, A_row_bytes, B_row_bytes,
                    ws=None, ws_bytes=0, stream=None):
    """Test hook (reference: gemm_force_tile): run tile MT x NT with `splits` K segments."""
    s = 0 if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream))
    _force(int(ot), M, N, Kp, MT, NT, splits, _addr(dA), _addr(dBsh), _addr(dsA), _addr(dsB), _addr(dD),
           A_row_bytes, B_row_bytes, _addr(ws), ws_bytes, s)


def gemm_force_route(ot, M, N, Kp, MT, NT, splits, stream_k, dA, dBsh, dsA, dsB, dD, A_row_bytes, B_row_bytes,
                     ws=None, ws_bytes=0, stream=None):
    """Test hook: gemm_force_tile plus the CTA pair's stream-K tail (stream_k 1) or banded split
    (stream_k 2, with `splits` short bands)."""
    s = 0 if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream))
    _force_route(int(ot), M, N, Kp, MT, NT, splits, int(stream_k), _addr(dA), _addr(dBsh), _addr(dsA),
                 _addr(dsB), _addr(dD), A_row_bytes, B_row_bytes, _addr(ws), ws_bytes, s)


def stream_k_bytes() -> int:
    """Workspace of the CTA pair's stream-K tail on this device (256 KB + 16 bytes per pair)."""
    return _sk_bytes()


def gemm_gather(ot, M, N, Kp, dA, dBsh, dsA, dsB, dDs, ldd, col0, A_row_bytes, B_row_bytes, ws=None, ws_bytes=0,
                stream=None):
    """mxfp6_gemm_gather: D written into every destination of dDs (tensors or device addresses),
    each a row-major [M][ldd] matrix, at column col0."""
    ptrs = (C.c_void_p * len(dDs))(*[_addr(d) for d in dDs])
    s = 0 if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream))
    _gather(int(ot), M, N, Kp, _addr(dA), _addr(dBsh), _addr(dsA), _addr(dsB), ptrs, len(dDs), ldd, col0,
            A_row_bytes, B_row_bytes, _addr(ws), ws_bytes, s)


def ipc_export(t) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding t, t's offset in it)."""
    h = (C.c_uint8 * 64)()
    off = C.c_size_t(0)
    rc = _ipc_export(_addr(t), h, C.byref(off))
    if rc != OK:
        raise RuntimeError(f"mxfp6_ipc_export failed ({rc})")
    return bytes(h), off.value


def ipc_import(handle: bytes, offset: int) -> tuple[int, int]:
    """Map a peer allocation: returns (base for ipc_close, device address of the tensor)."""
    h = (C.c_uint8 * 64).from_buffer_copy(handle)
    base, ptr = C.c_void_p(), C.c_void_p()
    rc = _ipc_import(h, offset, C.byref(base), C.byref(ptr))
    if rc != OK:
        raise RuntimeError(f"mxfp6_ipc_import failed ({rc})")
    return base.value, ptr.value


def ipc_close(base: int) -> int:
    return _ipc_close(base)


def gemm_static_workspace(ot, M, N, Kp, dA, dBsh, dsA, dsB, dD, A_row_bytes, B_row_bytes, stream=None):
    """mxfp6_gemm_static_workspace: gemm() without a caller workspace, for callers that cannot
    allocate device memory (split-K partials go to the library's fixed 32 MiB array)."""
    s = 0 if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream))
    _static_ws_gemm(int(ot), M, N, Kp, _addr(dA), _addr(dBsh), _addr(dsA), _addr(dsB), _addr(dD), A_row_bytes,
                    B_row_bytes, s)


def last_error_string() -> str:
    return _last_error_string().decode()


def device_status() -> int:
    """Synchronise and return (then clear) the kernels' sticky status bits; -1 if sync failed."""
    return _device_status()


# ---- host layout producers (C++ header helpers through the C ABI) --------------------------------

@dataclass
class QuantizedMatrix:
    packed_data: np.ndarray  # uint8 [rows][packed_row_bytes]
    scales: np.ndarray       # uint8 [rows][cols/32]
    rows: int
    cols: int

    @property
    def packed_row_bytes(self) -> int:
        return self.cols * 3 // 4

    @property
    def scale_cols(self) -> int:
        return self.cols // 32


def quantize_to_mxfp6(mat: np.ndarray, threads: int = 0) -> QuantizedMatrix:
    mat = np.ascontiguousarray(mat, dtype=np.float32)
    rows, cols = mat.shape
    if cols % 32:
        raise ValueError("cols must be a multiple of 32")
    packed = np.empty((rows, cols * 3 // 4), np.uint8)
    scales = np.empty((rows, cols // 32), np.uint8)
    _quantize(mat, rows, cols, packed, scales, threads)
    return QuantizedMatrix(packed, scales, rows, cols)


def quantize_device(d_mat, rows, cols, d_packed, d_scales, tiled=False, stream=None) -> int:
    """quantize_to_mxfp6 on the GPU (device pointers); scales raw or in the GEMM's atom layout."""
    s = 0 if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream))
    return _quantize_dev(_addr(d_mat), rows, cols, _addr(d_packed), _addr(d_scales), 1 if tiled else 0, s)


def quantize_device_padded(d_mat, rows, cols, padded_cols, d_packed, d_scales, tiled=False, stream=None) -> int:
    s = 0 if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream))
    return _quantize_dev_p(_addr(d_mat), rows, cols, padded_cols, _addr(d_packed), _addr(d_scales),
                           1 if tiled else 0, s)


def repad_rows_device(d_src, rows, src_row_bytes, bytes_used, d_dst, dst_row_bytes, stream=None) -> int:
    s = 0 if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream))
    return _repad_dev(_addr(d_src), rows, src_row_bytes, bytes_used, _addr(d_dst), dst_row_bytes, s)


def dequantize_mxfp6(q: QuantizedMatrix) -> np.ndarray:
    out = np.empty((q.rows, q.cols), np.float32)
    _dequantize(np.ascontiguousarray(q.packed_data), np.ascontiguousarray(q.scales), q.rows, q.cols, out)
    return out


def preprocess_B(B: np.ndarray, threads: int = 0) -> QuantizedMatrix:
    """B[K][N] -> quantised B^T[N][K]."""
    return quantize_to_mxfp6(np.ascontiguousarray(np.asarray(B, np.float32).T), threads)


def preshuffle_B(Bq: QuantizedMatrix) -> np.ndarray:
    """Identity on B200: the kernel reads B^T packed rows directly."""
    return Bq.packed_data


def tiled_scale_bytes(rows: int, cols: int) -> int:
    return _tiled_bytes(rows, cols)


def preprocess_scale(scales: np.ndarray, dim: int, K: int) -> np.ndarray:
    """Raw scales [dim][K/32] -> B200 atom layout (also what tile_scale returns)."""
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    out = np.empty(tiled_scale_bytes(dim, K), np.uint8)
    _tile(scales.reshape(-1), dim, K, out)
    return out


def tile_scale(ps: np.ndarray, group: int = 0, subs: int = 0) -> np.ndarray:
    """The atom layout is route independent; kept for the reference's call shape."""
    return ps


def untile_scales(tiled: np.ndarray, dim: int, K: int) -> np.ndarray:
    out = np.empty((dim, K // 32), np.uint8)
    _untile(np.ascontiguousarray(tiled, dtype=np.uint8), dim, K, out.reshape(-1))
    return out


# ---- import of buffers prepared for the reference library ------------------------------------------

def import_ref_B(ref_bsh: np.ndarray, N: int, Kp_ref: int, Kp: int | None = None) -> np.ndarray:
    """Reference preshuffle_B buffer -> B^T packed rows [N][3*Kp/4] (Kp = kpad(Kp_ref))."""
    Kp = Kp or kpad(Kp_ref)
    out = np.empty((N, Kp * 3 // 4), np.uint8)
    rc = _imp_B(np.ascontiguousarray(ref_bsh, dtype=np.uint8), N, Kp_ref, out.reshape(-1), Kp * 3 // 4)
    if rc != OK:
        raise ValueError(f"mxfp6_import_ref_B failed ({rc})")
    return out


def import_ref_scales(ref_tiled: np.ndarray, dim: int, Kp_ref: int, group: int, subs: int = 3,
                      Kp: int | None = None) -> np.ndarray:
    """Reference tiled scales -> raw scales [dim][Kp/32]; blocks past Kp_ref get the finite 127."""
    Kp = Kp or kpad(Kp_ref)
    raw = np.empty((dim, Kp_ref // 32), np.uint8)
    rc = _imp_sc(np.ascontiguousarray(ref_tiled, dtype=np.uint8), dim, Kp_ref, group, subs, raw.reshape(-1))
    if rc != OK:
        raise ValueError(f"mxfp6_import_ref_scales failed ({rc})")
    out = np.full((dim, Kp // 32), 127, np.uint8)
    out[:, :Kp_ref // 32] = raw
    return out


def _stream_arg(stream) -> int:
    if stream is None:
        return 0
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else _addr(stream)


def import_ref_B_device(d_ref_bsh, N: int, Kp_ref: int, d_out, out_row_bytes: int, stream=None) -> int:
    """mxfp6_import_ref_B_device: reference preshuffle_B buffer (device) -> B^T rows of
    out_row_bytes in d_out (device). Returns an mxfp6_status."""
    return _imp_B_dev(_addr(d_ref_bsh), N, Kp_ref, _addr(d_out), out_row_bytes, _stream_arg(stream))


def import_ref_scales_device(d_ref_tiled, dim: int, Kp_ref: int, group: int, subs: int, d_out_tiled, Kp: int,
                             stream=None) -> int:
    """mxfp6_import_ref_scales_device: reference tiled scales (device) -> this library's scale atoms
    for Kp in d_out_tiled (device). Returns an mxfp6_status."""
    return _imp_sc_dev(_addr(d_ref_tiled), dim, Kp_ref, group, subs, _addr(d_out_tiled), Kp, _stream_arg(stream))


def repad_rows(src: np.ndarray, bytes_used: int, dst_row_bytes: int) -> np.ndarray:
    src = np.ascontiguousarray(src, dtype=np.uint8)
    out = np.empty((src.shape[0], dst_row_bytes), np.uint8)
    rc = _repad(src.reshape(-1), src.shape[0], src.shape[1], bytes_used, out.reshape(-1), dst_row_bytes)
    if rc != OK:
        raise ValueError(f"mxfp6_repad_rows failed ({rc})")
    return out


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """Pack 6-bit codes (last axis, length % 4 == 0) four per three bytes, LSB first."""
    c = np.asarray(codes, dtype=np.uint32) & 63
    g = c.reshape(c.shape[:-1] + (-1, 4))
    w = g[..., 0] | (g[..., 1] << 6) | (g[..., 2] << 12) | (g[..., 3] << 18)
    out = np.stack([w & 255, (w >> 8) & 255, (w >> 16) & 255], axis=-1).astype(np.uint8)
    return out.reshape(c.shape[:-1] + (-1,))


def unpack_codes(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint32)
    g = p.reshape(p.shape[:-1] + (-1, 3))
    w = g[..., 0] | (g[..., 1] << 8) | (g[..., 2] << 16)
    out = np.stack([(w >> (6 * i)) & 63 for i in range(4)], axis=-1).astype(np.uint8)
    return out.reshape(p.shape[:-1] + (-1,))
