"""Python front end of the NVFP4 test oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only as the checker.  The product
(``fp4-gemm-blackwell_b200``) never imports it.

It wraps two shared libraries:

* ``libnvfp4_oracle.so`` -- the C restatement of the reference quantizer
  (``nvfp4_oracle.c``; each function cites fp4_gemm_lib.cu lines);
* ``_ref/libref_quant.so`` -- the reference's own quantizer source compiled for
  the host (``build.py``), used to pin the restatement and to make golden
  vectors.  It may be absent; ``ref_available()`` says so.

BF16 data is passed as numpy ``uint16`` arrays of raw bits (``bf16_bits``).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE_SO = os.path.join(HERE, "libnvfp4_oracle.so")
_REF_SO = os.path.join(HERE, "_ref", "libref_quant.so")

_lib = None
_ref = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)


def _ptr(a: np.ndarray, typ):
    return a.ctypes.data_as(typ)


def lib():
    """The C oracle, built on first use when its .so is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(_ORACLE_SO):
            from . import build as _build  # noqa: WPS433 (test-infra lazy build)
            _build.build_oracle()
        L = ctypes.CDLL(_ORACLE_SO)
        L.oracle_e2m1_code.restype = ctypes.c_uint8
        L.oracle_e2m1_code.argtypes = [ctypes.c_float]
        L.oracle_ue4m3_encode.restype = ctypes.c_uint8
        L.oracle_ue4m3_encode.argtypes = [ctypes.c_float]
        L.oracle_ue4m3_decode.restype = ctypes.c_float
        L.oracle_ue4m3_decode.argtypes = [ctypes.c_uint8]
        L.oracle_sf_index.restype = ctypes.c_long
        L.oracle_sf_index.argtypes = [ctypes.c_long, ctypes.c_long, ctypes.c_long]
        L.oracle_quantize.restype = ctypes.c_int
        L.oracle_quantize.argtypes = [_u16p, ctypes.c_long, ctypes.c_long, ctypes.c_long,
                                      ctypes.c_long, ctypes.c_long, _u8p, _u8p]
        L.oracle_dequantize.restype = ctypes.c_int
        L.oracle_dequantize.argtypes = [_u8p, _u8p, ctypes.c_long, ctypes.c_long, _f32p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF_SO)


def ref_lib():
    """The reference's own quantizer compiled for the host (oracle/_ref)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{_REF_SO} not built (python oracle/build.py)")
        R = ctypes.CDLL(_REF_SO)
        R.ref_quantize.restype = ctypes.c_int
        R.ref_quantize.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, _u8p, _u8p]
        R.ref_float_to_fp4.restype = ctypes.c_uint8
        R.ref_float_to_fp4.argtypes = [ctypes.c_float]
        R.ref_float_to_ue4m3.restype = ctypes.c_uint8
        R.ref_float_to_ue4m3.argtypes = [ctypes.c_float]
        R.ref_ue4m3_to_float.restype = ctypes.c_float
        R.ref_ue4m3_to_float.argtypes = [ctypes.c_uint8]
        R.ref_sf_index.restype = ctypes.c_int
        R.ref_sf_index.argtypes = [ctypes.c_int] * 4
        _ref = R
    return _ref


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def bf16_bits(x) -> np.ndarray:
    """Raw bf16 bits (uint16) of a torch bf16 tensor or an array of bits."""
    try:
        import torch
        if isinstance(x, torch.Tensor):
            assert x.dtype == torch.bfloat16
            return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    except ImportError:  # pragma: no cover
        pass
    a = np.asarray(x)
    assert a.dtype == np.uint16
    return a


def bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (NaN kept as a quiet NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def e2m1_code(v: float) -> int:
    return int(lib().oracle_e2m1_code(ctypes.c_float(v)))


def ue4m3_encode(v: float) -> int:
    return int(lib().oracle_ue4m3_encode(ctypes.c_float(v)))


def ue4m3_decode(b: int) -> float:
    return float(lib().oracle_ue4m3_decode(ctypes.c_uint8(b)))


def sf_index(r: int, kb: int, nsb: int) -> int:
    return int(lib().oracle_sf_index(r, kb, nsb))


def quantize(x, rows_pad: int | None = None, k_pad: int | None = None):
    """Quantize a 2-D bf16 matrix (torch bf16 or uint16 bits) like the reference.

    Returns ``(fp4 [rows_pad, k_pad/2] uint8, sf [rows_pad*k_pad/16] uint8)``;
    the pads default to the reference's round-up to 128.
    """
    bits = np.ascontiguousarray(bf16_bits(x))
    rows, cols = bits.shape
    rows_pad = rows_pad or round_up(max(rows, 1), 128)
    k_pad = k_pad or round_up(max(cols, 1), 128)
    fp4 = np.zeros((rows_pad, k_pad // 2), dtype=np.uint8)
    sf = np.zeros(rows_pad * k_pad // 16, dtype=np.uint8)
    rc = lib().oracle_quantize(_ptr(bits, _u16p), rows, cols, cols, rows_pad, k_pad,
                               _ptr(fp4, _u8p), _ptr(sf, _u8p))
    if rc != 0:
        raise ValueError(f"oracle_quantize: bad shape rows={rows} cols={cols} pads={rows_pad},{k_pad}")
    return fp4, sf


def dequantize(fp4: np.ndarray, sf: np.ndarray, rows: int, k_pad: int) -> np.ndarray:
    """fp32 [rows, k_pad] values that the packed operand represents."""
    fp4 = np.ascontiguousarray(fp4, dtype=np.uint8)
    sf = np.ascontiguousarray(sf, dtype=np.uint8)
    out = np.empty((rows, k_pad), dtype=np.float32)
    rc = lib().oracle_dequantize(_ptr(fp4, _u8p), _ptr(sf, _u8p), rows, k_pad, _ptr(out, _f32p))
    if rc != 0:
        raise ValueError("oracle_dequantize: rows and k_pad must be multiples of 128")
    return out


def ref_quantize(x) -> tuple[np.ndarray, np.ndarray]:
    """Run the reference's own quantizer (host build) on an already padded matrix."""
    bits = np.ascontiguousarray(bf16_bits(x))
    rows, K = bits.shape
    fp4 = np.zeros((rows, K // 2), dtype=np.uint8)
    sf = np.zeros(rows * K // 16, dtype=np.uint8)
    rc = ref_lib().ref_quantize(_ptr(bits, _u16p), rows, K, _ptr(fp4, _u8p), _ptr(sf, _u8p))
    if rc != 0:
        raise ValueError("ref_quantize: bad shape")
    return fp4, sf


def gemm_reference(x_bf16, w_fp4, w_sf, n_pad: int, k_pad: int, n_out: int,
                   bias=None, alpha: float = 1.0, beta: float = 0.0, c=None, threads: int | None = None):
    """fp32 result of the reference cached linear: alpha * dq(q(x)) @ dq(W)^T + beta*C (+ bias).

    Mirrors fp4_gemm_run_cached (fp4_gemm_lib.cu:754-840) with the FP4 GEMM
    replaced by an fp32 matmul of the dequantized operands, then the bias add
    of fp4_gemm.py:389-390.  Returns fp32 [M, n_out] (before the bf16 rounding).
    """
    import torch
    if threads:
        torch.set_num_threads(threads)
    bits = bf16_bits(x_bf16)
    M = bits.shape[0]
    m_pad = round_up(max(M, 1), 128)
    a_fp4, a_sf = quantize(bits, m_pad, k_pad)
    a = torch.from_numpy(dequantize(a_fp4, a_sf, m_pad, k_pad))[:M]
    w = torch.from_numpy(dequantize(w_fp4, w_sf, n_pad, k_pad))[:n_out]
    out = alpha * (a @ w.t())
    if c is not None and beta != 0.0:
        out = out + beta * torch.as_tensor(c).float()
    if bias is not None:
        out = out + torch.as_tensor(bias).float()
    return out
