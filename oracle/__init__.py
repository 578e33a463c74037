"""CPU oracle of PackR's training hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, and only as the checker.  The product (packr_b200) never
imports it and has no CPU fallback.

It restates the reference's arithmetic on the CPU with numpy:
  * decode_f32        packr/kernel.py:127-130   f32(W_f) + f32(fp16(lut[W_p]))
  * decode_bf16       packr/autograd.py:66-67   bf16(f32(W_f) + f32(bf16(lut[W_p])))
  * linear_forward    packr/kernel.py:133-136 + packr/layer.py:96-97
  * linear_backward   packr/autograd.py:65-83 + the autograd of layer.py:97
  * adam8_step        packr/cuda_adam_kernel.cu:19-69 (C, liboracle.so)
bf16 tensors are carried as uint16 bit patterns; conversions use the
round-to-nearest-even integer method of torch / cuda_adam_kernel.cu:62-64.
Pinned against tests/golden/ (made by importing the reference package) and,
for the optimizer, against the reference CUDA kernel built from its source.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent

# --------------------------------------------------------------------------
# bf16 / fp16 helpers (bit exact)
# --------------------------------------------------------------------------


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits (uint16), round to nearest even (NaN kept NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_to_f32(f32_to_bf16(x))


# --------------------------------------------------------------------------
# PackRLinear
# --------------------------------------------------------------------------


def decode_f32(W_p: np.ndarray, W_f: np.ndarray, lut: np.ndarray) -> np.ndarray:
    """Forward decode, packr/kernel.py:127-130: fp16 gather, then W_f(bf16) +
    decoded(fp16) promoted to float32 and added in float32."""
    dec16 = lut.astype(np.float32).astype(np.float16)[W_p]
    return (bf16_to_f32(W_f) + dec16.astype(np.float32)).astype(np.float32)


def decode_bf16(W_p: np.ndarray, W_f: np.ndarray, lut: np.ndarray) -> np.ndarray:
    """Backward decode, packr/autograd.py:66-67: bf16(lut[W_p]) then a bf16
    add (float32 add rounded to bf16).  Returns bf16 bits."""
    lut16 = round_bf16(lut.astype(np.float32))
    return f32_to_bf16(bf16_to_f32(W_f) + lut16[W_p])


def _x_f32(x: np.ndarray, x_is_bf16: bool) -> np.ndarray:
    return bf16_to_f32(x) if x_is_bf16 else np.ascontiguousarray(x, dtype=np.float32)


def linear_forward(x, W_p, W_f, lut, bias=None, x_is_bf16=False):
    """out[M,N] float32 = f32(x) @ decode_f32 + f32(bias): packr/kernel.py:133-136
    (fp32 GEMM) and packr/layer.py:96-97 (f32 out + bf16 bias -> f32)."""
    xf = _x_f32(x, x_is_bf16).reshape(-1, W_p.shape[0])
    out = np.matmul(xf, decode_f32(W_p, W_f, lut), dtype=np.float32)
    if bias is not None:
        out = out + bf16_to_f32(bias)[None, :]
    return out.astype(np.float32)


def bincount256(W_p: np.ndarray) -> np.ndarray:
    return np.bincount(W_p.reshape(-1), minlength=256).astype(np.int32)


def linear_backward(dY, x, W_p, W_f, lut, has_bias=False, x_is_bf16=False):
    """packr/autograd.py:65-83 with the bias gradient of layer.py:97.

    Returns dict with
      dX    [M,K]  bf16(bf16(dY) @ Wb^T) — bf16 bits if x is bf16, else the
                   same value widened to float32 (autograd casts to x.dtype)
      dW_f  [K,N]  bf16 bits of f32(x)^T @ f32(dY)
      dW    [K,N]  the float32 dW_full itself (for property checks)
      dlut  [256]  scatter_add(dW_full by W_p) / (bincount + 1e-8)
      dbias [N]    bf16 bits of dY.sum(0) (only if has_bias)
    """
    K, N = W_p.shape
    dY = np.ascontiguousarray(dY, dtype=np.float32).reshape(-1, N)
    xf = _x_f32(x, x_is_bf16).reshape(-1, K)
    Wb = bf16_to_f32(decode_bf16(W_p, W_f, lut))
    dYb = round_bf16(dY)
    acc = np.matmul(dYb, Wb.T, dtype=np.float32)
    dX16 = f32_to_bf16(acc)
    dX = dX16 if x_is_bf16 else bf16_to_f32(dX16)
    dW = np.matmul(xf.T, dY, dtype=np.float32)
    counts = bincount256(W_p).astype(np.float32)
    # scatter_add of fp32 dW by W_p; bins summed in float64 then rounded (the
    # reference's fp32 atomics have no fixed order; this is their exact value
    # to within one rounding)
    sums = np.bincount(W_p.reshape(-1), weights=dW.reshape(-1).astype(np.float64), minlength=256).astype(np.float32)
    dlut = (sums / (counts + np.float32(1e-8))).astype(np.float32)
    res = {"dX": dX, "dW_f": f32_to_bf16(dW), "dW": dW, "dlut": dlut}
    if has_bias:
        res["dbias"] = f32_to_bf16(dY.sum(axis=0, dtype=np.float32))
    return res


def max_rel(a: np.ndarray, b: np.ndarray) -> float:
    """max|a-b| / max|b|: the reference tests' relative error
    (tests/test_packr_kernel.py:45, tests/test_packr_core.py:41)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.abs(b).max()
    return float(np.abs(a - b).max() / den) if den > 0 else float(np.abs(a - b).max())


# --------------------------------------------------------------------------
# 8-bit AdamW (C)
# --------------------------------------------------------------------------

_lib = None


def _liboracle():
    global _lib
    if _lib is None:
        path = _HERE / "liboracle.so"
        if not path.exists():
            from . import build as _b
            _b.build_oracle()
        lib = ctypes.CDLL(str(path))
        f = lib.oracle_adam8_step
        f.restype = None
        f.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_int] + [ctypes.c_float] * 7
        _lib = lib
    return _lib


def adam8_step(p, g, m, v, ms, vs, lr, b1, b2, eps, bc1, bc2, wd):
    """In-place 8-bit AdamW step on numpy arrays.  p/g: uint16 (bf16 bits) or
    float32; m/v: int8; ms/vs: float32 [ceil(n/256)]."""
    is_bf16 = p.dtype == np.uint16
    assert g.dtype == p.dtype and m.dtype == np.int8 and v.dtype == np.int8
    assert ms.dtype == np.float32 and vs.dtype == np.float32
    for a in (p, g, m, v, ms, vs):
        assert a.flags["C_CONTIGUOUS"]
    n = p.size
    assert ms.size == (n + 255) // 256 == vs.size
    _liboracle().oracle_adam8_step(p.ctypes.data, g.ctypes.data, m.ctypes.data, v.ctypes.data,
                                   ms.ctypes.data, vs.ctypes.data, n, int(is_bf16), lr, b1, b2,
                                   eps, bc1, bc2, wd)


def adam8_bias_corrections(b1: float, b2: float, step: int):
    """bc1, bc2 as packr/cuda_adam.py:175-176 computes them (Python double)."""
    return 1.0 - b1 ** step, 1.0 - b2 ** step
