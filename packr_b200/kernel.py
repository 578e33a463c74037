"""PackR matmul on B200: thin torch-facing wrappers over libpackr_b200.so.

packr_matmul(x, W_p, W_f, lut, bias=None) keeps the signature, the float32
[M, N] result and the assertions of reference packr/kernel.py:98-141, but the
decode and the GEMM are one sm_100a kernel (tcgen05 tensor cores, TMEM
accumulator) that decodes W = bf16(W_f + bf16(lut[W_p])) in shared memory.
The operands are bf16: x (rounded to bf16 when it is f32) and the decoded W,
accumulated in f32.

forward() / backward() below are the raw entry points the autograd Function
uses; they allocate outputs and the workspace through torch's caching
allocator and launch on torch's current stream.  No CPU path exists: CPU
tensors raise.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

# dW precision: "auto" = fp32-faithful split (x . dY_hi + x . dY_lo
# [+ x_lo . dY_hi]) when x is f32, dY rounded to bf16 otherwise; "split" and
# "bf16" force one or the other.
DW_PRECISION = os.environ.get("PACKR_DW_PRECISION", "auto")


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.PACKR_DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.PACKR_DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def _as_operand(x: torch.Tensor) -> torch.Tensor:
    if x.dtype not in (torch.bfloat16, torch.float32):
        x = x.float()
    return x.contiguous()


def forward(x: torch.Tensor, W_p: torch.Tensor, W_f: torch.Tensor, lut: torch.Tensor,
            bias: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] float32 = x @ decode(W_p, W_f, lut) + bias, on the GPU."""
    lib = _lib.load()
    x = _as_operand(x)
    M, K = x.shape
    N = W_p.shape[1]
    dev = x.device
    W_f = W_f.contiguous()
    lut = lut.detach().float().contiguous()
    if bias is not None:
        bias = bias.detach()
        if bias.dtype not in (torch.bfloat16, torch.float32):
            bias = bias.float()
        bias = bias.contiguous()
    out = torch.empty(M, N, dtype=torch.float32, device=dev)
    xd = _dtype_code(x)
    with torch.cuda.device(dev):
        ws = _workspace(lib.packr_forward_workspace_bytes(M, K, N, xd), dev)
        code = lib.packr_forward(_ptr(x), xd, _ptr(W_p), _ptr(W_f), _ptr(lut), _ptr(bias),
                                 _dtype_code(bias) if bias is not None else 0, _ptr(out), M, K, N, _ptr(ws),
                                 0 if ws is None else ws.numel(), _stream(dev))
    _lib.check("packr_forward", code)
    return out


def forward_decoded(x: torch.Tensor, Wd: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] float32 = x @ Wd + bias for an already decoded bf16 Wd [K, N]
    (predecode_bf16), through the plain tcgen05 GEMM."""
    lib = _lib.load()
    x = _as_operand(x)
    M, K = x.shape
    N = Wd.shape[1]
    dev = x.device
    if Wd.dtype != torch.bfloat16 or tuple(Wd.shape) != (K, N):
        raise ValueError("Wd must be bf16 [K, N]")
    Wd = Wd.contiguous()
    if bias is not None:
        bias = bias.detach()
        if bias.dtype not in (torch.bfloat16, torch.float32):
            bias = bias.float()
        bias = bias.contiguous()
    out = torch.empty(M, N, dtype=torch.float32, device=dev)
    xd = _dtype_code(x)
    with torch.cuda.device(dev):
        ws = _workspace(lib.packr_forward_decoded_workspace_bytes(M, K, N, xd), dev)
        code = lib.packr_forward_decoded(_ptr(x), xd, _ptr(Wd), _ptr(bias), _dtype_code(bias) if bias is not None else 0,
                                         _ptr(out), M, K, N, _ptr(ws), 0 if ws is None else ws.numel(), _stream(dev))
    _lib.check("packr_forward_decoded", code)
    return out


def bincount256(W_p: torch.Tensor) -> torch.Tensor:
    """int32[256] counts of the byte values of W_p (on W_p's device)."""
    lib = _lib.load()
    W_p = W_p.contiguous()
    counts = torch.empty(256, dtype=torch.int32, device=W_p.device)
    with torch.cuda.device(W_p.device):
        code = lib.packr_bincount256(_ptr(W_p), W_p.numel(), _ptr(counts), _stream(W_p.device))
    _lib.check("packr_bincount256", code)
    return counts


def decode_bf16(W_p: torch.Tensor, W_f: torch.Tensor, lut: torch.Tensor) -> torch.Tensor:
    """bf16(W_f + bf16(lut[W_p])) through the GEMM's own decode routine."""
    lib = _lib.load()
    K, N = W_p.shape
    out = torch.empty(K, N, dtype=torch.bfloat16, device=W_p.device)
    with torch.cuda.device(W_p.device):
        code = lib.packr_decode_bf16(_ptr(W_p.contiguous()), _ptr(W_f.contiguous()),
                                     _ptr(lut.detach().float().contiguous()), _ptr(out), K, N, _stream(W_p.device))
    _lib.check("packr_decode_bf16", code)
    return out


def predecode_bf16(W_p: torch.Tensor, W_f: torch.Tensor, lut: torch.Tensor) -> torch.Tensor:
    """bf16(W_f + bf16(lut[W_p])) through the streaming decode kernel that feeds
    the plain GEMMs of large batches (N % 16 == 0)."""
    lib = _lib.load()
    K, N = W_p.shape
    out = torch.empty(K, N, dtype=torch.bfloat16, device=W_p.device)
    with torch.cuda.device(W_p.device):
        code = lib.packr_predecode_bf16(_ptr(W_p.contiguous()), _ptr(W_f.contiguous()),
                                        _ptr(lut.detach().float().contiguous()), _ptr(out), K, N, _stream(W_p.device))
    _lib.check("packr_predecode_bf16", code)
    return out


def dw_split_for(x_dtype: torch.dtype) -> bool:
    if DW_PRECISION == "split":
        return True
    if DW_PRECISION == "bf16":
        return False
    return x_dtype == torch.float32


def predecode_route(M: int, K: int, N: int, W_p: torch.Tensor, W_f: torch.Tensor) -> bool:
    """True when packr_forward decodes all of W first (then a plain GEMM) for
    this problem: the forward can keep that W for the backward."""
    return bool(_lib.load().packr_predecode_route(M, K, N, _ptr(W_p), _ptr(W_f)))


def backward(dY: torch.Tensor, x: torch.Tensor, W_p: torch.Tensor, W_f: torch.Tensor, lut: torch.Tensor,
             counts: torch.Tensor | None, need_dx: bool, need_dw: bool, need_dlut: bool, need_dbias: bool,
             dW_out: torch.Tensor | None = None, Wd: torch.Tensor | None = None):
    """Returns (dX, dW_f, dlut, dbias); entries not requested are None.
    dW_out: optional contiguous bf16 [K, N] tensor the dW_f result is written
    into (for example a view of an optimizer's flat gradient buffer).
    Wd: optional W decoded by predecode_bf16 (kept from the forward); the dX
    GEMM uses it instead of decoding W again."""
    lib = _lib.load()
    x = _as_operand(x)
    M, K = x.shape
    N = W_p.shape[1]
    dev = x.device
    dY = dY.float().contiguous()
    dX = torch.empty(M, K, dtype=x.dtype, device=dev) if need_dx else None
    if need_dw and dW_out is not None:
        if (dW_out.dtype != torch.bfloat16 or tuple(dW_out.shape) != (K, N) or not dW_out.is_contiguous()
                or dW_out.device != dev):
            raise ValueError("dW_out must be a contiguous bf16 [K, N] tensor on x's device")
        dW = dW_out
    else:
        dW = torch.empty(K, N, dtype=torch.bfloat16, device=dev) if need_dw else None
    dlut = torch.empty(256, dtype=torch.float32, device=dev) if need_dlut else None
    dbias = torch.empty(N, dtype=torch.bfloat16, device=dev) if need_dbias else None
    if not (need_dx or need_dw or need_dlut or need_dbias):
        return None, None, None, None
    xd = _dtype_code(x)
    flags = _lib.PACKR_BWD_DW_SPLIT if dw_split_for(x.dtype) else 0
    with torch.cuda.device(dev):
        if Wd is not None:
            if Wd.dtype != torch.bfloat16 or tuple(Wd.shape) != (K, N) or not Wd.is_contiguous():
                raise ValueError("Wd must be the contiguous bf16 [K, N] decoded W")
            ws = _workspace(lib.packr_backward_decoded_workspace_bytes(M, K, N, xd, flags), dev)
            code = lib.packr_backward_decoded(_ptr(dY), _ptr(x), xd, _ptr(W_p), _ptr(W_f.contiguous()),
                                              _ptr(lut.detach().float().contiguous()), _ptr(Wd), _ptr(counts),
                                              _ptr(dX), _ptr(dW), _ptr(dlut), _ptr(dbias), M, K, N, flags, _ptr(ws),
                                              0 if ws is None else ws.numel(), _stream(dev))
            _lib.check("packr_backward_decoded", code)
            return dX, dW, dlut, dbias
        ws = _workspace(lib.packr_backward_workspace_bytes(M, K, N, xd, flags), dev)
        code = lib.packr_backward(_ptr(dY), _ptr(x), xd, _ptr(W_p), _ptr(W_f.contiguous()),
                                  _ptr(lut.detach().float().contiguous()), _ptr(counts), _ptr(dX), _ptr(dW),
                                  _ptr(dlut), _ptr(dbias), M, K, N, flags, _ptr(ws), 0 if ws is None else ws.numel(),
                                  _stream(dev))
    _lib.check("packr_backward", code)
    return dX, dW, dlut, dbias


def abs_order_stats(w: torch.Tensor, rank_lo: int, rank_hi: int) -> torch.Tensor:
    """[2] f32 device tensor: the rank_lo-th and rank_hi-th smallest |w|
    (0-based) of a CUDA f32/bf16 tensor (packr_abs_order_stats)."""
    lib = _lib.load()
    w = w.contiguous()
    dev = w.device
    out = torch.empty(2, dtype=torch.float32, device=dev)
    ws = torch.empty(lib.packr_abs_order_stats_workspace_bytes(), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        code = lib.packr_abs_order_stats(_ptr(w), _dtype_code(w), w.numel(), rank_lo, rank_hi, _ptr(out), _ptr(ws),
                                         ws.numel(), _stream(dev))
    _lib.check("packr_abs_order_stats", code)
    return out


def quantile_abs(w: torch.Tensor, q: float, lerp_device=None) -> torch.Tensor:
    """torch.quantile(w.abs().float(), q) (linear interpolation) for any size:
    the same rank arithmetic (f32 q * (n - 1), floor, ceil, fractional weight)
    and the same torch.lerp, over order statistics found on w's GPU by the
    library's radix select instead of a full sort.  The lerp runs on
    `lerp_device` (default: w's device): torch.quantile of a host tensor
    interpolates with the CPU kernel."""
    n = w.numel()
    pos = torch.tensor(q, dtype=torch.float32) * (n - 1)
    lo, hi = int(torch.floor(pos)), int(torch.ceil(pos))
    v = abs_order_stats(w, lo, hi)
    if lerp_device is not None:
        v = v.to(lerp_device)
    return torch.lerp(v[0], v[1], (pos - lo).to(v.device))


def half_product_multiplier(scale: torch.Tensor, dtype: torch.dtype, device=None) -> torch.Tensor:
    """The f32 multiplier torch uses in `w * scale` for a bf16 or f16 tensor
    w and a 0-dim f32 tensor `scale` on `device` (default: scale's device):
    the product is computed in f32 and rounded to w's type, with the scalar
    either kept in f32 or first rounded to w's type, which differs between
    torch's CPU and CUDA kernels; probed once per (device type, dtype) with
    torch itself."""
    dev = torch.device(device) if device is not None else scale.device
    key = (dev.type, dtype)
    mode = _HALF_SCALAR_MODE.get(key)
    if mode is None:
        g = torch.Generator(device="cpu").manual_seed(0)
        probe_w = torch.randn(4096, generator=g).to(dtype).to(dev)
        probe_s = torch.tensor(1.0 + 2 ** -8 + 2 ** -12 + 2 ** -19, dtype=torch.float32, device=dev)
        got = probe_w * probe_s
        as_f32 = (probe_w.float() * probe_s).to(dtype)
        as_half = (probe_w.float() * probe_s.to(dtype).float()).to(dtype)
        if torch.equal(got, as_f32):
            mode = "f32"
        elif torch.equal(got, as_half):
            mode = "half"
        else:
            raise RuntimeError(f"{dtype} * f32 scalar: torch's product matches neither rounding")
        _HALF_SCALAR_MODE[key] = mode
    return scale if mode == "f32" else scale.to(dtype).float()


_HALF_SCALAR_MODE: dict = {}


def from_linear_encode(weight: torch.Tensor, codebook: torch.Tensor, scale: torch.Tensor,
                       target_scale: torch.Tensor | None = None):
    """(W_p u8 [in, out], W_f bf16 [in, out], lut f32 [256]) from an
    nn.Linear weight [out, in] of f32, bf16 or f16 (packr_from_linear_encode)."""
    lib = _lib.load()
    w = weight.contiguous()
    code = {torch.float32: _lib.PACKR_DTYPE_F32, torch.bfloat16: _lib.PACKR_DTYPE_BF16,
            torch.float16: _lib.PACKR_DTYPE_F16}.get(w.dtype)
    if code is None:
        raise TypeError(f"unsupported weight dtype {w.dtype}")
    dev = w.device
    out_f, in_f = w.shape
    W_p = torch.empty(in_f, out_f, dtype=torch.uint8, device=dev)
    W_f = torch.empty(in_f, out_f, dtype=torch.bfloat16, device=dev)
    lut = torch.empty(256, dtype=torch.float32, device=dev)
    cb = codebook.to(device=dev, dtype=torch.float32).contiguous()
    sc = scale.to(device=dev, dtype=torch.float32).reshape(1).contiguous()
    ts = target_scale.to(device=dev, dtype=torch.float32).reshape(1).contiguous() if target_scale is not None else sc
    with torch.cuda.device(dev):
        rc = lib.packr_from_linear_encode(_ptr(w), code, out_f, in_f, _ptr(cb), _ptr(sc), _ptr(ts),
                                          _ptr(W_p), _ptr(W_f), _ptr(lut), _stream(dev))
    _lib.check("packr_from_linear_encode", rc)
    return W_p, W_f, lut


def packr_matmul(x, W_p, W_f, lut, bias=None):
    """PackR matmul: out = x @ (W_f + lut[W_p]) + bias  (float32 [M, N]).

    Args:
        x:    [M, K] fp32 or bf16 activations (CUDA)
        W_p:  [K, N] uint8 byte indices (contiguous)
        W_f:  [K, N] bf16 residual weights
        lut:  [256]  fp32 lookup table
        bias: [N] optional bias (bf16 or fp32)
    """
    assert x.is_cuda and W_p.is_cuda and W_f.is_cuda and lut.is_cuda
    assert W_p.dtype == torch.uint8, f"W_p must be uint8, got {W_p.dtype}"
    assert W_p.is_contiguous(), "W_p must be contiguous"
    M, K = x.shape
    K2, N = W_f.shape
    assert K2 == K, f"W_f rows ({K2}) != x cols ({K})"
    assert W_f.dtype == torch.bfloat16, f"W_f must be bf16, got {W_f.dtype}"
    assert tuple(W_p.shape) == (K, N)
    return forward(x, W_p, W_f, lut, bias)


# Legacy alias (reference packr/__init__.py:33)
phr_matmul = packr_matmul
