"""packr_backward_static_scratch — the backward for callers that cannot
allocate device memory (its scratch is a static device array inside the
library) — against packr_backward with a caller-allocated workspace, through
the C ABI, on two calls in a row (the second call finds the previous call's
contents in the shared array).  This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from packr_b200 import _lib
from packr_b200.synthetic import linear_case

pytestmark = pytest.mark.gpu

TOL, TOL_LUT = 1e-2, 1e-3
STATIC_BYTES = 32 << 20


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _f32(t):
    return t.detach().float().cpu().numpy()


def _run(lib, c, static, flags):
    x = c["x"]
    M, K = x.shape
    N = c["W_p"].shape[1]
    xd = _lib.PACKR_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.PACKR_DTYPE_F32
    counts = torch.bincount(c["W_p"].reshape(-1).long(), minlength=256).to(torch.int32)
    dX = torch.full((M, K), float("nan"), dtype=x.dtype, device="cuda")
    dW = torch.full((K, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    dlut = torch.full((256,), float("nan"), device="cuda")
    dbias = torch.full((N,), float("nan"), dtype=torch.bfloat16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (_p(c["dY"]), _p(x), xd, _p(c["W_p"]), _p(c["W_f"]), _p(c["lut"]), _p(counts), _p(dX), _p(dW), _p(dlut),
            _p(dbias), M, K, N, flags)
    if static:
        rc = lib.packr_backward_static_scratch(*args, stream)
    else:
        ws = torch.empty(lib.packr_backward_workspace_bytes(M, K, N, xd, flags), dtype=torch.uint8, device="cuda")
        rc = lib.packr_backward(*args, _p(ws), ws.numel(), stream)
    torch.cuda.synchronize()
    assert rc == 0, (static, rc)
    return dX, dW, dlut, dbias


@pytest.mark.parametrize("dtype,flags", [(torch.bfloat16, 0), (torch.float32, _lib.PACKR_BWD_DW_SPLIT)])
def test_static_scratch_matches_workspace_backward(cuda, dtype, flags):
    lib = _lib.load()
    for call in range(2):  # two calls in a row share (and find stale data in) the static array
        c = {k: (v.cuda() if v is not None else None)
             for k, v in linear_case(192 + 64 * call, 512, 768, x_dtype=dtype, bias=True, seed=call).items()}
        want = _run(lib, c, static=False, flags=flags)
        got = _run(lib, c, static=True, flags=flags)
        for i, (g, w) in enumerate(zip(got, want)):
            assert torch.isfinite(g.float()).all(), (call, i)
            assert oracle.max_rel(_f32(g), _f32(w)) <= (TOL_LUT if i == 2 else TOL), (call, i)


def _bf16_need(M, K, N, pre, sk_bytes=0):
    """Scratch bytes of the backward for bf16 x (K % 8 == 0), no split, every
    gradient wanted, lut counts given: the carve of packr_backward (256-byte
    aligned pieces: [decoded W, stream-K slots,] bf16 dY, bias sums, lut
    sums)."""
    a = lambda v: (v + 255) // 256 * 256
    r8 = lambda v: (v + 7) // 8 * 8
    need = (a(K * N * 2) + a(sk_bytes) if pre else 0) + a(M * r8(N) * 2) + a(N * 4) + a(256 * 4)
    return need


@pytest.mark.parametrize("M,K,N,route,near_limit", [
    (1024, 1024, 1024, "decode-first", False),  # dX from W decoded into the static array
    (1024, 3584, 3584, "decode-first", True),   # decoded W + bf16 dY just under the array's size
    (4000, 512, 4096, "fused", True),           # bf16 dY alone just under it: dX decodes W in shared memory
])
def test_static_scratch_routes_near_the_limit(cuda, M, K, N, route, near_limit):
    """The large-row shapes, where the backward picks its dX route by what
    fits in the array, on two calls in a row against the workspace
    backward (bf16 x, no split)."""
    pre_need = _bf16_need(M, K, N, pre=True)
    assert (pre_need <= STATIC_BYTES) == (route == "decode-first")
    used = pre_need if route == "decode-first" else _bf16_need(M, K, N, pre=False)
    assert used <= STATIC_BYTES and (used > 0.95 * STATIC_BYTES) == near_limit
    lib = _lib.load()
    for call in range(2):
        c = {k: (v.cuda() if v is not None else None)
             for k, v in linear_case(M, K, N, x_dtype=torch.bfloat16, bias=True, seed=10 + call,
                                     fanin_scaled=True).items()}
        want = _run(lib, c, static=False, flags=0)
        got = _run(lib, c, static=True, flags=0)
        for i, (g, w) in enumerate(zip(got, want)):
            assert torch.isfinite(g.float()).all(), (call, i)
            assert oracle.max_rel(_f32(g), _f32(w)) <= (TOL_LUT if i == 2 else TOL), (call, i)


def test_static_scratch_rejects_oversized_problems(cuda):
    lib = _lib.load()
    M, K, N = 4096, 64, 8192  # bf16(dY) alone needs 64 MiB > the 32 MiB array
    assert M * N * 2 > STATIC_BYTES
    c = {k: (v.cuda() if v is not None else None)
         for k, v in linear_case(8, K, N, x_dtype=torch.bfloat16, bias=False, seed=1).items()}
    dY = torch.zeros(M, N, device="cuda")
    x = torch.zeros(M, K, dtype=torch.bfloat16, device="cuda")
    dW = torch.zeros(K, N, dtype=torch.bfloat16, device="cuda")
    rc = lib.packr_backward_static_scratch(_p(dY), _p(x), _lib.PACKR_DTYPE_BF16, _p(c["W_p"]), _p(c["W_f"]),
                                           _p(c["lut"]), None, None, _p(dW), None, None, M, K, N, 0,
                                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 4  # PACKR_ERR_WORKSPACE: beyond the static maximum, nothing launched
    assert (dW.float() == 0).all()
