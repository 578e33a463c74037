"""Generates tests/golden/packr_linear_golden.npz by running the REFERENCE
package's own PackRLinear forward/backward on the CPU.

    PACKR_REFERENCE_ROOT=<reference tree> python tests/golden/make_golden.py

The reference's packr_matmul asserts CUDA tensors (packr/kernel.py:117); this
script runs that same function with only the assert line removed and with the
reference's own torch decode backend (_kernel_loader._fallback_decode, which
is what the reference uses when no Triton/CUDA decoder is available).  All
other arithmetic is the reference's: PackRLinear.forward (layer.py:78-101),
PackRMatmulFunction (autograd.py:33-88), torch CPU GEMMs.

Small cases are stored whole.  For the 768->3072, M=1024 fp32 case the inputs
are regenerated from the seed by the test (packr_b200.synthetic.linear_case);
its dlut and dbias are stored whole, out/dX/dW_f as float64 sums plus 4096
sampled entries each.
"""
from __future__ import annotations

import inspect
import os
import sys
from pathlib import Path

import numpy as np
import torch

if not os.environ.get("PACKR_REFERENCE_ROOT"):
    raise SystemExit("set PACKR_REFERENCE_ROOT to the reference tree (the directory holding packr/)")
REF = Path(os.environ["PACKR_REFERENCE_ROOT"])
REPO = Path(__file__).resolve().parents[2]
sys.dont_write_bytecode = True
sys.path.insert(0, str(REF))
sys.path.insert(1, str(REPO))

import packr  # noqa: E402  (the reference package)
import packr.autograd  # noqa: E402
import packr.kernel  # noqa: E402
from packr._kernel_loader import _fallback_decode  # noqa: E402

from packr_b200.synthetic import linear_case  # noqa: E402


def _cpu_packr_matmul():
    src = inspect.getsource(packr.kernel.packr_matmul)
    line = "assert x.is_cuda and W_p.is_cuda and W_f.is_cuda and lut.is_cuda"
    assert line in src
    ns = dict(vars(packr.kernel))
    exec(src.replace(line, "pass"), ns)
    return ns["packr_matmul"]


packr.kernel._decode_fn = _fallback_decode
packr.autograd.packr_matmul = _cpu_packr_matmul()


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def run_reference(case: dict, three_d: bool = False) -> dict:
    K, N = case["W_p"].shape
    layer = packr.PackRLinear(K, N, bias=case["bias"] is not None)
    with torch.no_grad():
        layer.W_p.data = case["W_p"].clone()
        layer.W_f.data = case["W_f"].clone()
        layer.lut.data = case["lut"].clone()
        if case["bias"] is not None:
            layer.bias_f.data = case["bias"].clone()
    layer.lut.requires_grad_(True)
    x = case["x"].clone()
    if three_d:
        x = x.reshape(2, -1, K)
    x.requires_grad_(True)
    out = layer(x)
    dY = case["dY"].reshape(out.shape)
    out.backward(dY)
    res = {"out": bits(out.reshape(-1, N)), "dX": bits(x.grad.reshape(-1, K)), "dW_f": bits(layer.W_f.grad),
           "dlut": bits(layer.lut.grad)}
    if case["bias"] is not None:
        res["dbias"] = bits(layer.bias_f.grad)
    return res


SMALL = {  # name: (M, K, N, x dtype, bias, 3-D input)
    "f32_ragged": (33, 96, 160, torch.float32, True, False),
    "bf16_tiles": (64, 128, 256, torch.bfloat16, True, False),
    "bf16_m1": (1, 64, 48, torch.bfloat16, False, False),
    "f32_3d": (16, 64, 32, torch.float32, True, True),
}


def main() -> None:
    out = {}
    for name, (M, K, N, dt, bias, three_d) in SMALL.items():
        case = linear_case(M, K, N, x_dtype=dt, bias=bias, seed=7)
        ref = run_reference(case, three_d)
        out[f"{name}/meta"] = np.array([M, K, N, int(dt == torch.bfloat16), int(bias), int(three_d), 7], np.int64)
        for k in ("x", "W_p", "lut", "W_f", "bias", "dY"):
            if case[k] is not None:
                out[f"{name}/in_{k}"] = bits(case[k])
        for k, v in ref.items():
            out[f"{name}/ref_{k}"] = v
    # 768 -> 3072, M = 1024, fp32, seed 0
    M, K, N = 1024, 768, 3072
    case = linear_case(M, K, N, x_dtype=torch.float32, bias=True, seed=0)
    ref = run_reference(case)
    rng = np.random.default_rng(12345)
    out["cfg0/meta"] = np.array([M, K, N, 0, 1, 0, 0], np.int64)
    out["cfg0/dlut"] = ref["dlut"]
    out["cfg0/dbias"] = ref["dbias"]
    for k, shape in (("out", (M, N)), ("dX", (M, K)), ("dW_f", (K, N))):
        arr = ref[k]
        f = arr.astype(np.float32) if arr.dtype != np.uint16 else (arr.astype(np.uint32) << 16).view(np.float32)
        idx = rng.integers(0, arr.size, 4096)
        out[f"cfg0/{k}_idx"] = idx.astype(np.int64)
        out[f"cfg0/{k}_val"] = arr.reshape(-1)[idx]
        out[f"cfg0/{k}_sum"] = np.array([f.astype(np.float64).sum(), np.abs(f.astype(np.float64)).sum()])
    # inputs checksum so a changed generator is caught
    out["cfg0/in_checksum"] = np.array([case["x"].double().sum().item(), case["W_p"].double().sum().item(),
                                        case["lut"].double().sum().item(), case["W_f"].double().sum().item(),
                                        case["dY"].double().sum().item()])
    # from_linear: the reference's compression of seeded nn.Linear layers
    for name, (i, o, b) in {"fl_small": (64, 48, True), "fl_wide": (96, 320, False)}.items():
        torch.manual_seed(21 + i)
        lin = torch.nn.Linear(i, o, bias=b)
        pl = packr.PackRLinear.from_linear(lin)
        out[f"{name}/weight"] = lin.weight.detach().numpy().copy()
        if b:
            out[f"{name}/bias"] = lin.bias.detach().numpy().copy()
            out[f"{name}/bias_f"] = bits(pl.bias_f)
        out[f"{name}/W_p"] = bits(pl.W_p)
        out[f"{name}/lut"] = bits(pl.lut)
        out[f"{name}/W_f"] = bits(pl.W_f)
    dst = Path(__file__).resolve().parent / "packr_linear_golden.npz"
    np.savez_compressed(dst, **out)
    print(dst, dst.stat().st_size)


if __name__ == "__main__":
    main()
