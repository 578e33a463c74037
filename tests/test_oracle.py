"""The CPU oracle against golden vectors made by the reference itself:
tests/golden/packr_linear_golden.npz (reference PackRLinear on CPU, made by
tests/golden/make_golden.py) and tests/golden/adam8_golden.npz (reference CUDA
8-bit AdamW kernel built from source, made by make_adam_golden.py)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from packr_b200.synthetic import adam_grad, adam_params, linear_case

GOLD = Path(__file__).resolve().parent / "golden"
LIN = np.load(GOLD / "packr_linear_golden.npz")
SMALL = sorted(k for k in {k.split("/")[0] for k in LIN.files} - {"cfg0"} if not k.startswith("fl_"))


def _f(a):
    return oracle.bf16_to_f32(a) if a.dtype == np.uint16 else a.astype(np.float32)


@pytest.mark.parametrize("name", SMALL)
def test_linear_oracle_matches_reference(name):
    M, K, N, isbf, hasb, _, _ = LIN[f"{name}/meta"]
    g = lambda k: LIN[f"{name}/in_{k}"]
    b = g("bias") if hasb else None
    out = oracle.linear_forward(g("x"), g("W_p"), g("W_f"), g("lut"), b, x_is_bf16=bool(isbf))
    bw = oracle.linear_backward(g("dY"), g("x"), g("W_p"), g("W_f"), g("lut"), has_bias=bool(hasb),
                                x_is_bf16=bool(isbf))
    # Same arithmetic as the reference; only fp32 summation order may differ.
    assert oracle.max_rel(out, LIN[f"{name}/ref_out"]) < 1e-6
    for k in ["dX", "dW_f", "dlut"] + (["dbias"] if hasb else []):
        ref = LIN[f"{name}/ref_{k}"]
        assert bw[k].dtype == ref.dtype and bw[k].shape == ref.reshape(bw[k].shape).shape
        assert oracle.max_rel(_f(bw[k]), _f(ref).reshape(bw[k].shape)) < 1e-3, k
        # bf16 results: at most a handful of 1-ulp flips from summation order
        if ref.dtype == np.uint16:
            assert (bw[k].reshape(-1) != ref.reshape(-1)).mean() < 1e-3


def test_linear_oracle_matches_reference_768x3072():
    M, K, N = (int(v) for v in LIN["cfg0/meta"][:3])
    c = linear_case(M, K, N, x_dtype=torch.float32, bias=True, seed=0)
    chk = np.array([c["x"].double().sum().item(), c["W_p"].double().sum().item(), c["lut"].double().sum().item(),
                    c["W_f"].double().sum().item(), c["dY"].double().sum().item()])
    assert np.allclose(chk, LIN["cfg0/in_checksum"], rtol=0, atol=1e-6), "seeded generator changed"
    n = {k: (v.numpy() if v.dtype != torch.bfloat16 else v.view(torch.int16).numpy().view(np.uint16))
         for k, v in c.items() if v is not None}
    out = oracle.linear_forward(n["x"], n["W_p"], n["W_f"], n["lut"], n["bias"])
    bw = oracle.linear_backward(n["dY"], n["x"], n["W_p"], n["W_f"], n["lut"], has_bias=True)
    assert oracle.max_rel(bw["dlut"], LIN["cfg0/dlut"]) < 1e-4
    assert oracle.max_rel(_f(bw["dbias"]), _f(LIN["cfg0/dbias"])) < 1e-2
    for k, arr in (("out", out), ("dX", bw["dX"]), ("dW_f", bw["dW_f"])):
        flat = _f(arr).reshape(-1)
        idx = LIN[f"cfg0/{k}_idx"]
        ref = _f(LIN[f"cfg0/{k}_val"])
        assert np.abs(flat[idx] - ref).max() <= 1e-3 * np.abs(ref).max(), k
        s = LIN[f"cfg0/{k}_sum"]
        assert abs(flat.astype(np.float64).sum() - s[0]) <= 1e-4 * s[1], k


def test_decode_definitions():
    c = linear_case(8, 16, 24, seed=3)
    Wp = c["W_p"].numpy()
    Wf = c["W_f"].view(torch.int16).numpy().view(np.uint16)
    lut = c["lut"].numpy()
    ref_bf16 = (c["W_f"] + c["lut"][c["W_p"].long()].to(torch.bfloat16)).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.decode_bf16(Wp, Wf, lut), ref_bf16)
    ref_f32 = (c["W_f"] + c["lut"][c["W_p"].long()].to(torch.float16)).numpy()
    assert np.array_equal(oracle.decode_f32(Wp, Wf, lut), ref_f32)


ADAM = GOLD / "adam8_golden.npz"


@pytest.mark.skipif(not ADAM.exists(), reason="adam8_golden.npz not generated yet")
def test_adam_oracle_matches_reference_cuda_kernel():
    z = np.load(ADAM)
    names = sorted({k.split("/")[0] for k in z.files})
    assert names
    for name in names:
        n, isbf, steps = (int(v) for v in z[f"{name}/meta"])
        lr, wd, gstd, b1, b2, eps = (float(v) for v in z[f"{name}/hyper"])
        p = z[f"{name}/p0"].copy()
        m = np.zeros(n, np.int8)
        v = np.zeros(n, np.int8)
        nb = (n + 255) // 256
        ms = np.ones(nb, np.float32)
        vs = np.ones(nb, np.float32)
        for s in range(1, steps + 1):
            g = z[f"{name}/g{s}"]
            bc1, bc2 = oracle.adam8_bias_corrections(b1, b2, s)
            oracle.adam8_step(p, g, m, v, ms, vs, lr, b1, b2, eps, bc1, bc2, wd)
            assert np.array_equal(ms, z[f"{name}/ms{s}"]), (name, s)
            assert np.array_equal(vs, z[f"{name}/vs{s}"]), (name, s)
            assert np.array_equal(m, z[f"{name}/m{s}"]), (name, s)
            assert np.array_equal(v, z[f"{name}/v{s}"]), (name, s)
            assert np.array_equal(p, z[f"{name}/p{s}"]), (name, s)


def test_adam_oracle_invariants():
    n = 1000
    p = adam_params(n, dtype=torch.float32, seed=1).numpy()
    m = np.zeros(n, np.int8); v = np.zeros(n, np.int8)
    ms = np.ones(4, np.float32); vs = np.ones(4, np.float32)
    for s in range(1, 4):
        g = adam_grad(n, s, dtype=torch.float32).numpy()
        oracle.adam8_step(p, g, m, v, ms, vs, 1e-3, .9, .999, 1e-8, *oracle.adam8_bias_corrections(.9, .999, s), 0.0)
        assert v.min() >= 1 and v.max() <= 127 and m.min() >= -127 and m.max() <= 127
        assert (ms >= 1e-14).all() and (vs >= 1e-14).all()
        # each block's absmax code is +-127 (unless the block is all zero)
        for b in range(4):
            assert np.abs(m[b * 256:(b + 1) * 256]).max() == 127


def test_adam_oracle_tracks_fp32_adamw():
    """The reference's statistical check (tests/test_cuda_adam.py:24-130) on the
    oracle: first-step update-norm ratio in (0.8, 1.2), min cosine > 0.95."""
    torch.manual_seed(42)
    w = (torch.randn(64, 128) * 0.01)
    torch.manual_seed(123)
    grads = [torch.randn(64, 128) * 0.1 for _ in range(50)]
    p_ref = torch.nn.Parameter(w.clone())
    opt = torch.optim.AdamW([p_ref], lr=2e-5)
    p = w.clone().numpy().reshape(-1)
    n = p.size
    m = np.zeros(n, np.int8); v = np.zeros(n, np.int8)
    ms = np.ones((n + 255) // 256, np.float32); vs = ms.copy()
    ratios, cos = [], []
    for s, g in enumerate(grads, 1):
        p_ref.grad = g.clone()
        opt.step()
        oracle.adam8_step(p, g.numpy().reshape(-1).copy(), m, v, ms, vs, 2e-5, .9, .999, 1e-8,
                          *oracle.adam8_bias_corrections(.9, .999, s), 0.0)
        u_ref = (p_ref.detach() - w).reshape(-1)
        u = torch.from_numpy(p) - w.reshape(-1)
        ratios.append((u.norm() / u_ref.norm()).item())
        cos.append(torch.nn.functional.cosine_similarity(u_ref[None], u[None]).item())
    assert 0.8 < ratios[0] < 1.2
    assert min(cos) > 0.95
