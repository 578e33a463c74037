"""PackRLinear on the GPU against the CPU oracle (and, at Llama-FFN sizes the
oracle cannot finish quickly, a torch fp32 GPU reference of the same math).

Bars (north_star): decoded weights bit-exact with bf16(W_f + bf16(lut[W_p]));
out / dX / dW_f / dbias within 1e-2 max-relative, dlut within 1e-3, where
max-relative = max|a-b| / max|b| as in the reference tests."""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from packr_b200 import kernel as K
from packr_b200.synthetic import linear_case

pytestmark = pytest.mark.gpu

TOL = 1e-2       # out, dX, dW_f, dbias
TOL_LUT = 1e-3   # dlut
GOLD = np.load(Path(__file__).resolve().parent / "golden" / "packr_linear_golden.npz")


def bits(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def f32(a):
    return oracle.bf16_to_f32(a) if a.dtype == np.uint16 else a.astype(np.float32)


def to_cuda(c):
    return {k: (v.cuda() if v is not None else None) for k, v in c.items()}


def run_ours(c, need=(True, True, True, True)):
    out = K.forward(c["x"], c["W_p"], c["W_f"], c["lut"], c["bias"])
    counts = K.bincount256(c["W_p"])
    dX, dW, dlut, dbias = K.backward(c["dY"], c["x"], c["W_p"], c["W_f"], c["lut"], counts, need[0], need[1],
                                     need[2], need[3] and c["bias"] is not None)
    torch.cuda.synchronize()
    return out, dX, dW, dlut, dbias


def check_against_oracle(c_cpu, label=""):
    c = to_cuda(c_cpu)
    isbf = c_cpu["x"].dtype == torch.bfloat16
    n = {k: bits(v) for k, v in c_cpu.items() if v is not None}
    ref_out = oracle.linear_forward(n["x"], n["W_p"], n["W_f"], n["lut"], n.get("bias"), x_is_bf16=isbf)
    ref = oracle.linear_backward(n["dY"], n["x"], n["W_p"], n["W_f"], n["lut"], has_bias="bias" in n,
                                 x_is_bf16=isbf)
    out, dX, dW, dlut, dbias = run_ours(c)
    errs = {"out": oracle.max_rel(bits(out), ref_out),
            "dX": oracle.max_rel(f32(bits(dX)), f32(ref["dX"])),
            "dW_f": oracle.max_rel(f32(bits(dW)), f32(ref["dW_f"])),
            "dlut": oracle.max_rel(bits(dlut), ref["dlut"])}
    if "bias" in n:
        errs["dbias"] = oracle.max_rel(f32(bits(dbias)), f32(ref["dbias"]))
    print(label, {k: f"{v:.2e}" for k, v in errs.items()})
    assert out.dtype == torch.float32 and tuple(out.shape) == ref_out.shape
    assert dX.dtype == c["x"].dtype and dW.dtype == torch.bfloat16
    for k, v in errs.items():
        assert v <= (TOL_LUT if k == "dlut" else TOL), (label, k, v)
    return errs


@pytest.mark.parametrize("shape", [(64, 256), (100, 300), (768, 3072), (3072, 768), (8, 8), (1, 5)])
def test_decode_bit_exact(cuda, shape):
    Kd, Nd = shape
    c = linear_case(1, Kd, Nd, seed=11)
    W_p, W_f, lut = c["W_p"].cuda(), c["W_f"].cuda(), c["lut"].cuda()
    got = bits(K.decode_bf16(W_p, W_f, lut))
    want = oracle.decode_bf16(bits(c["W_p"]), bits(c["W_f"]), bits(c["lut"]))
    assert np.array_equal(got, want)
    # and against torch's own bf16 arithmetic, as the reference writes it (autograd.py:66-67)
    torch_ref = bits(W_f + lut[W_p.long()].to(torch.bfloat16))
    assert np.array_equal(got, torch_ref)


def test_decode_bit_exact_extreme_lut(cuda):
    """lut entries that round to bf16 ties, subnormals, +-0, large values."""
    c = linear_case(1, 64, 512, seed=12)
    lut = torch.tensor([0.0, -0.0, 1e-40, -1e-40, 3.0e38, -3.0e38, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8] +
                       list(np.linspace(-1, 1, 248)), dtype=torch.float32)
    W_f = (torch.randn(64, 512) * 10.0).to(torch.bfloat16)
    got = bits(K.decode_bf16(c["W_p"].cuda(), W_f.cuda(), lut.cuda()))
    want = oracle.decode_bf16(bits(c["W_p"]), bits(W_f), bits(lut))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("shape", [(64, 256), (1, 16), (768, 3072), (3072, 768), (37, 4112)])
def test_predecode_bit_exact(cuda, shape):
    """The streaming decode that feeds the plain GEMMs of large batches."""
    Kd, Nd = shape
    c = linear_case(1, Kd, Nd, seed=13)
    got = bits(K.predecode_bf16(c["W_p"].cuda(), c["W_f"].cuda(), c["lut"].cuda()))
    want = oracle.decode_bf16(bits(c["W_p"]), bits(c["W_f"]), bits(c["lut"]))
    assert np.array_equal(got, want)


def test_predecode_bit_exact_extreme_lut(cuda):
    c = linear_case(1, 64, 512, seed=12)
    lut = torch.tensor([0.0, -0.0, 1e-40, -1e-40, 3.0e38, -3.0e38, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8] +
                       list(np.linspace(-1, 1, 248)), dtype=torch.float32)
    W_f = (torch.randn(64, 512) * 10.0).to(torch.bfloat16)
    got = bits(K.predecode_bf16(c["W_p"].cuda(), W_f.cuda(), lut.cuda()))
    assert np.array_equal(got, oracle.decode_bf16(bits(c["W_p"]), bits(W_f), bits(lut)))


@pytest.mark.parametrize("M,Kd,Nd,dt,bias", [(512, 1024, 512, torch.bfloat16, True), (1100, 200, 264, torch.float32, True),
                                            (1, 64, 48, torch.bfloat16, False)])
def test_forward_decoded(cuda, M, Kd, Nd, dt, bias):
    """The plain GEMM over a predecoded W against the oracle; from 129 rows on
    it is exactly what packr_forward runs after its own predecode."""
    c_cpu = linear_case(M, Kd, Nd, x_dtype=dt, bias=bias, seed=M + 7)
    c = to_cuda(c_cpu)
    n = {k: bits(v) for k, v in c_cpu.items() if v is not None}
    ref = oracle.linear_forward(n["x"], n["W_p"], n["W_f"], n["lut"], n.get("bias"), x_is_bf16=dt == torch.bfloat16)
    Wd = K.decode_bf16(c["W_p"], c["W_f"], c["lut"])
    out = K.forward_decoded(c["x"], Wd, c["bias"])
    torch.cuda.synchronize()
    assert oracle.max_rel(bits(out), ref) <= TOL
    if M >= 129 and Nd % 16 == 0:
        assert torch.equal(out, K.forward(c["x"], c["W_p"], c["W_f"], c["lut"], c["bias"]))


def test_forward_route_follows_workspace(cuda):
    """A workspace sized for the fused route (no room for the decoded W) makes
    the forward fall back to it; both routes give the same bits."""
    from packr_b200 import _lib
    lib = _lib.load()
    M, Kd, Nd = 1024, 256, 512
    c = to_cuda(linear_case(M, Kd, Nd, x_dtype=torch.bfloat16, bias=True, seed=5))
    full = lib.packr_forward_workspace_bytes(M, Kd, Nd, 1)
    assert full >= Kd * Nd * 2
    outs = []
    for ws_bytes in (full, full - Kd * Nd * 2):
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
        out = torch.empty(M, Nd, dtype=torch.float32, device="cuda")
        rc = lib.packr_forward(c["x"].data_ptr(), 1, c["W_p"].data_ptr(), c["W_f"].data_ptr(), c["lut"].data_ptr(),
                               c["bias"].data_ptr(), 1, out.data_ptr(), M, Kd, Nd, ws.data_ptr(), ws_bytes,
                               torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("n", [0, 1, 15, 16, 1000, 768 * 3072 + 3])
def test_bincount(cuda, n):
    g = torch.Generator().manual_seed(n)
    w = torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8)
    got = K.bincount256(w.cuda()).cpu().numpy()
    assert np.array_equal(got, np.bincount(w.numpy(), minlength=256))


@pytest.mark.parametrize("name", sorted(k for k in {k.split("/")[0] for k in GOLD.files} - {"cfg0"} if not k.startswith("fl_")))
def test_golden_cases(cuda, name):
    M, Kd, Nd, isbf, hasb, _, _ = (int(v) for v in GOLD[f"{name}/meta"])
    g = lambda k: GOLD[f"{name}/in_{k}"]
    t = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) if a.dtype == np.uint16 else torch.from_numpy(a.copy())
    c = {"x": t(g("x")), "W_p": t(g("W_p")), "lut": t(g("lut")), "W_f": t(g("W_f")),
         "bias": t(g("bias")) if hasb else None, "dY": t(g("dY"))}
    c["x"] = c["x"].reshape(M, Kd)
    c["dY"] = c["dY"].reshape(M, Nd)
    out, dX, dW, dlut, dbias = run_ours(to_cuda(c))
    # against the reference's own outputs
    assert oracle.max_rel(bits(out), GOLD[f"{name}/ref_out"].reshape(M, Nd)) <= TOL
    assert oracle.max_rel(f32(bits(dX)), f32(GOLD[f"{name}/ref_dX"]).reshape(M, Kd)) <= TOL
    assert oracle.max_rel(f32(bits(dW)), f32(GOLD[f"{name}/ref_dW_f"])) <= TOL
    assert oracle.max_rel(bits(dlut), GOLD[f"{name}/ref_dlut"]) <= TOL_LUT
    if hasb:
        assert oracle.max_rel(f32(bits(dbias)), f32(GOLD[f"{name}/ref_dbias"])) <= TOL


CASES = [
    # (M, K, N, x dtype, bias)
    (1024, 768, 3072, torch.float32, True),     # the 768->3072 parity configuration
    (33, 96, 160, torch.float32, True),        # ragged: partial M, K, N tiles
    (1, 64, 48, torch.bfloat16, False),        # single token
    (257, 200, 264, torch.bfloat16, True),     # K, N not multiples of 64 / 256
    (130, 100, 36, torch.float32, False),      # K % 8 != 0 (padded activation copy)
    (512, 1024, 512, torch.bfloat16, True),
    (600, 256, 512, torch.bfloat16, True),     # 512-row pair tiles: second tile's upper subtile empty
    (300, 512, 1024, torch.float32, False),    # one 512-row tile, upper subtile partial
    (1500, 320, 528, torch.bfloat16, True),    # predecode + plain GEMM, ragged M / K / N tiles
    (1100, 192, 264, torch.float32, True),     # large M but N % 16 != 0: fused register-ring route
    (1024, 2048, 9728, torch.bfloat16, True),  # stream-K split of 76 FWD tiles over 74 pairs
    (512, 1024, 5120, torch.float32, True),    # f32 x: 3 dW reduction segments
    (128, 2560, 2048, torch.bfloat16, False),  # dW: 80 tiles on 74 pairs (a second, partial wave)
    (96, 2304, 2112, torch.float32, True),     # dW: 81 tiles, the last column tile ragged (64 valid columns)
    (4096, 2560, 512, torch.bfloat16, False),  # stream-K split of 80 DX tiles over 74 pairs
    (3, 200, 264, torch.float32, True),        # few-row CUDA-core forward, row bound 4
    (9, 512, 1000, torch.bfloat16, False),     # row bound 12, 4 columns per thread
    (13, 96, 36, torch.float32, True),         # row bound 16, one K split
    (60, 1024, 2048, torch.float32, True),     # skinny tcgen05 forward, 64-token MMA width, f32 x
    (100, 640, 512, torch.bfloat16, True),     # skinny tcgen05 forward, 128-token MMA width
    (7, 640, 512, torch.bfloat16, False),      # skinny tcgen05 forward, 32-token MMA width
    (4, 512, 1024, torch.bfloat16, True),      # CUDA-core forward, 4 rows
    (1, 4096, 11008, torch.bfloat16, True),    # CUDA-core forward, clusters of 8 CTAs along K
    (2, 11008, 4096, torch.float32, True),     # clusters of 16 along K, f32 x
    (8, 300, 1000, torch.bfloat16, True),      # row bound 8, 4 columns per lane (N % 16 != 0)
    (16, 4096, 11008, torch.bfloat16, True),   # Llama-7B gate/up, decode-bound M
    (16, 11008, 4096, torch.bfloat16, True),   # Llama-7B down
    (128, 4096, 11008, torch.bfloat16, True),  # skinny dX at its 128-token bound (32 row tiles x N splits)
    (5, 11008, 4096, torch.float32, True),     # skinny dX with f32 x (dX stored as f32 of bf16)
]


@pytest.mark.parametrize("M,Kd,Nd,dt,bias", CASES)
def test_against_oracle(cuda, M, Kd, Nd, dt, bias):
    c = linear_case(M, Kd, Nd, x_dtype=dt, bias=bias, seed=M + Kd, fanin_scaled=Kd > 768)
    check_against_oracle(c, f"{M}x{Kd}x{Nd} {dt}")


def test_768x3072_matches_reference_golden(cuda):
    """The 768->3072 fp32 case against the REFERENCE's outputs (sampled)."""
    M, Kd, Nd = (int(v) for v in GOLD["cfg0/meta"][:3])
    c = to_cuda(linear_case(M, Kd, Nd, x_dtype=torch.float32, bias=True, seed=0))
    out, dX, dW, dlut, dbias = run_ours(c)
    assert oracle.max_rel(bits(dlut), GOLD["cfg0/dlut"]) <= TOL_LUT
    assert oracle.max_rel(f32(bits(dbias)), f32(GOLD["cfg0/dbias"])) <= TOL
    for k, arr in (("out", out), ("dX", dX), ("dW_f", dW)):
        flat = f32(bits(arr)).reshape(-1)
        ref = f32(GOLD[f"cfg0/{k}_val"])
        assert np.abs(flat[GOLD[f"cfg0/{k}_idx"]] - ref).max() <= TOL * np.abs(ref).max(), k


def torch_reference(c):
    """fp32 torch reference on the GPU (TF32 off) of the same math."""
    torch.backends.cuda.matmul.allow_tf32 = False
    x = c["x"].float()
    Wfull = c["W_f"].float() + c["lut"][c["W_p"].long()].half().float()
    out = x @ Wfull
    if c["bias"] is not None:
        out = out + c["bias"].float()
    Wb = (c["W_f"] + c["lut"][c["W_p"].long()].to(torch.bfloat16)).float()
    dX = (c["dY"].to(torch.bfloat16).float() @ Wb.T).to(torch.bfloat16)
    dW = x.T @ c["dY"]
    cnt = torch.bincount(c["W_p"].reshape(-1).long(), minlength=256).float()
    s = torch.zeros(256, device=x.device).scatter_add_(0, c["W_p"].reshape(-1).long(), dW.reshape(-1))
    return out, dX, dW, s / (cnt + 1e-8)


@pytest.mark.parametrize("M,Kd,Nd", [(256, 4096, 11008), (256, 11008, 4096),
                                     (4096, 4096, 11008), (4096, 11008, 4096),
                                     (16384, 4096, 11008), (16384, 11008, 4096)])
def test_llama_ffn_full_size(cuda, M, Kd, Nd):
    """The Llama-7B FFN shapes (gate/up 4096 -> 11008, down 11008 -> 4096) at
    the sweep's many-row token counts: 256 (the fused-decode GEMM route),
    4096 and 16384 (the predecode route), against the fp32 torch reference."""
    c = to_cuda(linear_case(M, Kd, Nd, x_dtype=torch.bfloat16, bias=False, seed=1, device="cpu", fanin_scaled=True))
    out, dX, dW, dlut, _ = run_ours(c)
    r_out, r_dX, r_dW, r_dlut = torch_reference(c)
    mr = lambda a, b: ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()
    errs = {"out": mr(out, r_out), "dX": mr(dX, r_dX), "dW_f": mr(dW, r_dW), "dlut": mr(dlut, r_dlut)}
    print(errs)
    assert errs["out"] <= TOL and errs["dX"] <= TOL and errs["dW_f"] <= TOL and errs["dlut"] <= TOL_LUT
    # size-independent property: the bf16 dW_f is the rounding of an fp32 sum
    # whose bin sums reproduce dlut * (count + 1e-8)
    cnt = torch.bincount(c["W_p"].reshape(-1).long(), minlength=256).float()
    assert torch.allclose(dlut * (cnt + 1e-8), r_dlut * (cnt + 1e-8), rtol=0, atol=TOL_LUT * (r_dlut * cnt).abs().max().item())


def test_empty_batch(cuda):
    c = to_cuda(linear_case(1, 64, 32, seed=3))
    x = c["x"][:0]
    out = K.forward(x, c["W_p"], c["W_f"], c["lut"], c["bias"])
    assert out.shape == (0, 32)
    dX, dW, dlut, dbias = K.backward(c["dY"][:0], x, c["W_p"], c["W_f"], c["lut"], None, True, True, True, True)
    torch.cuda.synchronize()
    assert dX.shape == (0, 64) and (dW.float() == 0).all() and (dlut == 0).all() and (dbias.float() == 0).all()


@pytest.mark.parametrize("M,Kd,Nd,dt", [(1024, 768, 3072, torch.bfloat16), (1500, 320, 528, torch.float32),
                                        (4096, 256, 512, torch.bfloat16)])
def test_backward_with_forward_decoded_w(cuda, M, Kd, Nd, dt):
    """packr_backward_decoded with the forward's decoded W gives the same
    gradients as packr_backward decoding W itself (dlut and dbias: the same
    sums added by atomics in a run-dependent order)."""
    c = to_cuda(linear_case(M, Kd, Nd, x_dtype=dt, bias=True, seed=M + 3))
    assert K.predecode_route(M, Kd, Nd, c["W_p"], c["W_f"])
    Wd = K.predecode_bf16(c["W_p"], c["W_f"], c["lut"])
    counts = K.bincount256(c["W_p"])
    a = K.backward(c["dY"], c["x"], c["W_p"], c["W_f"], c["lut"], counts, True, True, True, True)
    b = K.backward(c["dY"], c["x"], c["W_p"], c["W_f"], c["lut"], counts, True, True, True, True, Wd=Wd)
    torch.cuda.synchronize()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert torch.allclose(a[2], b[2], rtol=1e-5, atol=1e-6 * a[2].abs().max().item())
    assert torch.allclose(a[3].float(), b[3].float(), rtol=2 ** -7, atol=0)


def test_layer_keeps_decoded_w_for_backward(cuda, monkeypatch):
    """With PACKR_KEEP_DECODED_W=1, PackRLinear on the many-row route decodes
    W once per step: forward and gradients equal the explicit forward +
    backward."""
    from packr_b200 import PackRLinear, autograd
    monkeypatch.setattr(autograd, "KEEP_DECODED_W", True)
    M, Kd, Nd = 1024, 512, 1024
    c = to_cuda(linear_case(M, Kd, Nd, x_dtype=torch.bfloat16, bias=True, seed=21))
    layer = PackRLinear(Kd, Nd).to("cuda")
    with torch.no_grad():
        layer.W_p.copy_(c["W_p"]); layer.W_f.copy_(c["W_f"]); layer.lut.copy_(c["lut"]); layer.bias_f.copy_(c["bias"])
    x = c["x"].clone().requires_grad_(True)
    out = layer(x)
    out.backward(c["dY"])
    ref_out = K.forward(c["x"], c["W_p"], c["W_f"], c["lut"], c["bias"])
    dX, dW, dlut, dbias = K.backward(c["dY"], c["x"], c["W_p"], c["W_f"], c["lut"], K.bincount256(c["W_p"]),
                                     True, True, True, True)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    assert torch.equal(x.grad, dX) and torch.equal(layer.W_f.grad, dW)
    assert torch.allclose(layer.bias_f.grad.float(), dbias.float(), rtol=2 ** -7, atol=0)
    assert torch.allclose(layer.lut.grad, dlut, rtol=1e-5, atol=1e-6 * dlut.abs().max().item())


def test_no_decoded_weight_held_between_forward_and_backward(cuda):
    """By default a PackRLinear holds only its packed weights from forward to
    backward (the memory budget of the reference's VRAM regression tests,
    tests/test_vram_regression.py:33-77, at the Llama-7B gate shape and the
    many-row route): what the forward leaves allocated is its output, not a
    decoded [K, N] bf16 W (90 MB here)."""
    from packr_b200 import PackRLinear, autograd
    assert not autograd.KEEP_DECODED_W
    M, Kd, Nd = 4096, 4096, 11008
    lay = PackRLinear.synthetic(Kd, Nd, bias=False, device=cuda, seed=1, lut_std=0.01, wf_std=0.001)
    x = torch.randn(M, Kd, device=cuda).to(torch.bfloat16).requires_grad_(True)
    lay.lut_counts()
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    out = lay(x)
    torch.cuda.synchronize()
    held = torch.cuda.memory_allocated() - base
    wd_bytes = Kd * Nd * 2
    assert held <= out.numel() * out.element_size() + wd_bytes // 8, held
    out.backward(torch.randn_like(out))
    torch.cuda.synchronize()
    assert lay.W_f.grad is not None and x.grad is not None


def _dlut_case(M, Kd, Nd, seed, x_scale_rows=None, x_scale=1.0, x_dtype=torch.float32):
    c = linear_case(M, Kd, Nd, x_dtype=torch.float32, bias=False, seed=seed)
    x = c["x"] * x_scale
    if x_scale_rows is not None:
        x = x * x_scale_rows[None, :]
    c["x"] = x.to(x_dtype)
    if x_dtype == torch.bfloat16:
        c["dY"] = c["dY"].to(torch.bfloat16).float()
    return c


def _dlut_of(c_cpu):
    c = to_cuda(c_cpu)
    counts = K.bincount256(c["W_p"])
    _, _, dlut, _ = K.backward(c["dY"], c["x"], c["W_p"], c["W_f"], c["lut"], counts, False, False, True, False)
    torch.cuda.synchronize()
    n = {k: bits(v) for k, v in c_cpu.items() if v is not None}
    ref = oracle.linear_backward(n["dY"], n["x"], n["W_p"], n["W_f"], n["lut"], has_bias=False,
                                 x_is_bf16=c_cpu["x"].dtype == torch.bfloat16)
    return bits(dlut), ref["dlut"]


@pytest.mark.parametrize("M,Kd,Nd", [(64, 512, 768), (1, 1024, 1024)])
def test_dlut_tiles_of_very_different_magnitude(cuda, M, Kd, Nd):
    """The lut gradient's histogram scales each dW tile by its own largest
    value: tiles (128-row blocks of K) whose magnitudes differ by up to
    2^+-30 each keep their precision, bin by bin (error against the bin's
    sum of |dW| terms, the scale of an f32 accumulation's error)."""
    scales = torch.tensor([2.0 ** (30 * ((k // 128) % 3 - 1)) for k in range(Kd)], dtype=torch.float32)
    c = _dlut_case(M, Kd, Nd, seed=3, x_scale_rows=scales)
    got, ref = _dlut_of(c)
    n = {k: bits(v) for k, v in c.items() if v is not None}
    dW = n["x"].astype(np.float64).T @ n["dY"].astype(np.float64)
    w = n["W_p"].reshape(-1).astype(np.int64)
    cnt = np.bincount(w, minlength=256).astype(np.float64)
    abs_sum = np.bincount(w, weights=np.abs(dW).reshape(-1), minlength=256) / (cnt + 1e-8)
    assert oracle.max_rel(got, ref) <= TOL_LUT
    assert np.all(np.abs(got.astype(np.float64) - ref) <= 1e-5 * abs_sum + 1e-30)


@pytest.mark.parametrize("x_scale", [1e-36, 1e30])
def test_dlut_extreme_magnitudes(cuda, x_scale):
    """Tiles whose values all lie below 2^-106 (added in f32 directly) and
    near the top of the f32 range (scaled down by the tile exponent)."""
    c = _dlut_case(96, 256, 512, seed=4, x_scale=x_scale)
    got, ref = _dlut_of(c)
    assert np.all(np.isfinite(got)) and oracle.max_rel(got, ref) <= TOL_LUT


def test_dlut_non_finite_gradient(cuda):
    """An Inf in dY (bf16 x): the bins holding the affected dW entries become
    Inf or NaN exactly where the oracle's f32 sums do; the other bins stay
    within tolerance."""
    c = _dlut_case(64, 384, 640, seed=5, x_dtype=torch.bfloat16)
    c["dY"][7, 100] = float("inf")
    got, ref = _dlut_of(c)
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(got), fin)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.sign(got[~np.isnan(ref) & ~fin]), np.sign(ref[~np.isnan(ref) & ~fin]))
    assert oracle.max_rel(got[fin], ref[fin]) <= TOL_LUT
