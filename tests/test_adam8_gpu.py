"""8-bit AdamW on the GPU (packr_adam8_multi through the C ABI / CUDA8BitAdam):
bit-exact against the C oracle, against the reference CUDA kernel compiled
from its source (codes within +-1, params within 1e-6 relative, the stated
bar), and the reference's own statistical checks (tests/test_cuda_adam.py)."""
import importlib.util

import numpy as np
import pytest
import torch

import oracle
from packr_b200.cuda_adam import CUDA8BitAdam, adam8_launch
from packr_b200.synthetic import adam_grad, adam_params
from conftest import REPO

pytestmark = pytest.mark.gpu


def np_bits(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def new_state(n, dev="cuda"):
    nb = (n + 255) // 256
    return (torch.zeros(n, dtype=torch.int8, device=dev), torch.zeros(n, dtype=torch.int8, device=dev),
            torch.ones(nb, device=dev), torch.ones(nb, device=dev))


def test_rounding_selfcheck(cuda):
    """The kernel's short correctly rounded reciprocal / square root /
    quotient / update sequences equal CUDA's IEEE operations: exhaustively
    over their argument ranges for the reciprocal and the square root, on
    2^30 pseudo-random cases for the quotient and the whole update."""
    from packr_b200.cuda_adam import selfcheck_rounding
    assert selfcheck_rounding(cuda) == [0, 0, 0, 0]


def _special_grads(n, step, dtype, nonfinite):
    """Gradients with exact zeros, tiny and huge values (and, with
    `nonfinite`, Inf and NaN) in some blocks: those blocks take the kernel's
    IEEE path."""
    g = adam_grad(n, step, dtype=dtype, device="cuda", std=1e-2).clone()
    if step == 1:
        g[0:300] = 0                 # zero moments
    g[700] = 1e-30                   # moments below the fast path's range
    g[1300] = 3e18                   # v above it
    if nonfinite and step == 3:
        g[2000] = float("inf")
        g[2600] = float("nan")
    return g


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("nonfinite", [False, True])
def test_special_values_vs_oracle(cuda, dtype, nonfinite):
    """Blocks outside the fast path's ranges equal the oracle bit for bit.
    With Inf/NaN gradients the codes and scales still do; the parameters are
    compared where the oracle's are finite (a NaN's bits are the CPU's or the
    GPU's own)."""
    n = 4096 + 77
    p = adam_params(n, dtype=dtype, seed=5, device="cuda")
    st = new_state(n)
    hp, hm, hv, hms, hvs = np_bits(p), *[np_bits(t) for t in st]
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.999, 1e-8, 0.01
    for s in range(1, 5):
        bc1, bc2 = oracle.adam8_bias_corrections(b1, b2, s)
        g = _special_grads(n, s, dtype, nonfinite)
        adam8_launch([(p, g, *st)], lr, b1, b2, eps, bc1, bc2, wd)
        torch.cuda.synchronize()
        oracle.adam8_step(hp, np_bits(g), hm, hv, hms, hvs, lr, b1, b2, eps, bc1, bc2, wd)
        assert np.array_equal(np_bits(st[2]).view(np.uint32), hms.view(np.uint32)), s
        assert np.array_equal(np_bits(st[3]).view(np.uint32), hvs.view(np.uint32)), s
        assert np.array_equal(np_bits(st[0]), hm), s
        assert np.array_equal(np_bits(st[1]), hv), s
        got = np_bits(p)
        if not nonfinite:
            assert np.array_equal(got, hp), s
        else:
            fin = np.isfinite(torch.from_numpy(hp.view(np.int16)).view(torch.bfloat16).float().numpy()
                              if dtype == torch.bfloat16 else hp)
            assert np.array_equal(got[fin], hp[fin]), s


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_zero_first_moments_vs_oracle(cuda, dtype):
    """Exact zero gradients on zero m codes give first moments of exactly 0
    in about half of the blocks (as rank-averaged gradients that cancel do);
    those blocks take the fast sequences with the zero update, and every
    code, scale and parameter (some of them -0) equals the oracle bit for
    bit."""
    n = 65536 + 300
    p = adam_params(n, dtype=dtype, seed=21, device="cuda")
    p[5::97] = -0.0
    st = new_state(n)
    hp, hm, hv, hms, hvs = np_bits(p), *[np_bits(t) for t in st]
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.999, 1e-8, 0.01
    keep = torch.Generator(device="cpu").manual_seed(3)
    for s in range(1, 7):
        bc1, bc2 = oracle.adam8_bias_corrections(b1, b2, s)
        g = adam_grad(n, s, dtype=dtype, device="cuda", std=1e-2).clone()
        if s > 1:
            g[(torch.rand(n, generator=keep) < 0.3).to("cuda")] = 0
        adam8_launch([(p, g, *st)], lr, b1, b2, eps, bc1, bc2, wd)
        torch.cuda.synchronize()
        oracle.adam8_step(hp, np_bits(g), hm, hv, hms, hvs, lr, b1, b2, eps, bc1, bc2, wd)
        assert np.array_equal(np_bits(st[2]).view(np.uint32), hms.view(np.uint32)), s
        assert np.array_equal(np_bits(st[3]).view(np.uint32), hvs.view(np.uint32)), s
        assert np.array_equal(np_bits(st[0]), hm), s
        assert np.array_equal(np_bits(st[1]), hv), s
        assert np.array_equal(np_bits(p), hp), s
    m = torch.from_numpy(hm.astype(np.int32))
    assert int((m == 0).sum()) > 100  # the case occurred


@pytest.mark.parametrize("wd", [0.0, 0.01])
def test_multi_tensor_bit_exact_vs_oracle(cuda, wd):
    sizes = [1, 7, 255, 256, 257, 4096 + 13, 3 * 256, 100_003]
    dtypes = [torch.bfloat16, torch.float32] * 4
    big = adam_params(20_000, dtype=torch.bfloat16, seed=9, device="cuda")
    params = [adam_params(n, dtype=dt, seed=i, device="cuda") for i, (n, dt) in enumerate(zip(sizes, dtypes))]
    # an unaligned view (element offset 3 of a bf16 buffer): exercises the scalar path
    params.append(big[3:3 + 5000])
    states = [new_state(p.numel()) for p in params]
    host = [(np_bits(p), *[np_bits(t) for t in st]) for p, st in zip(params, states)]
    lr, b1, b2, eps = 1e-3, 0.9, 0.999, 1e-8
    for s in range(1, 6):
        bc1, bc2 = oracle.adam8_bias_corrections(b1, b2, s)
        grads = [adam_grad(p.numel(), s + 31 * i, dtype=p.dtype, device="cuda", std=1e-2)
                 for i, p in enumerate(params)]
        adam8_launch([(p, g, *st) for p, g, st in zip(params, grads, states)], lr, b1, b2, eps, bc1, bc2, wd)
        torch.cuda.synchronize()
        for i, (p, g, st) in enumerate(zip(params, grads, states)):
            hp, hm, hv, hms, hvs = host[i]
            oracle.adam8_step(hp, np_bits(g), hm, hv, hms, hvs, lr, b1, b2, eps, bc1, bc2, wd)
            assert np.array_equal(np_bits(st[2]), hms), (i, s)
            assert np.array_equal(np_bits(st[3]), hvs), (i, s)
            assert np.array_equal(np_bits(st[0]), hm), (i, s)
            assert np.array_equal(np_bits(st[1]), hv), (i, s)
            assert np.array_equal(np_bits(p), hp), (i, s)


def _load_ref():
    so = REPO / "oracle" / "_ref" / "ref_adam8_cuda.so"
    if not so.exists():
        pytest.skip("oracle/_ref/ref_adam8_cuda.so not built (needs the reference sources)")
    spec = importlib.util.spec_from_file_location("ref_adam8_cuda", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("n,dtype,steps", [(110_000_000, torch.bfloat16, 100), (3_000_001, torch.float32, 20)])
def test_matches_reference_cuda_kernel(cuda, n, dtype, steps):
    """The reference kernel built from packr/cuda_adam_kernel.cu, driven as
    packr/cuda_adam.py:160-192 drives it, beside CUDA8BitAdam on the same seeded
    params and grads; states and params compared after every step."""
    ref = _load_ref()
    lr, b1, b2, eps, wd = 2e-5, 0.9, 0.999, 1e-8, 0.01
    p_ref = adam_params(n, dtype=dtype, seed=0, device="cuda")
    p_new = torch.nn.Parameter(p_ref.clone())
    m, v, ms, vs = new_state(n)
    opt = CUDA8BitAdam([p_new], lr=lr, betas=(b1, b2), eps=eps, weight_decay=wd)
    worst_code = 0
    worst_rel = 0.0
    for s in range(1, steps + 1):
        g = adam_grad(n, s, dtype=dtype, device="cuda")
        ref.launch_adam_8bit(p_ref, g, m, v, ms, vs, int(dtype == torch.bfloat16), lr, b1, b2, eps,
                             1.0 - b1 ** s, 1.0 - b2 ** s, wd)
        p_new.grad = g
        opt.step()
        st = opt.state[p_new]
        dm = (st["m"].int() - m.int()).abs().max().item()
        dv = (st["v"].int() - v.int()).abs().max().item()
        rel = ((p_new.detach().float() - p_ref.float()).abs() / p_ref.float().abs().clamp_min(1e-30)).max().item()
        worst_code = max(worst_code, dm, dv)
        worst_rel = max(worst_rel, rel)
        assert dm <= 1 and dv <= 1, (s, dm, dv)
        assert rel <= 1e-6, (s, rel)
        assert torch.equal(st["m_scale"], ms) or (st["m_scale"] - ms).abs().max().item() <= 1e-6 * ms.abs().max().item()
    print(f"\nworst |code diff| {worst_code}, worst param rel diff {worst_rel:.3g}")


def _fuzz(shape, dtype, lr=2e-5, steps=50):
    torch.manual_seed(42)
    w = torch.randn(*shape, dtype=dtype, device="cuda") * 0.01
    torch.manual_seed(123)
    grads = [torch.randn(*shape, dtype=dtype, device="cuda") * 0.1 for _ in range(steps)]
    p_ref = torch.nn.Parameter(w.clone())
    p_cut = torch.nn.Parameter(w.clone())
    o_ref = torch.optim.AdamW([p_ref], lr=lr)
    o_cut = CUDA8BitAdam([p_cut], lr=lr)
    ratios, cos = [], []
    for g in grads:
        p_ref.grad = g.clone()
        p_cut.grad = g.clone()
        o_ref.step(); o_cut.step()
        u_ref = (p_ref - w).float().flatten()
        u_cut = (p_cut - w).float().flatten()
        ratios.append(u_cut.norm().item() / max(u_ref.norm().item(), 1e-30))
        cos.append(torch.nn.functional.cosine_similarity(u_ref[None], u_cut[None]).item())
    return ratios, cos


@pytest.mark.parametrize("shape", [(768, 3072), (64, 128)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tracks_fp32_adamw(cuda, shape, dtype):
    """Reference tests/test_cuda_adam.py:93-130 bounds."""
    ratios, cos = _fuzz(shape, dtype)
    assert 0.8 < ratios[0] < 1.2
    assert min(cos) > 0.95


def test_weight_decay_direction(cuda):
    torch.manual_seed(42)
    p = torch.nn.Parameter(torch.randn(64, 64, dtype=torch.bfloat16, device="cuda") * 0.01)
    p2 = torch.nn.Parameter(p.detach().clone())
    g = torch.randn(64, 64, dtype=torch.bfloat16, device="cuda") * 0.1
    p.grad = g.clone(); p2.grad = g.clone()
    torch.optim.AdamW([p], lr=2e-5, weight_decay=0.01).step()
    CUDA8BitAdam([p2], lr=2e-5, weight_decay=0.01).step()
    u1 = p.detach().float().flatten(); u2 = p2.detach().float().flatten()
    assert torch.isfinite(u2).all()
    assert torch.nn.functional.cosine_similarity(u1[None], u2[None]).item() > 0.99


def test_state_layout_is_velvet_readable(cuda):
    p = torch.nn.Parameter(torch.randn(1000, device="cuda", dtype=torch.bfloat16))
    p.grad = torch.randn_like(p) * 1e-3
    opt = CUDA8BitAdam([p], lr=1e-3)
    opt.step()
    st = opt.state[p]
    assert st["m"].dtype == torch.int8 and st["m"].shape == (1000,)
    assert st["v"].dtype == torch.int8 and st["v"].shape == (1000,)
    assert st["m_scale"].dtype == torch.float32 and st["m_scale"].shape == (4,)
    assert st["v_scale"].dtype == torch.float32 and st["v_scale"].shape == (4,)
    assert st["v"].min().item() >= 1 and st["v"].max().item() <= 127
    # resume: the step count survives a state_dict round trip
    sd = opt.state_dict()
    opt2 = CUDA8BitAdam([p], lr=1e-3)
    opt2.load_state_dict(sd)
    assert opt2._step_count == 1


def test_resume_from_state_dict_is_exact(cuda):
    """Save after 3 steps (through torch.save), load into a new optimizer over
    copies of the parameters, 2 more steps: identical to 5 uninterrupted
    steps, bf16 and f32 parameters (the loader keeps the int8 codes and f32
    scales of bf16 parameters)."""
    import io
    def make():
        return [torch.nn.Parameter(adam_params(5000, dtype=torch.bfloat16, seed=1, device="cuda")),
                torch.nn.Parameter(adam_params(777, dtype=torch.float32, seed=2, device="cuda"))]
    def grads(s):
        return [adam_grad(5000, s, dtype=torch.bfloat16, device="cuda"), adam_grad(777, s + 50, dtype=torch.float32, device="cuda")]
    ref = make()
    ropt = CUDA8BitAdam(ref, lr=1e-3, weight_decay=0.01)
    run = make()
    opt = CUDA8BitAdam(run, lr=1e-3, weight_decay=0.01)
    for s in range(1, 4):
        for p, g in zip(ref, grads(s)):
            p.grad = g
        ropt.step()
        for p, g in zip(run, grads(s)):
            p.grad = g
        opt.step()
    buf = io.BytesIO()
    torch.save(opt.state_dict(), buf)
    buf.seek(0)
    resumed = [torch.nn.Parameter(p.detach().clone()) for p in run]
    opt2 = CUDA8BitAdam(resumed, lr=1e-3, weight_decay=0.01)
    opt2.load_state_dict(torch.load(buf, weights_only=False))
    assert opt2.state[resumed[0]]["m"].dtype == torch.int8
    assert opt2.state[resumed[0]]["m_scale"].dtype == torch.float32
    for s in range(4, 6):
        for p, g in zip(ref, grads(s)):
            p.grad = g
        ropt.step()
        for p, g in zip(resumed, grads(s)):
            p.grad = g
        opt2.step()
    torch.cuda.synchronize()
    for a, b in zip(ref, resumed):
        assert torch.equal(a.detach(), b.detach())


def test_fused_quantized_adam_step_with_closure(cuda):
    """FusedQuantizedAdam (the reference's Triton optimizer name, packr/
    optim.py:167-285) on the GPU: step(closure) re-evaluates the closure
    with gradients enabled and returns its loss, and the update equals
    CUDA8BitAdam's on the same gradients bit for bit (parameters, codes and
    scales; bf16 and f32 parameters, two parameter groups)."""
    from packr_b200.optim import FusedQuantizedAdam
    def make():
        return [torch.nn.Parameter(adam_params(3 * 256 + 77, dtype=torch.bfloat16, seed=3, device="cuda")),
                torch.nn.Parameter(adam_params(1000, dtype=torch.float32, seed=4, device="cuda"))]
    a, b = make(), make()
    fq = FusedQuantizedAdam([{"params": [a[0]]}, {"params": [a[1]], "lr": 3e-4}], lr=1e-3, weight_decay=0.01,
                            block_size=256)
    ref = CUDA8BitAdam([{"params": [b[0]]}, {"params": [b[1]], "lr": 3e-4}], lr=1e-3, weight_decay=0.01)
    for s in range(1, 4):
        targets = [adam_grad(p.numel(), s, dtype=torch.float32, device="cuda", std=1e-2) for p in a]
        calls = []

        def closure():
            fq.zero_grad(set_to_none=True)
            loss = sum((p.float() * t).sum() for p, t in zip(a, targets))
            loss.backward()
            calls.append(loss.detach())
            return loss
        loss = fq.step(closure)
        assert len(calls) == 1 and loss is not None and torch.equal(loss.detach(), calls[0])
        for p, q in zip(a, b):
            q.grad = p.grad.clone()
        ref.step()
    torch.cuda.synchronize()
    for p, q in zip(a, b):
        assert torch.equal(p.detach(), q.detach())
        for k in ("m", "v", "m_scale", "v_scale"):
            assert torch.equal(fq.state[p][k], ref.state[q][k]), k
    assert fq.step() is None  # without a closure there is no loss to return


def test_push_stores_every_copy(cuda):
    """packr_adam8_multi_push on one GPU with the "peer" copies in local
    buffers: after each step every copy equals the updated parameter bit for
    bit (vector stores, ragged tails, an unaligned view, bf16 and f32), and
    the parameters equal the oracle's."""
    from packr_b200.cuda_adam import adam8_launch_push
    sizes = [1, 255, 257, 4096 + 13, 100_003]
    dtypes = [torch.bfloat16, torch.float32, torch.bfloat16, torch.float32, torch.bfloat16]
    params = [adam_params(n, dtype=dt, seed=40 + i, device="cuda") for i, (n, dt) in enumerate(zip(sizes, dtypes))]
    big = adam_params(9000, dtype=torch.bfloat16, seed=99, device="cuda")
    params.append(big[5:5 + 7000])  # an unaligned view: the element-wise path
    states = [new_state(p.numel()) for p in params]
    host = [(np_bits(p), *[np_bits(t) for t in st]) for p, st in zip(params, states)]
    copies = [[torch.full_like(p, 7.0) for _ in range(3)] for p in params]
    lr, b1, b2, eps, wd = 1e-3, 0.9, 0.999, 1e-8, 0.01
    for s in range(1, 4):
        bc1, bc2 = oracle.adam8_bias_corrections(b1, b2, s)
        grads = [adam_grad(p.numel(), s + 17 * i, dtype=p.dtype, device="cuda", std=1e-2)
                 for i, p in enumerate(params)]
        adam8_launch_push([(p, g, *st) for p, g, st in zip(params, grads, states)],
                          [[c.data_ptr() for c in cs] for cs in copies], lr, b1, b2, eps, bc1, bc2, wd)
        torch.cuda.synchronize()
        for i, (p, g) in enumerate(zip(params, grads)):
            hp, hm, hv, hms, hvs = host[i]
            oracle.adam8_step(hp, np_bits(g), hm, hv, hms, hvs, lr, b1, b2, eps, bc1, bc2, wd)
            assert np.array_equal(np_bits(p), hp), (i, s)
            for c in copies[i]:
                assert np.array_equal(np_bits(c), hp), (i, s)
