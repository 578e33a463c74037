"""Data-parallel sharded 8-bit AdamW (packr_b200.dp.ShardedAdam8): host-side
logic on CPU with gloo, world_size 2 and 3, the optimizer arithmetic played
by the oracle.  The N-rank step must equal the single-process step on the
rank-averaged gradient, element for element, and every rank must end with
identical parameters."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from packr_b200.dp import ShardedAdam8


def _np(t):
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def oracle_adam_fn(entries, lr, b1, b2, eps, bc1, bc2, wd):
    for p, g, m, v, ms, vs in entries:
        oracle.adam8_step(_np(p), _np(g).copy(), m.numpy(), v.numpy(), ms.numpy(), vs.numpy(), lr, b1, b2, eps, bc1,
                          bc2, wd)


SHAPES = [((96, 40), torch.bfloat16), ((256,), torch.float32), ((40,), torch.bfloat16), ((300, 7), torch.bfloat16),
          ((1,), torch.float32)]


def make_params():
    g = torch.Generator().manual_seed(0)
    return [torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).to(dt)) for s, dt in SHAPES]


def make_grads(rank, step):
    """(B + rank*D) * 2^-12 with small integers B, D: every partial sum over
    ranks and the average (B + D*(world-1)/2 for world 2 and 3 with even D...)
    is exact in bf16 and f32, so the reduce-scatter average is exact."""
    g = torch.Generator().manual_seed(step)
    out = []
    for s, dt in SHAPES:
        B = torch.randint(-48, 49, s, generator=g).float()
        D = 2 * torch.randint(-4, 5, s, generator=g).float()
        out.append(((B + rank * D) * 2.0 ** -12).to(dt))
    return out


def _worker(rank, world, port, steps, q, mode="assign"):
    """mode "assign": gradients set on .grad; "overlap": produced by a backward
    (sum(p * g)) with the reduce-scatter started from the gradient hooks, the
    buckets small enough to hold one or two parameters, and a first backward
    of each step under no_sync() whose gradient is then replaced."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        params = make_params()
        if mode == "overlap":
            opt = ShardedAdam8(params, lr=1e-3, weight_decay=0.01, adam_fn=oracle_adam_fn, bucket_bytes=1024,
                               overlap_grad_reduce=True)
            assert len(opt.buckets) > 2
        else:
            opt = ShardedAdam8(params, lr=1e-3, weight_decay=0.01, adam_fn=oracle_adam_fn)
        for s in range(1, steps + 1):
            grads = make_grads(rank, s)
            if mode == "overlap":
                opt.zero_grad()
                with opt.no_sync():  # an accumulation micro-batch: no reduce-scatter
                    sum((p * g).sum() for p, g in zip(params, grads)).backward()
                opt.zero_grad()
                sum((p * g).sum() for p, g in zip(params, grads)).backward()
                assert all(b.work is not None for b in opt.buckets)  # every bucket already in flight
            else:
                for p, gr in zip(params, grads):
                    p.grad = gr
            opt.step()
        q.put((rank, [_np(p.detach()).copy() for p in params], opt.shard_numel))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def expected(world, steps):
    """Single process: the exact rank-average of the gradients, then the
    oracle step per parameter."""
    params = [p.detach().clone() for p in make_params()]
    state = [(np.zeros(p.numel(), np.int8), np.zeros(p.numel(), np.int8),
              np.ones((p.numel() + 255) // 256, np.float32), np.ones((p.numel() + 255) // 256, np.float32))
             for p in params]
    for s in range(1, steps + 1):
        grads = [make_grads(r, s) for r in range(world)]
        bc1, bc2 = oracle.adam8_bias_corrections(0.9, 0.999, s)
        for i, p in enumerate(params):
            avg = (sum(grads[r][i].double() for r in range(world)) / world).to(p.dtype)
            m, v, ms, vs = state[i]
            oracle.adam8_step(_np(p), _np(avg.contiguous()).copy(), m, v, ms, vs, 1e-3, 0.9, 0.999, 1e-8, bc1, bc2,
                              0.01)
    return [_np(p).copy() for p in params]


@pytest.mark.parametrize("world,mode", [(2, "assign"), (3, "assign"), (2, "overlap")])
def test_sharded_step_equals_single_process(world, mode):
    steps = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, steps, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, ps, shard = q.get(timeout=120)
        results[r] = (ps, shard)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = expected(world, steps)
    for r in range(world):
        for a, b in zip(results[r][0], results[0][0]):
            assert np.array_equal(a, b), "ranks disagree"
    total_state = sum(results[r][1] for r in range(world))
    assert total_state == sum(results[0][1] for _ in range(world))  # equal shards
    for i, (got, exp) in enumerate(zip(results[0][0], want)):
        if got.dtype == np.uint16:
            gf, ef = oracle.bf16_to_f32(got), oracle.bf16_to_f32(exp)
        else:
            gf, ef = got, exp
        assert np.array_equal(got, exp), i


def test_single_process_layout_and_views():
    params = make_params()
    before = [p.detach().clone() for p in params]
    opt = ShardedAdam8(params, lr=1e-3, adam_fn=oracle_adam_fn)
    # parameters now live in the flat buffers, values unchanged, 256-aligned starts
    for p, b in zip(params, before):
        assert torch.equal(p.detach(), b)
    for b in opt.buckets:
        assert len({s.param.dtype for s in b.slots}) == 1
        for s in b.slots:
            assert s.offset % 256 == 0
            assert s.param.data_ptr() == b.flat[s.offset:].data_ptr()
    for p, gr in zip(params, make_grads(0, 1)):
        p.grad = gr
    opt.step()
    assert opt.step_count == 1
    assert all(not torch.equal(p.detach(), b) for p, b in zip(params, before))


# ------------------------------------------------------------- checkpoints
def expected_with_state(worlds):
    """Single process: step s averages the gradients of worlds[s-1] ranks.
    Returns (params, [(m, v, ms, vs)] per parameter) as numpy."""
    params = [p.detach().clone() for p in make_params()]
    state = [(np.zeros(p.numel(), np.int8), np.zeros(p.numel(), np.int8),
              np.ones((p.numel() + 255) // 256, np.float32), np.ones((p.numel() + 255) // 256, np.float32))
             for p in params]
    for s, world in enumerate(worlds, start=1):
        grads = [make_grads(r, s) for r in range(world)]
        bc1, bc2 = oracle.adam8_bias_corrections(0.9, 0.999, s)
        for i, p in enumerate(params):
            avg = (sum(grads[r][i].double() for r in range(world)) / world).to(p.dtype)
            m, v, ms, vs = state[i]
            oracle.adam8_step(_np(p), _np(avg.contiguous()).copy(), m, v, ms, vs, 1e-3, 0.9, 0.999, 1e-8, bc1, bc2,
                              0.01)
    return [_np(p).copy() for p in params], state


def _to_np(sd):
    return {**sd, "state": {i: {k: v.numpy().copy() for k, v in st.items()} for i, st in sd["state"].items()}}


def _from_np(sd):
    return {**sd, "state": {i: {k: torch.from_numpy(v.copy()) for k, v in st.items()} for i, st in sd["state"].items()}}


def _ckpt_worker(rank, world, port, first_step, last_step, init, q):
    """Steps first_step..last_step on `world` ranks; with `init` = (param
    values, consolidated state) it starts from a checkpoint."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        params = make_params()
        if init is not None:
            with torch.no_grad():
                for p, v in zip(params, init[0]):
                    p.copy_(v)
        opt = ShardedAdam8(params, lr=1e-3, weight_decay=0.01, adam_fn=oracle_adam_fn, bucket_bytes=700)
        if init is not None:
            opt.load_consolidated_state_dict(_from_np(init[1]))
        for s in range(first_step, last_step + 1):
            for p, gr in zip(params, make_grads(rank, s)):
                p.grad = gr
            opt.step()
        sd = opt.consolidated_state_dict()
        # numpy through the queue: torch tensors would travel as shared-memory
        # handles that vanish with this process
        q.put((rank, [_np(p.detach()).copy() for p in params], _to_np(sd)))
    finally:
        dist.destroy_process_group()


def _run(world, first, last, init):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ckpt_worker, args=(r, world, port, first, last, init, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, ps, sd = q.get(timeout=120)
        out[r] = (ps, _from_np(sd))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def test_consolidated_checkpoint_resumes_at_another_world_size():
    """2 ranks for steps 1-2, a world-size independent checkpoint, then 3
    ranks for step 3: state and parameters equal the single process with the
    same averaged gradients, bit for bit."""
    first = _run(2, 1, 2, None)
    params2, sd2 = first[0]
    want_p, want_s = expected_with_state([2, 2])
    for i, (m, v, ms, vs) in enumerate(want_s):
        st = sd2["state"][i]
        assert st["m"].dtype == torch.int8 and st["m_scale"].dtype == torch.float32
        assert np.array_equal(st["m"].numpy(), m) and np.array_equal(st["v"].numpy(), v), i
        assert np.array_equal(st["m_scale"].numpy(), ms) and np.array_equal(st["v_scale"].numpy(), vs), i
    assert sd2["packr_step_count"] == 2
    for r in first:  # every rank gets the whole dict
        assert all(torch.equal(first[r][1]["state"][i]["m"], sd2["state"][i]["m"]) for i in sd2["state"])
    vals = [torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) if a.dtype == np.uint16 else torch.from_numpy(a)
            for a in params2]
    second = _run(3, 3, 3, (vals, _to_np(sd2)))
    want_p, want_s = expected_with_state([2, 2, 3])
    for r in second:
        for got, exp in zip(second[r][0], want_p):
            assert np.array_equal(got, exp)
    for i, (m, v, ms, vs) in enumerate(want_s):
        st = second[0][1]["state"][i]
        assert np.array_equal(st["m"].numpy(), m) and np.array_equal(st["v_scale"].numpy(), vs), i


def test_cuda8bit_adam_loads_consolidated_state():
    """The consolidated format is CUDA8BitAdam's: its loader keeps int8 codes
    and f32 scales for bf16 parameters (torch's own loader casts them)."""
    from packr_b200.cuda_adam import CUDA8BitAdam
    params = make_params()
    opt = ShardedAdam8(params, lr=1e-3, weight_decay=0.01, adam_fn=oracle_adam_fn)
    for s in (1, 2):
        for p, gr in zip(params, make_grads(0, s)):
            p.grad = gr
        opt.step()
    sd = opt.consolidated_state_dict()
    fresh = make_params()
    single = CUDA8BitAdam(fresh, lr=1e-3, weight_decay=0.01)
    single.load_state_dict(sd)
    assert single._step_count == 2
    for i, p in enumerate(fresh):
        st = single.state[p]
        assert st["m"].dtype == torch.int8 and st["v"].dtype == torch.int8
        assert st["m_scale"].dtype == torch.float32 and st["v_scale"].dtype == torch.float32
        assert torch.equal(st["m"], sd["state"][i]["m"]) and torch.equal(st["v_scale"], sd["state"][i]["v_scale"])
    again = single.state_dict()
    back = ShardedAdam8(make_params(), lr=1e-3, weight_decay=0.01, adam_fn=oracle_adam_fn)
    back.load_consolidated_state_dict(again)
    re = back.consolidated_state_dict()
    for i in sd["state"]:
        for k in ("m", "v", "m_scale", "v_scale"):
            assert torch.equal(re["state"][i][k], sd["state"][i][k]), (i, k)


def _transport_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = {}
        opt = ShardedAdam8(make_params(), lr=1e-3, adam_fn=oracle_adam_fn)
        out["auto"] = opt.transport
        opt = ShardedAdam8(make_params(), lr=1e-3)
        out["auto_default_adam"] = opt.transport
        try:
            ShardedAdam8(make_params(), lr=1e-3, transport="push")
            out["push"] = "accepted"
        except RuntimeError as e:
            out["push"] = str(e)
        try:
            ShardedAdam8(make_params(), lr=1e-3, transport="bogus")
            out["bogus"] = "accepted"
        except ValueError:
            out["bogus"] = "ValueError"
        opt.close()  # nothing mapped: no collective, returns
        out["closed"] = opt.transport
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_transport_selection_on_gloo():
    """The push transport needs NCCL and CUDA parameters on one node: with
    gloo every rank agrees on the all-gather ("nccl"), an explicit request for
    "push" raises on every rank with the reason, and an unknown name raises."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_transport_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        o = res[r]
        assert o["auto"] == "nccl" and o["auto_default_adam"] == "nccl" and o["closed"] == "nccl"
        assert "unavailable" in o["push"] and "NCCL" in o["push"], o["push"]
        assert o["bogus"] == "ValueError"
