"""Data-parallel training over NCCL on 2 GPUs (skipped with fewer): the
sharded 8-bit AdamW step (reduce-scatter, sm_100a AdamW on the rank's shard,
the new parameters pushed into the other rank's buckets by the AdamW kernel,
or all-gathered) equals the single-GPU CUDA8BitAdam step on the averaged gradient,
bit for bit; and a two-layer compressed model trained data-parallel stays
identical on both ranks and close to single-GPU training on the whole batch."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [((96, 40), torch.bfloat16), ((256,), torch.float32), ((3000, 7), torch.bfloat16), ((5,), torch.float32)]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _params(dev):
    g = torch.Generator().manual_seed(0)
    return [torch.nn.Parameter((torch.randn(*s, generator=g) * 0.02).to(dt).to(dev)) for s, dt in SHAPES]


def _grads(rank, step, dev):
    g = torch.Generator().manual_seed(step)
    out = []
    for s, dt in SHAPES:
        B = torch.randint(-48, 49, s, generator=g).float()
        D = 2 * torch.randint(-4, 5, s, generator=g).float()
        out.append(((B + rank * D) * 2.0 ** -12).to(dt).to(dev))
    return out


def _worker(rank, world, port, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from packr_b200.dp import ShardedAdam8
        from packr_b200.cuda_adam import CUDA8BitAdam
        # 1. optimizer step vs single GPU on the (exactly) averaged gradient,
        #    with the parameters pushed to the peers by the AdamW kernel and
        #    with the NCCL all-gather
        exact = True
        for transport in ("push", "nccl"):
            ps = _params(dev)
            opt = ShardedAdam8(ps, lr=1e-3, weight_decay=0.01, transport=transport)
            exact = exact and opt.transport == transport
            ref = [torch.nn.Parameter(p.detach().clone()) for p in _params(dev)]
            ropt = CUDA8BitAdam(ref, lr=1e-3, weight_decay=0.01)
            for s in range(1, 4):
                for p, gr in zip(ps, _grads(rank, s, dev)):
                    p.grad = gr
                opt.step()
                avg = [(sum(_grads(r, s, dev)[i].double() for r in range(world)) / world).to(ref[i].dtype)
                       for i in range(len(ref))]
                for p, gr in zip(ref, avg):
                    p.grad = gr
                ropt.step()
            torch.cuda.synchronize()
            exact = exact and all(torch.equal(a.detach(), b.detach()) for a, b in zip(ps, ref))
            opt.close()
        # 2. two compressed layers trained data-parallel for 3 steps
        from packr_b200 import PackRLinear
        torch.manual_seed(7)
        layers = [PackRLinear.synthetic(64, 128, device=dev, seed=11), PackRLinear.synthetic(128, 32, device=dev, seed=12)]
        mp_ = [p for l in layers for p in (l.W_f, l.lut, l.bias_f)]
        # several buckets, each reduce-scatter started from the gradient hooks
        dopt = ShardedAdam8(mp_, lr=1e-2, bucket_bytes=1 << 14, overlap_grad_reduce=True)
        same_transport = dopt.transport == "push"  # the default on one node
        gx = torch.Generator().manual_seed(99)
        X = torch.randn(8, 64, generator=gx).to(dev)
        Y = torch.randn(8, 32, generator=gx).to(dev)
        xs, ys = X[rank * 4:(rank + 1) * 4], Y[rank * 4:(rank + 1) * 4]
        p0 = torch.cat([p.detach().float().reshape(-1) for p in mp_])
        first_grad = None
        for step in range(3):
            for p in mp_:
                p.grad = None
            out = layers[1](layers[0](xs).to(torch.bfloat16))
            ((out - ys) ** 2).mean().backward()
            if step == 0:  # the rank-averaged gradient of the first step
                first_grad = torch.cat([p.grad.detach().float().reshape(-1) for p in mp_])
                dist.all_reduce(first_grad, op=dist.ReduceOp.AVG)
            dopt.step()
        torch.cuda.synchronize()
        flat = torch.cat([p.detach().float().reshape(-1) for p in mp_])
        gathered = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(gathered, flat)
        same = same_transport and all(torch.equal(gathered[0], g) for g in gathered)
        # VelvetController's v means over the sharded state: one all-reduce,
        # the same on every rank, and a controller step sets the same lr
        from packr_b200 import VelvetController
        means = dopt.v_means()
        mv = torch.tensor([means[id(p)] for p in mp_], dtype=torch.float64, device=dev)
        mg = [torch.empty_like(mv) for _ in range(world)]
        dist.all_gather(mg, mv)
        same = same and all(torch.equal(mg[0], m) for m in mg) and bool(torch.isfinite(mv).all()) and bool((mv > 0).all())
        ctl = VelvetController(dopt, total_opt_steps=100)
        ctl.step()
        ctl.step()
        lr = torch.tensor([dopt.lr], dtype=torch.float64, device=dev)
        lg = [torch.empty_like(lr) for _ in range(world)]
        dist.all_gather(lg, lr)
        same = same and all(torch.equal(lg[0], x) for x in lg)
        q.put((rank, exact, same, (flat - p0).cpu().numpy(), first_grad.cpu().numpy()))
    finally:
        dist.destroy_process_group()


def test_sharded_adam_and_training_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, exact, same, upd, g0 = q.get(timeout=300)
        res[r] = (exact, same, upd, g0)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][0], f"rank {r}: sharded step differs from the single-GPU step"
        assert res[r][1], f"rank {r}: ranks hold different parameters"
    # single GPU on the whole batch (mean loss over 8 = mean of the two
    # half-batch means): same first gradient; the three-step update points the
    # same way (Adam normalises each element, so near-zero gradients may flip)
    from packr_b200 import PackRLinear
    from packr_b200.cuda_adam import CUDA8BitAdam
    dev = torch.device("cuda", 0)
    layers = [PackRLinear.synthetic(64, 128, device=dev, seed=11), PackRLinear.synthetic(128, 32, device=dev, seed=12)]
    mp_ = [p for l in layers for p in (l.W_f, l.lut, l.bias_f)]
    opt = CUDA8BitAdam(mp_, lr=1e-2)
    gx = torch.Generator().manual_seed(99)
    X = torch.randn(8, 64, generator=gx).to(dev)
    Y = torch.randn(8, 32, generator=gx).to(dev)
    p0 = torch.cat([p.detach().float().reshape(-1) for p in mp_])
    g_first = None
    for step in range(3):
        for p in mp_:
            p.grad = None
        out = layers[1](layers[0](X).to(torch.bfloat16))
        ((out - Y) ** 2).mean().backward()
        if step == 0:
            g_first = torch.cat([p.grad.detach().float().reshape(-1) for p in mp_]).cpu().numpy()
        opt.step()
    upd = (torch.cat([p.detach().float().reshape(-1) for p in mp_]) - p0).cpu().numpy()
    g_dp = res[0][3]
    assert np.abs(g_dp - g_first).max() / np.abs(g_first).max() < 1e-2
    u_dp = res[0][2]
    cos = float(np.dot(u_dp, upd) / (np.linalg.norm(u_dp) * np.linalg.norm(upd)))
    assert cos > 0.95, cos


def test_grad_sink_single_gpu(cuda):
    """World size 1: PackRLinear's backward writes dW_f straight into the
    optimizer's flat gradient buffer (no copy), accumulation still adds, and
    the step equals CUDA8BitAdam on the same gradients (W_f bit for bit; the
    lut gradient is an atomic sum, reproducible to rounding only)."""
    from packr_b200 import PackRLinear
    from packr_b200.cuda_adam import CUDA8BitAdam
    from packr_b200.dp import ShardedAdam8
    dev = torch.device("cuda")
    lays = [PackRLinear.synthetic(256, 512, bias=False, device=dev, seed=3),
            PackRLinear.synthetic(512, 128, bias=False, device=dev, seed=4)]
    twins = [PackRLinear.synthetic(256, 512, bias=False, device=dev, seed=3),
             PackRLinear.synthetic(512, 128, bias=False, device=dev, seed=4)]
    opt = ShardedAdam8([p for l in lays for p in (l.W_f, l.lut)], lr=1e-3, weight_decay=0.01)
    ropt = CUDA8BitAdam([p for l in twins for p in (l.W_f, l.lut)], lr=1e-3, weight_decay=0.01)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(300, 256, generator=g, device=dev).to(torch.bfloat16)
    dy = torch.randn(300, 128, generator=g, device=dev)
    opt.zero_grad()
    ropt.zero_grad()
    for _ in range(2):  # two micro-batches: the second accumulates into the sink
        lays[1](lays[0](x).to(torch.bfloat16)).backward(dy)
        twins[1](twins[0](x).to(torch.bfloat16)).backward(dy)
    close = lambda a, b: torch.allclose(a, b, rtol=1e-5, atol=1e-6 * b.abs().max().item())
    for l, t in zip(lays, twins):
        gptr = l.W_f.grad.data_ptr()
        flat = opt.bucket_of(l.W_f).grad
        assert flat.data_ptr() <= gptr < flat.data_ptr() + flat.numel() * flat.element_size()
        assert torch.equal(l.W_f.grad, t.W_f.grad)
        assert close(l.lut.grad, t.lut.grad)
    opt.step()
    ropt.step()
    torch.cuda.synchronize()
    for l, t in zip(lays, twins):
        assert torch.equal(l.W_f, t.W_f)
        assert close(l.lut, t.lut)
