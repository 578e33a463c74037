"""Benchmark of PackR's training hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload ffn|adam8|decode|bert|llama8b|from_linear]
                    [--impl ours|reference]

Prints ONE JSON line (rank 0).  For N>1 it is launched by torchrun, one rank
per GPU (NCCL); every rank runs the same per-GPU workload (weak scaling) and
the step time is the max over ranks of CUDA-event time.

Workloads (synthetic, seeded; no dataset exists for this path):
  ffn    (default) PackRLinear forward+backward of the Llama-7B FFN shapes:
         gate 4096->11008, up 4096->11008, down 11008->4096, M = 4096 tokens
         of bf16 activations per GPU, f32 upstream gradients holding
         bf16-exact values; one step = the three layers' forward and backward
         through autograd (out, dX, dW_f, dlut) plus the data-parallel 8-bit
         AdamW update; metric TFLOP/s over 6*M*K*N per layer.  Per step the
         operands (~0.9 GB) exceed L2.
  decode forward of the same three layers at M = 16 tokens (--tokens to
         change): the decode-bound regime; metric GB/s of packed weights
         (3 bytes per weight) streamed per second.
  bert   BERT-base fine-tune step (FFN layers compressed, batch 32 x seq 128,
         CUDA8BitAdam); metric sequences/s, with the PackRLinear and Adam
         shares of the step.
  llama8b Llama-3-8B-shaped decoder, every Linear a PackRLinear, seq 2048,
         micro-batch 1 per GPU, data parallel; metric tokens/s.
  from_linear  PackRLinear.from_linear of one Llama-3-8B decoder layer's
         seven bf16 Linear weights (q, k, v, o 4096-wide; gate, up 4096->14336;
         down 14336->4096: 218 M weights, three of them above torch.quantile's
         2^24 limit); metric Gweights/s.
  adam8  CUDA8BitAdam step over one flat 110,000,000-element bf16 parameter
         (lr 2e-5, betas (0.9, 0.999), eps 1e-8, wd 0.01, block 256); metric
         Gparam/s.  Per step the inputs (1.1 GB) exceed L2 (126 MB).
The reference arm (--impl reference) times the reference's own CPU
implementation of the same workload on this host's cores (bounded sample).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

ADAM_N = 110_000_000
ADAM_BYTES_PER_PARAM = 10.0 + 16.0 / 256.0  # p2+g2+m1+v1 read, p2+m1+v1 write, 2 f32 scales read+write per block


def load_peaks() -> tuple[dict, str]:
    f = REPO / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            return json.loads(f.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons of one GPU while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self._t is not None:
                self._t.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        # NCCL's own messages (its version banner included) go to stderr, so
        # that stdout carries the one JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(fn, steps: int, warmup: int, world: int, flush=None, warm_seconds: float = 0.0) -> tuple[float, list[float]]:
    """Runs fn() `warmup` times (and keeps warming until `warm_seconds` have
    passed, so clock samples cover steady state), then times `steps` calls
    with CUDA events on the current stream; returns (max-over-ranks total ms,
    per-step ms)."""
    t0 = time.perf_counter()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if warm_seconds > 0:
        # the extra warm-up count is agreed over ranks (MAX): every rank
        # must take the same collective steps
        t1 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        one = max(time.perf_counter() - t1, 1e-6)
        extra = min(int(math.ceil(max(0.0, warm_seconds - (time.perf_counter() - t0)) / one)), 5000)
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([extra], device="cuda", dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            extra = int(t.item())
        for i in range(extra):
            fn()
            if (i + 1) % 16 == 0:
                torch.cuda.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    per = []
    total = 0.0
    for i in range(steps):
        if flush is not None:
            flush()
        evs[i].record(stream)
        fn()
        end = torch.cuda.Event(enable_timing=True)
        end.record(stream)
        evs[i + 1] = end
        per.append((evs[i], end))
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in per]
    total = sum(ms)
    return max_over_ranks(total, world), ms


def write_timeline(step, path: str, rank: int, meta: dict) -> None:
    """Three more steps under torch.profiler (CUPTI) on every rank; rank 0
    writes each GPU activity (kernel, copy, memset) as [start_us, dur_us,
    name, stream] relative to the first, plus `meta`."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(3):
            step()
        torch.cuda.synchronize()
    if rank != 0:
        return
    evs = sorted((e.time_range.start, e.time_range.end, e.name, getattr(e, "device_resource_id", -1))
                 for e in prof.events() if e.device_type.name == "CUDA")
    t0 = evs[0][0] if evs else 0
    out = dict(meta, events=[[round(a - t0, 1), round(b - a, 1), n, sid] for a, b, n, sid in evs])
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    with open(path, "w") as f:
        json.dump(out, f)


def b2b_ms(fn, reps: int, warm: int = 3, min_seconds: float = 0.0) -> float:
    """Mean device time of one fn() call over `reps` calls launched back to
    back between one pair of CUDA events on the current stream (after `warm`
    untimed calls; more calls while the first `reps` took under
    `min_seconds`), so that the host's launch gaps between calls are not
    counted where the GPU has queued work."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = reps
    while True:
        a.record(s)
        for _ in range(n):
            fn()
        b.record(s)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        if ms * 1e-3 >= min_seconds or n >= 64 * reps:
            return ms / n
        n *= 2


def graph_b2b_ms(fn, reps: int = 10) -> float:
    """Mean device time of one fn() call over `reps` calls captured back to
    back in one CUDA graph and replayed between one pair of CUDA events: no
    host launch gaps between the calls, whatever the host's per-call cost."""
    replay = graph_of(lambda: [fn() for _ in range(reps)])
    replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


# ---------------------------------------------------------------- CPU baselines
def cpu_adam_reference(n: int, reps_budget_s: float, min_reps: int = 3):
    """Times the reference's C++ CPU 8-bit AdamW (packr/offload.py:39-130,
    built from source into oracle/_ref) on n fp32 params; single-threaded as
    written.  Falls back to the oracle's C port when the build is absent."""
    import importlib.util
    so = REPO / "oracle" / "_ref" / "ref_cpu_adam8.so"
    g = torch.Generator().manual_seed(0)
    p = (torch.randn(n, generator=g) * 0.02)
    gr = (torch.randn(n, generator=g) * 1e-3)
    m = torch.zeros(n, dtype=torch.int8)
    v = torch.zeros(n, dtype=torch.int8)
    nb = (n + 255) // 256
    ms = torch.ones(nb)
    vs = torch.ones(nb)
    if so.exists():
        spec = importlib.util.spec_from_file_location("ref_cpu_adam8", so)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        z = torch.zeros(1, dtype=torch.int64)
        args = (m, v, ms, vs, p, gr, z, torch.tensor([n]), z.clone(), torch.tensor([nb]), 1)

        def run(step):
            mod.cpu_fused_adam_8bit_kernel(*args, 2e-5, 0.9, 0.999, 1e-8, 1.0 - 0.9 ** step, 1.0 - 0.999 ** step,
                                           0.01, 256)
        kind, desc = "reference", "reference C++ CPU 8-bit AdamW (packr/offload.py:39-130), 1 thread"
    else:
        import oracle
        pn, gn, mn, vn, msn, vsn = (t.numpy() for t in (p, gr, m, v, ms, vs))

        def run(step):
            oracle.adam8_step(pn, gn, mn, vn, msn, vsn, 2e-5, 0.9, 0.999, 1e-8, 1.0 - 0.9 ** step,
                              1.0 - 0.999 ** step, 0.01)
        kind, desc = "port", "oracle C port of packr/cuda_adam_kernel.cu, 1 thread"
    run(1)
    times = []
    t_start = time.perf_counter()
    step = 2
    while len(times) < min_reps or time.perf_counter() - t_start < reps_budget_s:
        t0 = time.perf_counter()
        run(step)
        times.append(time.perf_counter() - t0)
        step += 1
    sec = statistics.median(times)
    return {"value": n / sec / 1e9, "unit": "Gparam/s", "cores": 1, "kind": kind,
            "sample": f"{n} fp32 params, {len(times)} timed steps (median), {desc}",
            "host_cores": os.cpu_count()}


# ---------------------------------------------------------------- workloads
def bench_adam8(args, world, rank, peaks, peak_kind):
    from packr_b200.cuda_adam import CUDA8BitAdam
    from packr_b200.synthetic import adam_grad, adam_params
    n = ADAM_N
    p = torch.nn.Parameter(adam_params(n, dtype=torch.bfloat16, seed=rank, device="cuda"))
    g = adam_grad(n, 1, dtype=torch.bfloat16, device="cuda")
    p.grad = g
    opt = CUDA8BitAdam([p], lr=2e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    step = opt.step
    with ClockSampler(torch.cuda.current_device()) as clk:
        total_ms, per = timed(step, args.steps, args.warmup, world, warm_seconds=1.5)
    ms_step = total_ms / args.steps
    value = world * n / (ms_step * 1e-3) / 1e9
    kernel_ms = statistics.mean(per)
    achieved = n * ADAM_BYTES_PER_PARAM / (kernel_ms * 1e-3) / 1e9
    # end to end through the public API with host buffers
    hg = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)
    hg.copy_(g.cpu())
    hp = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)

    def e2e_step():
        p.grad.copy_(hg, non_blocking=True)
        opt.step()
        hp.copy_(p.detach(), non_blocking=True)
    e2e_ms, _ = timed(e2e_step, args.steps, max(args.warmup, 1), world)
    e2e_val = world * n / (e2e_ms / args.steps * 1e-3) / 1e9
    line = {
        "metric": "8-bit AdamW Gparam/s", "value": round(value, 3), "unit": "Gparam/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 params, int8 states, f32 math",
        "data": "synthetic (seeded N(0,0.02) params, N(0,1e-3) grads)",
        "config": {"workload": "adam8: CUDA8BitAdam step, 110,000,000 bf16 params per GPU",
                   "lr": 2e-5, "betas": [0.9, 0.999], "eps": 1e-8, "weight_decay": 0.01, "block": 256,
                   "l2": "inputs larger than L2 (1.1 GB per step)", "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": load_traffic("adam8_kernel", "adam8_110M"),
                     "peak_source": f"{peak_kind} hbm_gbs", "kernel": "adam8_kernel<bf16>",
                     "algorithmic_bytes_per_launch": n * ADAM_BYTES_PER_PARAM},
        "e2e": {"value": round(e2e_val, 3), "unit": "Gparam/s", "h2d_bytes_per_step": 2 * n,
                "d2h_bytes_per_step": 2 * n},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_adam_reference(1 << 24, args.cpu_seconds)
    return line


# ---------------------------------------------------------------- ffn workload
FFN_HIDDEN, FFN_INTER, FFN_M = 4096, 11008, 4096
FFN_LAYERS = (("gate", FFN_HIDDEN, FFN_INTER), ("up", FFN_HIDDEN, FFN_INTER), ("down", FFN_INTER, FFN_HIDDEN))


def ffn_flops(M: int) -> float:
    return float(sum(6 * M * k * n for _, k, n in FFN_LAYERS))


def load_traffic(kernel: str, workload: str):
    """dram bytes per launch of `kernel` from the committed ncu summary, or None."""
    f = REPO / "profiles" / "traffic.json"
    if not f.exists():
        return None
    try:
        return json.loads(f.read_text()).get(workload, {}).get(kernel)
    except Exception:
        return None


def cpu_linear_port(budget_s: float, M: int = 1024):
    """Times the reference PackRLinear forward + backward arithmetic on the
    host (oracle/reference_port.py: torch CPU, the reference's own op sequence
    of packr/kernel.py:127-139 and packr/autograd.py:65-83, all host threads)
    on one gate-shaped layer (4096 -> 11008) at M tokens per sample."""
    from oracle import reference_port as rp
    from packr_b200.synthetic import linear_case
    K, N = FFN_HIDDEN, FFN_INTER
    c = linear_case(M, K, N, x_dtype=torch.bfloat16, bias=False, seed=0, fanin_scaled=True)

    def run():
        rp.forward(c["x"], c["W_p"], c["W_f"], c["lut"])
        rp.backward(c["dY"], c["x"], c["W_p"], c["W_f"], c["lut"])
    run()
    times = []
    t0 = time.perf_counter()
    while len(times) < 2 or time.perf_counter() - t0 < budget_s:
        a = time.perf_counter()
        run()
        times.append(time.perf_counter() - a)
    sec = statistics.median(times)
    return {"value": 6.0 * M * K * N / sec / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"one 4096->11008 layer, M={M}, fwd+bwd, {len(times)} timed samples (median); "
                                      "torch-CPU restatement of the reference path (oracle/reference_port.py)",
            "host_cores": os.cpu_count()}


def cpu_decode_port(budget_s: float, M: int):
    """Times the reference PackRLinear forward (oracle/reference_port.py,
    torch CPU, all host threads) over the three FFN layers at M tokens."""
    from oracle import reference_port as rp
    from packr_b200.synthetic import linear_case
    cases = [linear_case(M, k, n, x_dtype=torch.bfloat16, bias=False, seed=i, fanin_scaled=True)
             for i, (_, k, n) in enumerate(FFN_LAYERS)]

    def run():
        for c in cases:
            rp.forward(c["x"], c["W_p"], c["W_f"], c["lut"])
    run()
    times = []
    t0 = time.perf_counter()
    while len(times) < 2 or time.perf_counter() - t0 < budget_s:
        a = time.perf_counter()
        run()
        times.append(time.perf_counter() - a)
    sec = statistics.median(times)
    wbytes = sum(3.0 * k * n for _, k, n in FFN_LAYERS)
    return {"value": wbytes / sec / 1e9, "unit": "GB/s (weight bytes)", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"forward of the three FFN layers at M={M}, {len(times)} timed samples "
                                      "(median); torch-CPU restatement of the reference path",
            "host_cores": os.cpu_count()}


def graph_of(fn, warm: int = 2):
    """fn captured once in a CUDA graph; returns a callable that replays it
    (the tensors fn writes are the graph's own, reused every replay)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g.replay


def bench_decode(args, world, rank, peaks, peak_kind):
    """Decode-bound forward: the three Llama-7B FFN layers at M (default 16)
    tokens, no bias; value = packed-weight bytes (3 per weight) / time."""
    from packr_b200 import kernel as K
    M = args.tokens if args.tokens_given else 16
    dev = torch.device("cuda", torch.cuda.current_device())
    from packr_b200.synthetic import linear_case
    layers = []
    for i, (_, k, n) in enumerate(FFN_LAYERS):
        c = linear_case(M, k, n, x_dtype=torch.bfloat16, bias=False, seed=100 + i, fanin_scaled=True)
        layers.append({kk: (v.to(dev) if v is not None else None) for kk, v in c.items()})
    wbytes = sum(3.0 * k * n for _, k, n in FFN_LAYERS)
    algo = sum(3.0 * k * n + 2.0 * M * k + 4.0 * M * n for _, k, n in FFN_LAYERS)

    def eager():
        for c in layers:
            K.forward(c["x"], c["W_p"], c["W_f"], c["lut"], None)
    # A decode loop replays its per-token launches from a CUDA graph (as a
    # serving loop does): the host's per-call overhead (~20 us of Python and
    # ctypes) is comparable to a layer's kernel time at these sizes.
    step = graph_of(eager)
    with ClockSampler(torch.cuda.current_device()) as clk:
        total_ms, per = timed(step, args.steps, args.warmup, world, warm_seconds=1.5)
    ms_step = total_ms / args.steps
    value = world * wbytes / (ms_step * 1e-3) / 1e9
    achieved = algo / (statistics.mean(per) * 1e-3) / 1e9
    eager_ms, _ = timed(eager, args.steps, args.warmup, world)
    hx = [c["x"].cpu().pin_memory() for c in layers]
    dx = [torch.empty_like(c["x"]) for c in layers]
    hout = [torch.empty(M, n, dtype=torch.float32, pin_memory=True) for _, _, n in FFN_LAYERS]

    def e2e_eager():
        for i, c in enumerate(layers):
            dx[i].copy_(hx[i], non_blocking=True)
            hout[i].copy_(K.forward(dx[i], c["W_p"], c["W_f"], c["lut"], None), non_blocking=True)
    e2e_ms, _ = timed(graph_of(e2e_eager), args.steps, max(args.warmup, 1), world)
    line = {
        "metric": f"PackRLinear decode forward GB/s of packed weights (M={M})", "value": round(value, 1),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 x, f32 decode and accumulate", "data": "synthetic (seeded)",
        "config": {"workload": f"decode: forward of the Llama-7B FFN gate/up/down layers at M={M} tokens",
                   "weight_bytes_per_step": wbytes, "l2": "weights 0.27 GB per step, larger than L2",
                   "parallelism": f"replicas x{world}", "launch": "CUDA graph of the three packr_forward calls",
                   "eager_ms_per_step": round(eager_ms / args.steps, 5)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": f"{peak_kind} hbm_gbs",
                     "kernel": "gemv_cluster_kernel (M <= 4) or skinny tcgen05 + reduce (three layers)",
                     "algorithmic_bytes_per_launch": algo},
        "e2e": {"value": round(world * wbytes / (e2e_ms / args.steps * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in hx),
                "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in hout)},
        "gpu_launches": args.steps * (1 if M <= 4 else 2) * len(FFN_LAYERS),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_port(args.cpu_seconds, M)
    return line


def bench_bert(args, world, rank, peaks, peak_kind):
    """BERT-base fine-tune step (12 layers, hidden 768, FFN 3072, 12 heads,
    vocab 30522), random init, FFN Linear layers compressed to PackRLinear,
    batch 32 x seq 128 of random ids, 2-class labels, CUDA8BitAdam over all
    ~110M params (fp32 model, bf16 W_f)."""
    from packr_b200 import kernel as K
    from packr_b200 import workloads as wl
    from packr_b200.cuda_adam import CUDA8BitAdam
    from packr_b200.dp import ShardedAdam8
    dev = torch.device("cuda", torch.cuda.current_device())
    model = wl.bert_classifier(dev, seed=0)
    model.train()
    params = [p for p in model.parameters() if p.requires_grad]
    n_params = sum(p.numel() for p in params)
    if world > 1:
        opt = ShardedAdam8(params, lr=2e-5, weight_decay=0.01, overlap_grad_reduce=True)
    else:
        opt = CUDA8BitAdam(params, lr=2e-5, weight_decay=0.01)
    ids, labels = wl.bert_batch(dev, seed=rank)

    def step():
        opt.zero_grad(set_to_none=True)
        model(input_ids=ids, labels=labels).loss.backward()
        opt.step()
    with ClockSampler(torch.cuda.current_device()) as clk:
        total_ms, per = timed(step, args.steps, args.warmup, world, warm_seconds=1.5)
    ms_step = total_ms / args.steps
    value = world * 32 / (ms_step * 1e-3)
    # shares: the optimizer step alone, and the 24 compressed layers' fwd+bwd alone
    _, a_per = timed(opt.step, max(args.steps, 10), 3, 1)
    adam_ms = statistics.mean(a_per)
    layers = [m for m in model.modules() if m.__class__.__name__ == "PackRLinear"]
    xs = {l: torch.randn(32 * 128, l.in_features, device=dev) for l in layers[:2]}
    dys = {l: torch.randn(32 * 128, l.out_features, device=dev) for l in layers[:2]}

    def packr_layers():
        for l in layers[:2]:
            cnt = l.lut_counts()
            K.forward(xs[l], l.W_p, l.W_f, l.lut, l.bias_f)
            K.backward(dys[l], xs[l], l.W_p, l.W_f, l.lut, cnt, True, True, True, l.bias_f is not None)
    _, l_per = timed(packr_layers, max(args.steps, 10), 3, 1)
    packr_ms = statistics.mean(l_per) * len(layers) / 2
    flops_packr = sum(6.0 * 32 * 128 * l.in_features * l.out_features for l in layers)
    line = {
        "metric": "BERT-base fine-tune sequences/s (FFN compressed to PackRLinear)", "value": round(value, 1),
        "unit": "sequences/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 model, bf16 W_f operands", "data": "synthetic (random ids, 2-class labels)",
        "config": {"workload": "bert: BERT-base (12 x 768, FFN 3072, 12 heads, vocab 30522), FFN layers as "
                               "PackRLinear (compress_model, layer_scope='ffn'), batch 32 x seq 128 per GPU",
                   "params": n_params, "packr_layers": len(layers),
                   "optimizer": "CUDA8BitAdam" if world == 1 else "ShardedAdam8 (ZeRO-1, overlapped reduce-scatter)",
                   "parallelism": f"dp{world}"},
        "shares_ms": {"step": round(ms_step, 4), "packr_linear_fwd_bwd": round(packr_ms, 4),
                      "adam": round(adam_ms, 4)},
        "roofline": {"bound": "tensor", "achieved": round(flops_packr / (packr_ms * 1e-3) / 1e12, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(flops_packr / (packr_ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4),
                     "traffic": None, "peak_source": f"{peak_kind} bf16_tflops",
                     "kernel": "PackRLinear forward + backward of the 24 compressed layers (f32 x: fp32-faithful dW)",
                     "algorithmic_flops_per_launch": flops_packr},
        "gpu_launches": None,
        "clocks": clk.summary(),
    }
    return line


def bench_llama(args, world, rank, peaks, peak_kind):
    """Llama-3-8B-shaped decoder (32 x 4096, FFN 14336, 32 q / 8 kv heads,
    vocab 128256), random init, every Linear a synthetic PackRLinear, bf16,
    seq 2048, micro-batch 1 per GPU, data parallel with ShardedAdam8."""
    from packr_b200 import workloads as wl
    from packr_b200.dp import ShardedAdam8
    dev = torch.device("cuda", torch.cuda.current_device())
    layers = int(os.environ.get("PACKR_BENCH_LLAMA_LAYERS", "32"))
    model = wl.llama_decoder(dev, layers=layers, seed=0)
    model.train()
    params = [p for p in model.parameters() if p.requires_grad]
    n_params = sum(p.numel() for p in params)
    opt = ShardedAdam8(params, lr=2e-5, weight_decay=0.01, overlap_grad_reduce=True)
    seq = args.tokens if args.tokens_given else 2048
    ids = wl.llama_batch(dev, seq=seq, seed=rank)
    linear_weights = sum(m.inner.in_features * m.inner.out_features for m in model.modules()
                         if m.__class__.__name__ == "_Cast")

    def step():
        opt.zero_grad(set_to_none=True)
        model(input_ids=ids, labels=ids).loss.backward()
        opt.step()
    with ClockSampler(torch.cuda.current_device()) as clk:
        total_ms, per = timed(step, args.steps, args.warmup, world, warm_seconds=1.5)
    ms_step = total_ms / args.steps
    value = world * seq / (ms_step * 1e-3)
    flops = 6.0 * seq * linear_weights
    line = {
        "metric": "Llama-3-8B-shaped training tokens/s (every Linear a PackRLinear)", "value": round(value, 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 activations, bf16 W_f operands, f32 accumulate", "data": "synthetic (random ids)",
        "config": {"workload": f"llama8b: {layers} x 4096, FFN 14336, 32/8 heads, vocab 128256, every Linear "
                               f"PackRLinear (synthetic init), seq {seq}, micro-batch 1 per GPU",
                   "params": n_params, "linear_weights": linear_weights,
                   "optimizer": "ShardedAdam8 (ZeRO-1, overlapped reduce-scatter)", "parallelism": f"dp{world}"},
        "roofline": {"bound": "tensor", "achieved": round(flops / (ms_step * 1e-3) / 1e12, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(flops / (ms_step * 1e-3) / 1e12 / peaks["bf16_tflops"], 4), "traffic": None,
                     "peak_source": f"{peak_kind} bf16_tflops",
                     "kernel": "whole step; FLOPs = 6 x tokens x Linear weights (attention not counted)",
                     "algorithmic_flops_per_launch": flops},
        "gpu_launches": None,
        "clocks": clk.summary(),
    }
    return line


def layer_launches(M: int, K: int, N: int) -> int:
    """libpackr_b200 kernels one PackRLinear forward + backward launches for
    bf16 x (K % 8 == 0), no bias, cached lut counts: forward = [predecode] +
    GEMM; backward = dY split + [predecode] + DX GEMM + DW GEMM + lut finalize.
    The predecode route is taken from 129 rows on when N % 16 == 0."""
    pre = 1 if (M >= 129 and N % 16 == 0) else 0
    return (pre + 1) + (1 + pre + 1 + 1 + 1)


def bench_ffn(args, world, rank, peaks, peak_kind):
    from packr_b200 import PackRLinear
    from packr_b200 import kernel as K
    from packr_b200.dp import ShardedAdam8
    M = args.tokens
    dev = torch.device("cuda", torch.cuda.current_device())
    layers, xs, dys = [], [], []
    for i, (name, k, n) in enumerate(FFN_LAYERS):
        # identical parameters on every rank (data parallel)
        lay = PackRLinear.synthetic(k, n, bias=False, device=dev, seed=100 + i, lut_std=0.02 * math.sqrt(768 / k),
                                    wf_std=0.002 * math.sqrt(768 / k))
        g = torch.Generator(device=dev).manual_seed(1000 * rank + i)  # each rank its own micro-batch
        xs.append(torch.randn(M, k, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True))
        dys.append(torch.randn(M, n, generator=g, device=dev).to(torch.bfloat16).float())
        layers.append(lay)
    params = [p for lay in layers for p in (lay.W_f, lay.lut)]
    opt = ShardedAdam8(params, lr=2e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                       overlap_grad_reduce=True, transport=getattr(args, "transport", "auto"))

    def zero():
        for lay, x in zip(layers, xs):
            lay.W_f.grad = None
            lay.lut.grad = None
            x.grad = None

    def fwd_bwd():
        zero()
        for lay, x, dy in zip(layers, xs, dys):
            lay(x).backward(dy)

    def step():
        fwd_bwd()
        opt.step()

    with ClockSampler(torch.cuda.current_device()) as clk:
        total_ms, per = timed(step, args.steps, args.warmup, world, warm_seconds=1.5)
    ms_step = total_ms / args.steps
    flops = ffn_flops(M)
    value = world * flops / (ms_step * 1e-3) / 1e12
    if getattr(args, "timeline", None):
        write_timeline(step, args.timeline, rank, {"n_gpus": world, "transport": opt.transport, "tokens": M,
                                                  "ms_per_step": ms_step})
    fb_total, _ = timed(fwd_bwd, args.steps, 2, world)
    fb_ms = fb_total / args.steps
    # the forward of the gate layer (predecode + GEMM), then its two kernels
    # timed alone: the GEMM over the decoded W (the dominant kernel) and the
    # HBM-bound predecode (5 bytes per weight)
    # (each timed over back-to-back calls between one event pair; a call's
    # operands and results, 0.3 GB for the GEMM, exceed L2)
    lay, x = layers[0], xs[0].detach()
    reps = max(args.steps, 10)
    fwd = lambda: K.forward(x, lay.W_p, lay.W_f, lay.lut, None)
    f_ms = b2b_ms(fwd, reps)
    Wd = K.predecode_bf16(lay.W_p, lay.W_f, lay.lut)
    g_ms = b2b_ms(lambda: K.forward_decoded(x, Wd, None), reps)
    p_ms = b2b_ms(lambda: K.predecode_bf16(lay.W_p, lay.W_f, lay.lut), reps)
    # the same two kernels replayed 10x from a CUDA graph (no host gaps)
    g_ms_graph = graph_b2b_ms(lambda: K.forward_decoded(x, Wd, None))
    p_ms_graph = graph_b2b_ms(lambda: K.predecode_bf16(lay.W_p, lay.W_f, lay.lut))
    del Wd
    f_flops = 2.0 * M * FFN_HIDDEN * FFN_INTER
    achieved = f_flops / (g_ms_graph * 1e-3) / 1e12
    pre_bytes = 5.0 * FFN_HIDDEN * FFN_INTER
    pre_gbs = pre_bytes / (p_ms_graph * 1e-3) / 1e9
    cnt = lay.lut_counts()
    bwd = lambda: K.backward(dys[0], x, lay.W_p, lay.W_f, lay.lut, cnt, True, True, True, False)
    b_ms = b2b_ms(bwd, reps)
    # the dW GEMM with its lut histogram, the step's largest kernel (launch
    # list): the full backward less the backward without dW and dlut (same
    # dY prep and dX GEMM), each as 10 calls replayed from one CUDA graph;
    # the difference also holds the dlut finalize (≈ 3 µs)
    full_g = graph_b2b_ms(lambda: K.backward(dys[0], x, lay.W_p, lay.W_f, lay.lut, cnt, True, True, True, False))
    dx_g = graph_b2b_ms(lambda: K.backward(dys[0], x, lay.W_p, lay.W_f, lay.lut, cnt, True, False, False, False))
    dw_ms = max(full_g - dx_g, 1e-6)
    dw_tflops = f_flops / (dw_ms * 1e-3) / 1e12
    # end to end: every step copies x and dY from pinned host memory and reads dlut back
    hx = [t.detach().cpu().pin_memory() for t in xs]
    hdy = [t.cpu().pin_memory() for t in dys]
    hres = torch.empty(len(layers), 256, dtype=torch.float32, pin_memory=True)
    # two sets of device input buffers: step i's copies go into set i % 2 as
    # soon as the step two back (the last reader of that set) is done with
    # it, so they run under the previous step's compute
    dx_in = [[torch.empty_like(t) for t in xs] for _ in range(2)]
    ddy_in = [[torch.empty_like(t) for t in dys] for _ in range(2)]
    set_free = [None, None]
    n_e2e = [0]

    copy_stream = torch.cuda.Stream()

    def e2e_step():
        # all host->device copies of the step go out on a copy stream; layer i
        # waits only for its own inputs
        k = n_e2e[0] & 1
        n_e2e[0] += 1
        zero()
        main = torch.cuda.current_stream()
        if set_free[k] is not None:
            copy_stream.wait_event(set_free[k])
        ready = []
        with torch.cuda.stream(copy_stream):
            for i in range(len(layers)):
                dx_in[k][i].copy_(hx[i], non_blocking=True)
                ddy_in[k][i].copy_(hdy[i], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                ready.append(ev)
        for i, lay in enumerate(layers):
            main.wait_event(ready[i])
            xi = dx_in[k][i].detach().requires_grad_(True)
            lay(xi).backward(ddy_in[k][i])
            hres[i].copy_(lay.lut.grad, non_blocking=True)
        opt.step()
        done = torch.cuda.Event()
        done.record(main)
        set_free[k] = done
    e2e_total, _ = timed(e2e_step, args.steps, max(args.warmup, 1), world)
    e2e_val = world * flops / (e2e_total / args.steps * 1e-3) / 1e12
    h2d = sum(t.numel() * t.element_size() for t in hx) + sum(t.numel() * t.element_size() for t in hdy)
    line = {
        "metric": "PackRLinear fwd+bwd TFLOP/s (Llama FFN shapes)", "value": round(value, 2), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 operands, f32 accumulate",
        "data": "synthetic (seeded; bf16 x ~ N(0,1), bf16-valued f32 dY ~ N(0,1), uniform W_p, fan-in scaled lut/W_f)",
        "config": {"workload": f"ffn: Llama-7B FFN gate/up/down (4096<->11008) PackRLinear training step, "
                               f"M={M} tokens per GPU",
                   "step": "forward + backward of the three layers, then the data-parallel 8-bit AdamW update "
                           "(gradient reduce-scatter started per bucket from the gradient hooks during the "
                           "backward, AdamW on this rank's 1/N state shard; transport 'push': the AdamW kernel "
                           "also stores the new W_f/lut shard into every other GPU's copy over NVLink, then one "
                           "1-element all-reduce; 'nccl': all-gather; no collectives at N=1); value counts the "
                           "6*M*K*N GEMM FLOPs",
                   "hidden": FFN_HIDDEN, "intermediate": FFN_INTER, "tokens_per_gpu": M,
                   "flops_per_step_per_gpu": flops, "l2": "inputs larger than L2 (~0.9 GB of operands per step)",
                   "parallelism": f"dp{world}, ZeRO-1 sharded 8-bit optimizer state",
                   "transport": opt.transport if world > 1 else None},
        "fwd_bwd_only": {"tflops": round(world * flops / (fb_ms * 1e-3) / 1e12, 2), "ms_per_step": round(fb_ms, 4)},
        "phases_ms_gate_layer": {"forward": round(f_ms, 4), "forward_gemm": round(g_ms, 4),
                                 "predecode": round(p_ms, 4), "backward": round(b_ms, 4),
                                 "timing": "back-to-back calls between one pair of CUDA events"},
        "roofline": {"bound": "tensor", "achieved": round(dw_tflops, 1), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(dw_tflops / peaks["bf16_tflops"], 4),
                     "traffic": load_traffic("packr_gemm_kernel<DW>", "ffn_gate_M%d" % M),
                     "peak_source": f"{peak_kind} bf16_tflops (burst; kernel timed alone)",
                     "kernel": "packr_gemm_kernel<DW> with the lut histogram (gate 4096->11008): the step's "
                               "largest kernel; time = full backward - backward without dW/dlut, each replayed "
                               "10x from a CUDA graph",
                     "ms": round(dw_ms, 4), "algorithmic_flops_per_launch": f_flops},
        "roofline_fwd": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                         "traffic": load_traffic("packr_gemm_kernel<FWD,plain>", "ffn_gate_M%d" % M),
                         "peak_source": f"{peak_kind} bf16_tflops (burst; kernel timed alone)",
                         "kernel": "packr_gemm_kernel<FWD, B_PLAIN, 512-row tiles> (gate 4096->11008, decoded W), "
                                   "replayed 10x from a CUDA graph",
                         "ms": round(g_ms_graph, 4),
                         "algorithmic_flops_per_launch": f_flops},
        "roofline_predecode": {"bound": "hbm", "achieved": round(pre_gbs, 1), "peak": peaks["hbm_gbs"],
                               "unit": "GB/s", "frac": round(pre_gbs / peaks["hbm_gbs"], 4),
                               "traffic": load_traffic("predecode_kernel", "ffn_gate"),
                               "kernel": "predecode_kernel (gate W 4096x11008), replayed 10x from a CUDA graph",
                               "ms": round(p_ms_graph, 4),
                               "algorithmic_bytes_per_launch": pre_bytes},
        "e2e": {"value": round(e2e_val, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": hres.numel() * 4,
                "how": "each step copies x and dY of the three layers from pinned host memory (copy stream, "
                       "two alternating device buffer sets, so a step's copies run under the previous step's "
                       "compute) and reads dlut back"},
        "gpu_launches": args.steps * (sum(layer_launches(M, k, n) for _, k, n in FFN_LAYERS) + len(opt.buckets)),
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_linear_port(args.cpu_seconds)
    del layers, xs, dys, opt, hx, hdy, dx_in, ddy_in
    torch.cuda.empty_cache()
    if not args.no_extras:
        line.update(ffn_extras(args, world, rank, peaks))
    return line


# ---------------------------------------------------------------- extras of the default line
SWEEP_M = (1, 16, 256, 4096, 16384)


def ffn_bytes(M: int) -> float:
    """Algorithmic bytes of one fwd+bwd of the three FFN layers: per layer
    8KN + 6MK + 8MN (W_f / W_p read by the forward and by the dX GEMM, dW_f
    written; x, dX, out and dY once each)."""
    return float(sum(8 * k * n + 6 * M * k + 8 * M * n for _, k, n in FFN_LAYERS))


def replayable(fn):
    """fn captured in a CUDA graph (its launches then run without the host's
    gaps between them), or fn itself when capture is not possible."""
    try:
        return graph_of(fn), "CUDA graph replay"
    except Exception:
        torch.cuda.synchronize()
        return fn, "eager"


def ffn_sweep(dev, peaks) -> dict:
    """fwd+bwd of the gate/up/down layers through PackRLinear's autograd at
    each token count of the sweep (bf16 x, f32 dY, dW_f + dlut + dX)."""
    from packr_b200 import PackRLinear
    layers = [PackRLinear.synthetic(k, n, bias=False, device=dev, seed=200 + i, lut_std=0.02 * math.sqrt(768 / k),
                                    wf_std=0.002 * math.sqrt(768 / k)) for i, (_, k, n) in enumerate(FFN_LAYERS)]
    for lay in layers:
        lay.lut_counts()
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    out = {}
    for M in SWEEP_M:
        g = torch.Generator(device=dev).manual_seed(7000 + M)
        xs = [torch.randn(M, k, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
              for _, k, _ in FFN_LAYERS]
        dys = [torch.randn(M, n, generator=g, device=dev).to(torch.bfloat16).float() for _, _, n in FFN_LAYERS]

        def fb():
            for lay, x, dy in zip(layers, xs, dys):
                lay.W_f.grad = None
                lay.lut.grad = None
                x.grad = None
                lay(x).backward(dy)
        run, how = replayable(fb) if M <= 256 else (fb, "eager")
        ms = b2b_ms(run, 10, min_seconds=0.05)
        flops, nbytes = ffn_flops(M), ffn_bytes(M)
        tf, gbs = flops / (ms * 1e-3) / 1e12, nbytes / (ms * 1e-3) / 1e9
        bound = "tensor" if flops / nbytes >= ridge else "hbm"
        out[str(M)] = {"ms": round(ms, 4), "tflops": round(tf, 2), "gbs": round(gbs, 1), "bound": bound,
                       "frac": round(tf / peaks["bf16_tflops"] if bound == "tensor" else gbs / peaks["hbm_gbs"], 4),
                       "launch": how}
        del xs, dys, run
    return out


def decode_points(dev, peaks) -> dict:
    """Forward of the three FFN layers at 1 and 16 tokens, replayed from a
    CUDA graph; GB/s of packed weights (3 bytes per weight)."""
    from packr_b200 import kernel as K
    from packr_b200.synthetic import linear_case
    wbytes = sum(3.0 * k * n for _, k, n in FFN_LAYERS)
    out = {}
    for M in (1, 16):
        cases = []
        for i, (_, k, n) in enumerate(FFN_LAYERS):
            c = linear_case(M, k, n, x_dtype=torch.bfloat16, bias=False, seed=100 + i, fanin_scaled=True)
            cases.append({kk: (v.to(dev) if v is not None else None) for kk, v in c.items()})

        def fwd():
            for c in cases:
                K.forward(c["x"], c["W_p"], c["W_f"], c["lut"], None)
        ms = b2b_ms(graph_of(fwd), 50)
        algo = sum(3.0 * k * n + 2.0 * M * k + 4.0 * M * n for _, k, n in FFN_LAYERS)
        out[str(M)] = {"ms": round(ms, 5), "gbs": round(wbytes / (ms * 1e-3) / 1e9, 1),
                       "frac": round(algo / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                       "kernel": "gemv_cluster_kernel" if M <= 4 else "skinny_kernel + gemv_reduce_kernel"}
        del cases
    return out


def adam8_point(dev, peaks) -> dict:
    """CUDA8BitAdam over one 110,000,000-element bf16 parameter (lr 2e-5,
    betas (0.9, 0.999), eps 1e-8, wd 0.01): Gparam/s and HBM fraction at
    10.0625 algorithmic bytes per parameter."""
    from packr_b200.cuda_adam import CUDA8BitAdam
    from packr_b200.synthetic import adam_grad, adam_params
    n = ADAM_N
    p = torch.nn.Parameter(adam_params(n, dtype=torch.bfloat16, seed=0, device=dev))
    p.grad = adam_grad(n, 1, dtype=torch.bfloat16, device=dev)
    opt = CUDA8BitAdam([p], lr=2e-5, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    ms = b2b_ms(opt.step, 20)
    gbs = n * ADAM_BYTES_PER_PARAM / (ms * 1e-3) / 1e9
    return {"ms": round(ms, 5), "gparam_s": round(n / (ms * 1e-3) / 1e9, 2), "gbs": round(gbs, 1),
            "frac": round(gbs / peaks["hbm_gbs"], 4), "kernel": "adam8_kernel<bf16>",
            "bytes_per_param": ADAM_BYTES_PER_PARAM}


def llama8b_point(args, world, rank, dev) -> dict:
    """The Llama-3-8B-shaped decoder (32 x 4096, FFN 14336, 32/8 heads, vocab
    128256, every Linear a PackRLinear), seq 2048, micro-batch 1 per GPU,
    data parallel over all ranks with ShardedAdam8: whole-job tokens/s."""
    from packr_b200 import workloads as wl
    from packr_b200.dp import ShardedAdam8
    layers = int(os.environ.get("PACKR_BENCH_LLAMA_LAYERS", "32"))
    t0 = time.perf_counter()
    model = wl.llama_decoder(dev, layers=layers, seed=0)
    model.train()
    opt = ShardedAdam8([p for p in model.parameters() if p.requires_grad], lr=2e-5, weight_decay=0.01,
                       overlap_grad_reduce=True)
    ids = wl.llama_batch(dev, seq=2048, seed=rank)
    build_s = time.perf_counter() - t0

    def step():
        opt.zero_grad(set_to_none=True)
        model(input_ids=ids, labels=ids).loss.backward()
        opt.step()
    steps = 5
    total_ms, _ = timed(step, steps, 3, world)
    ms = total_ms / steps
    del model, opt
    torch.cuda.empty_cache()
    return {"tokens_s": round(world * 2048 / (ms * 1e-3), 1), "ms_per_step": round(ms, 2), "n_gpus": world,
            "layers": layers, "steps": steps, "warmup": 3, "build_s": round(build_s, 1),
            "workload": "Llama-3-8B shape, every Linear a PackRLinear, seq 2048, micro-batch 1 per GPU, "
                        "dp with ShardedAdam8 (max over ranks)"}


def ffn_extras(args, world, rank, peaks) -> dict:
    """The rest of the headline metric beside the ffn step: the 8-bit AdamW
    rate, the fwd+bwd token-count sweep and the decode-bound forward (one
    GPU), and the Llama-3-8B-shaped data-parallel step (every N)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    ex = {}
    if world == 1:
        ex["adam8"] = adam8_point(dev, peaks)
        torch.cuda.empty_cache()
        ex["sweep"] = ffn_sweep(dev, peaks)
        torch.cuda.empty_cache()
        ex["decode"] = decode_points(dev, peaks)
        torch.cuda.empty_cache()
    if not args.no_llama:
        ex["llama8b"] = llama8b_point(args, world, rank, dev)
    return ex


def profile_once(args):
    """One forward and one backward of the gate layer (4096 -> 11008, M
    tokens), then one CUDA8BitAdam step over its W_f: the launch sequence an
    ncu capture of this workload sees (forward GEMM first)."""
    from packr_b200 import PackRLinear
    from packr_b200.cuda_adam import CUDA8BitAdam
    dev = torch.device("cuda", torch.cuda.current_device())
    M = args.tokens
    lay = PackRLinear.synthetic(FFN_HIDDEN, FFN_INTER, bias=True, device=dev, seed=100)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(M, FFN_HIDDEN, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(M, FFN_INTER, generator=g, device=dev).to(torch.bfloat16).float()
    lay.lut_counts()
    lay(x).backward(dy)
    CUDA8BitAdam([lay.W_f, lay.lut], lr=2e-5, weight_decay=0.01).step()
    torch.cuda.synchronize()


LLAMA_LINEARS = [("q_proj", 4096, 4096), ("k_proj", 4096, 1024), ("v_proj", 4096, 1024), ("o_proj", 4096, 4096),
                 ("gate_proj", 4096, 14336), ("up_proj", 4096, 14336), ("down_proj", 14336, 4096)]


def cpu_from_linear_port(budget_s: float):
    """The reference's from_linear operation sequence (packr/layer.py:106-159,
    restated op for op in oracle/reference_port.py) on the host cores, on a
    1024 -> 4096 bf16 layer (the reference's torch.quantile refuses the full
    Llama layers)."""
    from oracle import reference_port
    torch.manual_seed(0)
    lin = torch.nn.Linear(1024, 4096, bias=False).to(torch.bfloat16)
    times = []
    t0 = time.perf_counter()
    while len(times) < 2 or time.perf_counter() - t0 < budget_s:
        a = time.perf_counter()
        reference_port.from_linear(lin.weight, None)
        times.append(time.perf_counter() - a)
    sec = statistics.median(times)
    return {"value": 1024 * 4096 / sec / 1e9, "unit": "Gweights/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"from_linear of a 1024->4096 bf16 Linear, {len(times)} timed samples (median); "
                                      "the reference's torch operation sequence on the CPU",
            "host_cores": os.cpu_count()}


def bench_from_linear(args, world, rank, peaks, peak_kind):
    """PackRLinear.from_linear (GPU path) of one Llama-3-8B decoder layer's
    seven bf16 weights; algorithmic bytes 5 per weight (read W 2, write W_p 1
    and W_f 2)."""
    from packr_b200 import PackRLinear, kernel as K
    from packr_b200.layer import _build_codebook
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(0)
    lins = []
    for name, k, n in LLAMA_LINEARS:
        lin = torch.nn.Linear(k, n, bias=False, device="meta")
        lin.weight = torch.nn.Parameter((torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16))
        lins.append(lin)
    nw = sum(k * n for _, k, n in LLAMA_LINEARS)

    def step():
        for lin in lins:
            PackRLinear.from_linear(lin)
    with ClockSampler(torch.cuda.current_device()) as clk:
        total_ms, per = timed(step, args.steps, args.warmup, world, warm_seconds=1.0)
    ms_step = total_ms / args.steps
    value = world * nw / (ms_step * 1e-3) / 1e9
    # the encode pass alone (the dominant kernel), on the largest weight
    big = lins[4].weight.detach()
    cb = _build_codebook().to(dev)
    scale = torch.full((), 40.0, device=dev)
    _, enc = timed(lambda: K.from_linear_encode(big, cb, scale), args.steps, args.warmup, world)
    enc_bytes = 5.0 * big.numel()
    achieved = enc_bytes / (statistics.mean(enc) * 1e-3) / 1e9
    host = [lin.weight.detach().cpu().pin_memory() for lin in lins]
    dlin = []
    for (name, k, n), h in zip(LLAMA_LINEARS, host):
        lin = torch.nn.Linear(k, n, bias=False, device="meta")
        lin.weight = torch.nn.Parameter(torch.empty_like(h, device=dev))
        dlin.append(lin)
    hwp = [torch.empty(k, n, dtype=torch.uint8, pin_memory=True) for _, k, n in LLAMA_LINEARS]
    hwf = [torch.empty(k, n, dtype=torch.bfloat16, pin_memory=True) for _, k, n in LLAMA_LINEARS]

    def e2e_step():
        for i, lin in enumerate(dlin):
            lin.weight.data.copy_(host[i], non_blocking=True)
            pk = PackRLinear.from_linear(lin)
            hwp[i].copy_(pk.W_p, non_blocking=True)
            hwf[i].copy_(pk.W_f, non_blocking=True)
    e2e_ms, _ = timed(e2e_step, max(1, args.steps // 2), max(args.warmup, 1), world)
    e2e_steps = max(1, args.steps // 2)
    line = {
        "metric": "PackRLinear.from_linear Gweights/s (Llama-3-8B decoder layer, bf16)", "value": round(value, 3),
        "unit": "Gweights/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 weights, f32 select and encode", "data": "synthetic (seeded N(0, 0.02) weights)",
        "config": {"workload": "from_linear: q/k/v/o/gate/up/down weights of one Llama-3-8B layer "
                               f"({nw / 1e6:.1f} M weights) per GPU",
                   "l2": "weights 0.44 GB per step, larger than L2", "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": f"{peak_kind} hbm_gbs",
                     "kernel": "encode_kernel<bf16> on the 14336 x 4096 gate weight",
                     "algorithmic_bytes_per_launch": enc_bytes},
        "e2e": {"value": round(world * nw / (e2e_ms / e2e_steps * 1e-3) / 1e9, 3), "unit": "Gweights/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host),
                "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in hwp + hwf)},
        "gpu_launches": args.steps * len(LLAMA_LINEARS) * 9,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_from_linear_port(args.cpu_seconds)
    return line


def reference_arm(args, world, rank):
    if rank != 0:
        return None
    # torchrun sets OMP_NUM_THREADS=1 in every rank; this arm runs in rank 0
    # alone and may use every host thread the process is allowed
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    if args.workload == "adam8":
        cb = cpu_adam_reference(1 << 24, max(2.0, 0.5 * args.steps))
        return {"impl": "reference", "metric": "8-bit AdamW Gparam/s", "value": round(cb["value"], 5),
                "unit": "Gparam/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": {"workload": "adam8: 8-bit AdamW step (bounded CPU sample)"},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": round(cb["value"], 5), "unit": "Gparam/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "decode":
        M = args.tokens if args.tokens_given else 16
        cb = cpu_decode_port(max(5.0, 0.5 * args.steps), M)
        return {"impl": "reference", "metric": f"PackRLinear decode forward GB/s of packed weights (M={M})",
                "value": round(cb["value"], 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic",
                "config": {"workload": f"decode: forward of the Llama-7B FFN layers at M={M} (CPU)"},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": round(cb["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "from_linear":
        cb = cpu_from_linear_port(max(5.0, 0.5 * args.steps))
        return {"impl": "reference", "metric": "PackRLinear.from_linear Gweights/s (Llama-3-8B decoder layer, bf16)",
                "value": round(cb["value"], 5), "unit": "Gweights/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16 weights", "data": "synthetic",
                "config": {"workload": "from_linear: 1024->4096 bf16 Linear (CPU; the reference refuses the "
                                       "Llama gate/up/down weights above 2^24 elements)"},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": round(cb["value"], 5), "unit": "Gweights/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "ffn":
        cb = cpu_linear_port(max(5.0, 0.5 * args.steps))
        return {"impl": "reference", "metric": "PackRLinear fwd+bwd TFLOP/s (Llama FFN shapes)",
                "value": round(cb["value"], 5), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 (bf16-valued operands)", "data": "synthetic",
                "config": {"workload": "ffn: Llama-7B FFN PackRLinear fwd+bwd (bounded CPU sample)"},
                "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": round(cb["value"], 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
    if args.workload == "llama8b":
        return {"impl": "reference", "unavailable": "no CPU arm for the Llama-3-8B-shaped step: that configuration "
                "is a scale-out measurement (a host step of the 8B-parameter model would take hours); the ffn "
                "workload's reference arm times the same PackRLinear op sequence on the host"}
    if args.workload == "bert":
        return {"impl": "reference", "unavailable": "no CPU arm for the BERT-base training step (encoder, loss and "
                "optimizer on the host exceed a bounded sample); the ffn workload's reference arm times the same "
                "PackRLinear op sequence on the host"}
    raise SystemExit(f"unknown workload {args.workload}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="ffn",
                    choices=["ffn", "adam8", "decode", "bert", "llama8b", "from_linear"])
    ap.add_argument("--tokens", type=int, default=None, help="tokens per GPU (ffn: 4096, decode: 16)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="ffn: leave out the adam8 / sweep / decode / llama8b keys of the default line")
    ap.add_argument("--no-llama", action="store_true", help="ffn: leave out the llama8b key")
    ap.add_argument("--transport", default="auto", choices=["auto", "push", "nccl"],
                    help="ffn, N>1: how ShardedAdam8 hands out the new parameters")
    ap.add_argument("--timeline", default=None,
                    help="ffn: after the timed steps, write rank 0's CUPTI timeline of 3 more steps "
                         "(every kernel and copy: start, duration, stream) to this JSON file")
    ap.add_argument("--profile-once", action="store_true",
                    help="ffn: run each kernel of one gate-layer step once (for ncu captures), print nothing")
    args = ap.parse_args()
    args.tokens_given = args.tokens is not None
    if args.tokens is None:
        args.tokens = FFN_M
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = reference_arm(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup()
    peaks, peak_kind = load_peaks()
    if args.profile_once:
        profile_once(args)
        return
    fn = {"ffn": bench_ffn, "adam8": bench_adam8, "decode": bench_decode, "bert": bench_bert,
          "llama8b": bench_llama, "from_linear": bench_from_linear}[args.workload]
    line = fn(args, world, rank, peaks, peak_kind)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
