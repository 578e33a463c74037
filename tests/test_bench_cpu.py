"""bench.py's reference arm (the reference's CPU implementation of the path,
timed on the host cores) keeps its JSON contract: one line, impl
"reference", the metric / unit / direction of the GPU arm for the same
workload, a cpu_baseline describing the run, and an e2e entry with no
host<->device bytes.  Under a 2-rank launch only rank 0 prints."""
import json
import subprocess
import sys

import pytest

from conftest import REPO

UNITS = {"ffn": "TFLOP/s", "adam8": "Gparam/s", "decode": "GB/s", "from_linear": "Gweights/s"}


def run_bench(*args, timeout=300):
    r = subprocess.run([sys.executable, *args], cwd=REPO, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]


@pytest.mark.parametrize("workload", sorted(UNITS))
def test_reference_arm_line(workload):
    lines = run_bench("bench.py", "--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "3")
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["higher_is_better"] is True
    assert d["unit"] == UNITS[workload] and d["value"] > 0 and d["metric"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    # the line's value is cpu_baseline's, rounded to 3 or more decimals
    assert cb["value"] == pytest.approx(d["value"], rel=1e-3, abs=5e-4)
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("workload", ["bert", "llama8b"])
def test_reference_arm_without_cpu_baseline_says_so(workload):
    lines = run_bench("bench.py", "--impl", "reference", "--workload", workload, "--steps", "1", "--warmup", "3")
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["unavailable"]


def test_reference_arm_two_ranks_prints_once():
    lines = run_bench("-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
                      "127.0.0.1", "--master-port", "29541", "bench.py", "--impl", "reference", "--workload", "adam8",
                      "--gpus", "2", "--steps", "1", "--warmup", "3")
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2
