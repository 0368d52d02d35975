"""bench.py's JSON contract, checked on the CPU.

* `--impl reference` (the reference's own CPU path -- its torch oracle from the offline install
  under baseline/_ref, or the numpy port when that is absent -- timed on the host cores on
  whole sequences of the workload) prints one JSON line with the keys the driver reads: impl, metric, value, unit,
  steps / warmup, higher_is_better, config.workload, a cpu_baseline describing the run, and an
  e2e object with zero host<->device bytes.
* The product arm has no CPU fallback: without a GPU it exits non-zero.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args, timeout=300):
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_json_line():
    r = _run("--impl", "reference", "--workload", "fp16_b1_ctx4k", "--steps", "1",
             "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TB/s" and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 0 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"].startswith("fp16_b1_ctx4k")
    cb = d["cpu_baseline"]
    installed = os.path.exists(os.path.join(ROOT, "baseline", "_ref", "bpt", "reference.py"))
    assert cb["kind"] == ("reference" if installed else "port")
    assert cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert "[4096] tokens" in cb["sample"], "whole sequences at their true length"
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_under_torchrun_prints_once():
    """Launched like the driver's N-GPU runs: rank 0 alone runs and prints one line, the other
    ranks exit 0 without work."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port",
                        str(port), os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--gpus", "2", "--workload", "fp16_b1_ctx4k", "--steps", "1",
                        "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    assert json.loads(lines[0])["impl"] == "reference"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure path")
def test_product_arm_fails_without_gpu():
    r = _run("--steps", "1", "--warmup", "0", timeout=120)
    assert r.returncode != 0
    assert not any(ln.startswith("{") for ln in r.stdout.splitlines())
