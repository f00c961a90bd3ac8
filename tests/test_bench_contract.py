"""bench.py's reference arm (--impl reference) on CPU: one JSON line with the
keys of the benchmark contract, the same metric and config as the CUDA arm,
a cpu_baseline describing the run and an e2e block with no copies; under
torchrun only rank 0 prints, every rank exits 0.  (The CUDA arm needs a
B200 and is run there.)"""
import json
import os
import socket
import subprocess
import sys

import pytest

import holo_b200 as hb
from conftest import ROOT

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}
ARGS = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3", "--cpu-budget", "0.3"]


def json_lines(out):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def check_line(d):
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["warmup"] >= 3 and d["steps"] == 1
    assert d["higher_is_better"] is True and d["unit"] == "GB/s"
    assert d["config"]["workload"].startswith("quant matvec sweep")
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_one_line():
    p = subprocess.run([sys.executable] + ARGS, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]
    lines = json_lines(p.stdout)
    assert len(lines) == 1, p.stdout
    check_line(lines[0])
    assert lines[0]["n_gpus"] == 1


def test_reference_arm_under_torchrun():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}"] + ARGS[:1] + ["--gpus", "2"] + ARGS[1:]
    p = subprocess.run(["timeout", "-k", "30", "600"] + cmd, cwd=ROOT, capture_output=True, text=True,
                       env=dict(os.environ, OMP_NUM_THREADS="1"))
    assert p.returncode == 0, p.stderr[-3000:]
    lines = json_lines(p.stdout)
    assert len(lines) == 1, p.stdout   # rank 0 alone
    check_line(lines[0])
    assert lines[0]["n_gpus"] == 2


def test_decode_cpu_extrapolation():
    """The 70B decode's CPU figure (matmul_q on row samples of the layer
    shapes, scaled to the model): finite, and slower for more layers."""
    sys.path.insert(0, str(ROOT))
    import bench
    cfg = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=768, vocab=1000,
               layer_type=hb.Q4_0, out_type=hb.Q4_0)
    a = bench.decode_cpu_extrapolated(cfg, budget_s=0.2)
    if a["value"] is None:
        pytest.skip(a["sample"])
    b = bench.decode_cpu_extrapolated(dict(cfg, n_layers=20), budget_s=0.2)
    assert a["kind"] == "reference" and a["unit"] == "tokens/s" and a["cores"] >= 1
    assert 0 < b["value"] < a["value"]
