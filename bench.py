#!/usr/bin/env python3
"""Benchmark of the B200 decode-path library (one JSON line on rank 0).

Workload: the quantized matvec sweep over the
Llama-7B FFN shapes -- Q4_0 and Q4_K, 11008x4096 (up/gate) and 4096x11008
(down), seeds 0-3: 16 distinct matrices, 406 MB of GGUF blocks per pass, so
every pass streams more than the 126 MB L2 and no matrix is re-read from L2.
One step = one pass of the 16 matvecs (replayed as one CUDA graph).

Metric: quant matvec HBM GB/s = algorithmic bytes (GGUF weight bytes + fp32
x + fp32 y) / time.  With --gpus N every rank runs the sweep on its own GPU
(weak scaling); value = bytes of all ranks / max-over-ranks time.

--impl reference times the reference engine's own CPU matvec (matmul_q,
src/ai/llm.c:770-926, compiled from source into oracle/_ref) on the host
cores, on a row sample of the same sweep sized to finish in about a minute.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "google-classic_b200"))

import holo_b200 as hb  # noqa: E402
from holo_b200 import synth  # noqa: E402

METRIC = "quant matvec HBM GB/s (% of 8 TB/s); batch-1 decode tokens/s at 1/2/4/8 B200"
UNIT = "GB/s"
SHAPES = [(11008, 4096), (4096, 11008)]
TYPES = [hb.Q4_0, hb.Q4_K]
SEEDS = [0, 1, 2, 3]
FALLBACK_HBM_GBS = 6650.0


def sweep_specs():
    return [(gt, r, c, s) for gt in TYPES for (r, c) in SHAPES for s in SEEDS]


def algo_bytes(gt, rows, cols):
    return rows * hb.row_bytes(gt, cols) + 4 * cols + 4 * rows


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def config(args, n):
    return {
        "workload": "quant matvec sweep: Q4_0+Q4_K x {11008x4096, 4096x11008} x seeds 0-3 (BASELINE configs[1])",
        "matrices_per_step": len(sweep_specs()),
        "weight_bytes_per_step": sum(r * hb.row_bytes(gt, c) for gt, r, c, _ in sweep_specs()),
        "act_mode": args.act,
        "l2": "inputs larger than L2: 406 MB of distinct weights per step, each read once",
        "parallelism": f"replicas x{n}" if n > 1 else "1 GPU",
    }


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = []
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = time.mktime(time.strptime(f[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
            except ValueError:
                continue
            rows.append((ts, f))
        window = [f for ts, f in rows if self.t0 is not None and self.t0 - 1 <= ts <= (self.t1 or ts) + 1]
        use = window or [f for _, f in rows]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for f in use:
            for n_, v in zip(names, f[6:10]):
                if v.lower() == "active":
                    reasons.add(n_)
        sm = [float(f[2]) for f in use if f[2].replace(".", "").isdigit()]
        mx = [float(f[3]) for f in use if f[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(use), "in_window": len(window)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = hb.Device(local_rank, world)
    lib = dev.lib
    specs = sweep_specs()
    bytes_step = sum(algo_bytes(gt, r, c) for gt, r, c, _ in specs)

    # weights resident in HBM, tiled once
    mats = []
    for gt, r, c, s in specs:
        W = synth.quant_matrix(gt, r, c, s)
        Wd = dev.upload_quant(W, gt, r, c)
        x = synth.activation(c, s)
        mats.append(dict(gt=gt, rows=r, cols=c, W=W, Wd=Wd, x=x, xd=dev.upload(x), yd=dev.alloc(4 * r)))
    dev.check("upload")
    stream = torch.cuda.ExternalStream(lib.cuda_get_stream())
    lib.cuda_set_pdl(0 if args.no_pdl else 1)   # weights are constant from here on

    def capture(act):
        for m in mats:   # one-time set-up outside capture
            lib.cuda_matvec(m["yd"], m["Wd"], m["xd"], m["rows"], m["cols"], m["gt"], act, None)
        dev.sync()
        if lib.cuda_capture_begin() != 0:
            dev.check("capture")
        for m in mats:
            lib.cuda_matvec(m["yd"], m["Wd"], m["xd"], m["rows"], m["cols"], m["gt"], act, None)
        g = lib.cuda_capture_end()
        dev.check("capture end")
        return g

    def timed(graph, steps, warmup, sampler=None):
        for _ in range(warmup):
            lib.cuda_graph_launch(graph)
        dev.sync()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if sampler:
            sampler.mark("t0")
        e0.record(stream)
        for _ in range(steps):
            lib.cuda_graph_launch(graph)
        e1.record(stream)
        e1.synchronize()
        if sampler:
            sampler.mark("t1")
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dist.barrier()
        dev.check("timed region")
        return float(t.item())

    acts = {"q8": hb.ACT_Q8, "f32": hb.ACT_F32}
    primary = acts[args.act]
    g_main = capture(primary)
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ms_total = timed(g_main, args.steps, args.warmup, sampler)
    clocks = sampler.stop() if sampler else None
    ms_step = ms_total / args.steps
    value = world * bytes_step / (ms_step * 1e-3) / 1e9

    # the other activation mode, same sweep (reported beside the headline)
    other = "f32" if args.act == "q8" else "q8"
    g_other = capture(acts[other])
    ms_other = timed(g_other, max(1, args.steps // 4), max(3, args.warmup // 2)) / max(1, args.steps // 4)
    lib.cuda_graph_free(g_other)

    # per-launch kernel time of the dominant kernel (the tiled matvec): event
    # pairs around each launch on the library stream, outside graphs
    kt = []
    for _ in range(3):
        for m in mats:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            lib.cuda_matvec(m["yd"], m["Wd"], m["xd"], m["rows"], m["cols"], m["gt"], primary, None)
            b.record(stream)
            kt.append((a, b, algo_bytes(m["gt"], m["rows"], m["cols"])))
    torch.cuda.synchronize()
    k_ms = [a.elapsed_time(b) for a, b, _ in kt]
    k_bytes = [nb for _, _, nb in kt]
    peak, peak_kind = peaks()
    kernel_gbs = sum(k_bytes) / (sum(k_ms) * 1e-3) / 1e9

    # end to end through the reference-facing C ABI: pinned host x in, host y
    # out, every step (cuda_memcpy_h2d, cuda_matmul_q4_*, cuda_memcpy_d2h)
    lib.cuda_set_act_mode(primary)
    pins = []
    for m in mats:
        hx = torch.from_numpy(m["x"]).pin_memory()
        hy = torch.empty(m["rows"], dtype=torch.float32).pin_memory()
        pins.append((hx, hy))
    fn = {hb.Q4_0: lib.cuda_matmul_q4_0, hb.Q4_K: lib.cuda_matmul_q4_k}
    e2e_steps = max(3, min(args.steps, 200))
    h2d = sum(4 * m["cols"] for m in mats)
    d2h = sum(4 * m["rows"] for m in mats)

    def e2e_step():
        for m, (hx, hy) in zip(mats, pins):
            lib.cuda_memcpy_h2d(m["xd"], hx.data_ptr(), 4 * m["cols"])
            fn[m["gt"]](m["yd"], m["Wd"], m["xd"], m["rows"], m["cols"])
            lib.cuda_memcpy_d2h(hy.data_ptr(), m["yd"], 4 * m["rows"])

    for _ in range(3):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())
    dev.check("e2e")
    e2e_value = world * bytes_step * e2e_steps / e2e_s / 1e9
    # the library output of the last e2e step equals the graph's output
    lib.cuda_set_act_mode(hb.ACT_Q8)

    # the reference's own CUDA kernels (src/ai/cuda_ops.cu built for sm_100a) on
    # raw blocks: the GPU kernels this library replaces
    ref_gpu = None
    if rank == 0 and not args.no_ref_gpu:
        ref_gpu = ref_gpu_kernels(mats, dev, torch)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(mats, bytes_step, budget_s=args.cpu_budget)

    traffic = read_traffic()
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 (dp4a) x q4 codes, fp32 scales" if args.act == "q8" else "f32",
        "data": "synthetic (seeded GGUF blocks with the BASELINE config distributions)",
        "config": config(args, world),
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(kernel_gbs / peak, 4), "peak_source": peak_kind,
                     "traffic": traffic.get("bytes_per_launch") if traffic else None,
                     "algorithmic_bytes_per_launch": round(sum(k_bytes) / len(k_bytes)),
                     "kernel_avg_us": round(1e3 * sum(k_ms) / len(k_ms), 3),
                     "step_frac": round(value / world / peak, 4)},
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "cuda_memcpy_h2d + cuda_matmul_q4_0/q4_k + cuda_memcpy_d2h per matvec (reference ABI)"},
        "gpu_launches": args.steps * len(mats),
        "clocks": clocks,
        "other_act_mode": {"act": other, "value": round(world * bytes_step / (ms_other * 1e-3) / 1e9, 2),
                           "ms_per_step": round(ms_other, 5)},
    }
    if ref_gpu:
        line["reference_gpu_kernels"] = ref_gpu
    if cpu:
        line["cpu_baseline"] = cpu
    lib.cuda_graph_free(g_main)
    for m in mats:
        for k in ("Wd", "xd", "yd"):
            dev.free(m[k])
    if rank == 0:
        print(json.dumps(line), flush=True)


def read_traffic():
    p = ROOT / "profiles" / "matvec_traffic.txt"
    if not p.exists():
        return None
    out = {}
    for line in p.read_text().splitlines():
        if "=" in line and not line.startswith("#"):
            k, v = line.split("=", 1)
            try:
                out[k.strip()] = float(v.strip())
            except ValueError:
                pass
    return out


def ref_gpu_kernels(mats, dev, torch):
    import ctypes as C
    so = ROOT / "oracle" / "_ref" / "libholo_ref_cuda.so"
    if not so.exists():
        return None
    ref = C.CDLL(str(so))
    for n in ("cuda_matmul_q4_0", "cuda_matmul_q4_k"):
        getattr(ref, n).argtypes = [C.c_void_p] * 3 + [C.c_int, C.c_int]
    fn = {hb.Q4_0: ref.cuda_matmul_q4_0, hb.Q4_K: ref.cuda_matmul_q4_k}
    raws = [dev.upload(m["W"]) for m in mats]
    dev.sync()
    torch.cuda.synchronize()

    def one():
        for m, raw in zip(mats, raws):
            fn[m["gt"]](m["yd"], raw, m["xd"], m["rows"], m["cols"])

    for _ in range(3):
        one()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    a.record()
    for _ in range(reps):
        one()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    for r in raws:
        dev.free(r)
    nbytes = sum(algo_bytes(m["gt"], m["rows"], m["cols"]) for m in mats)
    return {"value": round(nbytes / (ms * 1e-3) / 1e9, 2), "unit": UNIT, "ms_per_step": round(ms, 4),
            "what": "reference src/ai/cuda_ops.cu cuda_matmul_q4_0/q4_k built for sm_100a, raw GGUF blocks, fp32 x"}


def cpu_baseline(mats, bytes_step, budget_s):
    sys.path.insert(0, str(ROOT / "oracle"))
    import holo_oracle
    try:
        ref = holo_oracle.Reference()
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}
    threads = os.cpu_count() or 1
    n, t0 = 0, time.perf_counter()
    while True:
        for m in mats:
            ref.matmul_q(m["gt"], m["W"], m["x"], m["rows"], m["cols"], threads=threads)
        n += 1
        if time.perf_counter() - t0 >= budget_s or n >= 50:
            break
    dt = time.perf_counter() - t0
    return {"value": round(bytes_step * n / dt / 1e9, 3), "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"{n} full sweeps (16 matvecs each) through matmul_q on row slices, {threads} threads, {dt:.1f} s"}


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU matvec on the host cores
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import holo_oracle
    try:
        ref = holo_oracle.Reference()
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU library not built: {e}"}))
        return
    threads = os.cpu_count() or 1
    specs = sweep_specs()
    mats = []
    for gt, r, c, s in specs:
        mats.append(dict(gt=gt, rows=r, cols=c, W=synth.quant_matrix(gt, r, c, s), x=synth.activation(c, s)))

    def step(frac):
        nb = 0
        for m in mats:
            rr = max(32, int(m["rows"] * frac))
            rb = hb.row_bytes(m["gt"], m["cols"])
            ref.matmul_q(m["gt"], m["W"][: rr * rb], m["x"], rr, m["cols"], threads=threads)
            nb += algo_bytes(m["gt"], rr, m["cols"])
        return nb

    # size each step so that warmup + steps take about a minute
    t0 = time.perf_counter()
    step(0.05)
    per_full = (time.perf_counter() - t0) / 0.05
    frac = min(1.0, max(0.01, 60.0 / max(1, args.steps + args.warmup) / max(per_full, 1e-6)))
    for _ in range(args.warmup):
        step(frac)
    t0 = time.perf_counter()
    nb = 0
    for _ in range(args.steps):
        nb += step(frac)
    dt = time.perf_counter() - t0
    value = nb / dt / 1e9
    sample = f"{frac:.3f} of the rows of each of the 16 matvecs per step, matmul_q on row slices, {threads} threads"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded GGUF blocks with the BASELINE config distributions)",
        "config": config(args, world),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_profile_case(args):
    """Small case for ncu: one matvec shape, a few plain launches, no graph."""
    name, shape = args.profile_case.split(":")
    gt = {"q8_0": hb.Q8_0, "q4_0": hb.Q4_0, "q4_k": hb.Q4_K}[name]
    rows, cols = (int(v) for v in shape.split("x"))
    dev = hb.Device(0, 1)
    W = synth.quant_matrix(gt, rows, cols, 0)
    x = synth.activation(cols, 0)
    Wd, xd, yd = dev.upload_quant(W, gt, rows, cols), dev.upload(x), dev.alloc(4 * rows)
    act = hb.ACT_Q8 if args.act == "q8" else hb.ACT_F32
    for _ in range(args.iters):
        dev.lib.cuda_matvec(yd, Wd, xd, rows, cols, gt, act, None)
    dev.sync()
    dev.check("profile case")
    print(json.dumps({"profile_case": args.profile_case, "act": args.act, "iters": args.iters,
                      "algorithmic_bytes_per_launch": algo_bytes(gt, rows, cols)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--act", choices=["q8", "f32"], default="q8")
    ap.add_argument("--cpu-budget", type=float, default=8.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--profile-case", default=None, help="e.g. q4_k:11008x4096 (ncu small case)")
    ap.add_argument("--iters", type=int, default=4)
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args)
        return
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
