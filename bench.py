#!/usr/bin/env python3
"""Benchmark of the B200 decode-path library (one JSON line on rank 0).

Workload: the quantized matvec sweep over the
Llama-7B FFN shapes -- Q4_0 and Q4_K, 11008x4096 (up/gate) and 4096x11008
(down), seeds 0-3: 16 distinct matrices, 406 MB of GGUF blocks per pass, so
every pass streams more than the 126 MB L2 and no matrix is re-read from L2.
One step = one pass of the 16 matvecs: the 16 independent matvecs in one
cuda_matvec_batch call (one persistent launch per weight type), replayed as
a CUDA graph; the same pass as 16 separate cuda_matvec calls is reported
beside it (per_call_chain).

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

    import ctypes as C
    n_m = len(mats)
    b_dst = (C.c_void_p * n_m)(*[m["yd"] for m in mats])
    b_w = (C.c_void_p * n_m)(*[m["Wd"] for m in mats])
    b_x = (C.c_void_p * n_m)(*[m["xd"] for m in mats])

    def enqueue(act, batched):
        if batched:   # the 16 independent matvecs in one cuda_matvec_batch call (a launch per type)
            lib.cuda_matvec_batch(n_m, b_dst, b_w, b_x, act)
        else:         # one cuda_matvec call a matrix
            for m in mats:
                lib.cuda_matvec(m["yd"], m["Wd"], m["xd"], m["rows"], m["cols"], m["gt"], act, None)

    def capture(act, batched=True):
        enqueue(act, batched)   # one-time set-up outside capture
        dev.sync()
        if lib.cuda_capture_begin() != 0:
            dev.check("capture")
        enqueue(act, batched)
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
    # the same sweep as 16 dependent-order calls (one cuda_matvec a matrix,
    # PDL between them): what a caller issuing one matvec at a time gets
    g_chain = capture(primary, batched=False)
    chain_steps = max(1, args.steps // 4)
    ms_chain = timed(g_chain, chain_steps, max(3, args.warmup // 2)) / chain_steps
    lib.cuda_graph_free(g_chain)

    # Roofline of the dominant kernel (the batched matvec, one launch per
    # weight type: Q4_0 and Q4_K, 8 matrices each): its average launch
    # duration over the timed region = the timed region's device time /
    # launches (CUDA events on the library stream); beside it, the duration
    # of an isolated call (event pair around one cuda_matvec_batch, nothing
    # to overlap with).
    launches_per_step = len({m["gt"] for m in mats})
    region_us_per_launch = 1e3 * ms_step / launches_per_step
    kt = []
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        enqueue(primary, True)
        b.record(stream)
        kt.append((a, b))
    torch.cuda.synchronize()
    k_ms = [a.elapsed_time(b) for a, b in kt]
    peak, peak_kind = peaks()
    isolated_gbs = bytes_step / (statistics.median(k_ms) * 1e-3) / 1e9
    kernel_gbs = (bytes_step / launches_per_step) / (region_us_per_launch * 1e-6) / 1e9

    # End to end through the C ABI, host buffers in and out, every step: the
    # 16 activations from pinned host memory (one cuda_memcpy_h2d_stream), the
    # 16 matvecs (cuda_matmul_q4_0 / cuda_matmul_q4_k), the 16 results back to
    # pinned host memory (one cuda_memcpy_d2h_stream) -- enqueued once into a
    # CUDA graph with cuda_capture_begin/end -- then cuda_graph_launch and
    # cuda_sync() to wait for the host results.  Wall clock, max over ranks.
    lib.cuda_set_act_mode(primary)
    fn = {hb.Q4_0: lib.cuda_matmul_q4_0, hb.Q4_K: lib.cuda_matmul_q4_k}
    h2d = sum(4 * m["cols"] for m in mats)
    d2h = sum(4 * m["rows"] for m in mats)
    hx_all = torch.from_numpy(np.concatenate([m["x"] for m in mats])).pin_memory()
    hy_all = torch.zeros(d2h // 4, dtype=torch.float32).pin_memory()
    dx_all, dy_all = dev.alloc(h2d), dev.alloc(d2h)
    offs_x, offs_y, ox, oy = [], [], 0, 0
    for m in mats:
        offs_x.append(ox)
        offs_y.append(oy)
        ox += 4 * m["cols"]
        oy += 4 * m["rows"]

    e_dst = (C.c_void_p * n_m)(*[dy_all + yo for yo in offs_y])
    e_x = (C.c_void_p * n_m)(*[dx_all + xo for xo in offs_x])

    def e2e_enqueue():
        lib.cuda_memcpy_h2d_stream(dx_all, hx_all.data_ptr(), h2d)
        lib.cuda_matvec_batch(n_m, e_dst, b_w, e_x, primary)
        lib.cuda_memcpy_d2h_stream(hy_all.data_ptr(), dy_all, d2h)

    e2e_enqueue()
    lib.cuda_sync()
    if lib.cuda_capture_begin() != 0:
        dev.check("e2e capture")
    e2e_enqueue()
    g_e2e = lib.cuda_capture_end()
    dev.check("e2e capture end")
    e2e_steps = max(3, min(args.steps, 2000))

    def e2e_run(n):
        for _ in range(n):
            lib.cuda_graph_launch(g_e2e)
            lib.cuda_sync()

    e2e_run(3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_run(e2e_steps)
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())
    dev.check("e2e")
    e2e_value = world * bytes_step * e2e_steps / e2e_s / 1e9
    # the host results equal the device-timed graph's outputs
    e2e_same = all(np.array_equal(hy_all.numpy()[yo // 4: yo // 4 + m["rows"]], dev.download(m["yd"], (m["rows"],),
                                                                                            np.float32))
                   for m, yo in zip(mats, offs_y))

    # the same through the reference's own call pattern: per matvec a
    # synchronous cuda_memcpy_h2d, cuda_matmul_*, synchronous cuda_memcpy_d2h
    def sync_calls_step():
        for m, xo, yo in zip(mats, offs_x, offs_y):
            lib.cuda_memcpy_h2d(m["xd"], hx_all.data_ptr() + xo, 4 * m["cols"])
            fn[m["gt"]](m["yd"], m["Wd"], m["xd"], m["rows"], m["cols"])
            lib.cuda_memcpy_d2h(hy_all.data_ptr() + yo, m["yd"], 4 * m["rows"])

    sync_steps = max(3, min(args.steps, 200))
    for _ in range(3):
        sync_calls_step()
    t0 = time.perf_counter()
    for _ in range(sync_steps):
        sync_calls_step()
    sync_s = time.perf_counter() - t0
    t = torch.tensor([sync_s], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    sync_value = world * bytes_step * sync_steps / float(t.item()) / 1e9
    lib.cuda_graph_free(g_e2e)
    dev.free(dx_all)
    dev.free(dy_all)
    lib.cuda_set_act_mode(hb.ACT_Q8)

    # the reference's own CUDA kernels (src/ai/cuda_ops.cu built for sm_100a) on
    # raw blocks: the GPU kernels this library replaces
    # Single-GPU sub-benchmarks (the reference's kernels, prefill, other weight
    # types) run at N = 1 only: they are per-GPU figures, and at N > 1 rank 0
    # alone would run them while the other ranks wait to tear down.
    single = rank == 0 and world == 1
    ref_gpu = None
    if single and not args.no_ref_gpu:
        ref_gpu = ref_gpu_kernels(mats, dev, torch)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(mats, bytes_step, budget_s=args.cpu_budget)

    decode = decode70 = decode70_b8 = None
    if not args.no_decode:
        decode = decode_bench(args, world, rank, torch)
    if not args.no_decode and not args.no_70b:
        # the 70B Q4_0 model, row-sharded over the N GPUs
        # at batch 1 (every N), and batch 8 on one GPU (N = 1 only)
        a70 = argparse.Namespace(**dict(vars(args), decode_model="70b", decode_batch=1))
        decode70 = decode_bench(a70, world, rank, torch)
        if world == 1:
            decode70_b8 = decode_bench(argparse.Namespace(**dict(vars(a70), decode_batch=8)), world, rank, torch)
    prefill = prefill_bench(dev, torch) if single and not args.no_prefill else None
    other_types = other_types_bench(dev, torch) if single and not args.no_prefill else None
    c1 = c1_q8_0_bench(dev, torch) if single and not args.no_prefill else None

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
                     "traffic_source": ("static: ncu dram__bytes of one isolated launch of the same kernel on the "
                                        "same 8-matrix group (profiles/matvec_traffic.txt), not measured in this "
                                        "run") if traffic else None,
                     "algorithmic_bytes_per_launch": round(bytes_step / launches_per_step),
                     "kernel": "mv_multi_kernel (cuda_matvec_batch), one launch per weight type",
                     "kernel_avg_us": round(region_us_per_launch, 3),
                     "isolated_call": {"us": round(1e3 * statistics.median(k_ms), 3), "launches": launches_per_step,
                                       "achieved": round(isolated_gbs, 1), "frac": round(isolated_gbs / peak, 4)},
                     "step_frac": round(value / world / peak, 4)},
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "host_results_equal_device": bool(e2e_same),
                "path": "C ABI, pinned host buffers: cuda_memcpy_h2d_stream (16 x) + cuda_matvec_batch (16 matvecs) + "
                        "cuda_memcpy_d2h_stream (16 y) in one CUDA graph (cuda_capture_begin/end), "
                        "cuda_graph_launch + cuda_sync per step, wall clock",
                "per_call_sync": {"value": round(sync_value, 3), "unit": UNIT, "steps": sync_steps,
                                  "path": "per matvec: cuda_memcpy_h2d + cuda_matmul_q4_* + cuda_memcpy_d2h "
                                          "(the reference's synchronous call pattern)"}},
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clocks,
        "other_act_mode": {"act": other, "value": round(world * bytes_step / (ms_other * 1e-3) / 1e9, 2),
                           "ms_per_step": round(ms_other, 5)},
        "per_call_chain": {"value": round(world * bytes_step / (ms_chain * 1e-3) / 1e9, 2), "unit": UNIT,
                           "ms_per_step": round(ms_chain, 5), "us_per_matvec": round(1e3 * ms_chain / len(mats), 3),
                           "path": "16 cuda_matvec calls a step (one launch a matrix, PDL), CUDA graph"},
    }
    if decode:
        line["decode"] = decode
    if decode70:
        line["decode_70b"] = decode70
    if decode70_b8:
        line["decode_70b_batch8"] = decode70_b8
    if prefill:
        line["prefill"] = prefill
    if other_types is not None:
        line["other_types"] = other_types
    if c1 is not None:
        line["c1_q8_0"] = c1
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
# batch-1 decode of the Llama-2-7B-shape Q4_K model
# ---------------------------------------------------------------------------
DECODE_PROMPT, DECODE_NEW = 128, 256


def decode_bytes_per_token(cfg, n_prompt=DECODE_PROMPT, n_new=DECODE_NEW, kv_bytes=2):
    """Algorithmic HBM bytes per generated token: every layer matrix and the
    output matrix in GGUF packing, one embedding row, and the K and V rows of
    every cached position (mean over the decode positions)."""
    dim, ffn, V = cfg["dim"], cfg["ffn_dim"], cfg["vocab"]
    q_dim, kv_dim = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    lt = cfg["layer_type"]
    layer = (hb.row_bytes(lt, dim) * (q_dim + 2 * kv_dim + 2 * ffn) + hb.row_bytes(lt, q_dim) * dim
             + hb.row_bytes(lt, ffn) * dim)
    weights = cfg["n_layers"] * layer + hb.row_bytes(cfg["out_type"], dim) * V + dim * 2
    mean_kv_len = n_prompt + (n_new - 1) / 2.0
    kv = cfg["n_layers"] * 2 * mean_kv_len * kv_dim * kv_bytes
    return weights + kv, weights


# decode workloads: BASELINE configs[3] (7B, Q4_K) and configs[4] (70B, Q4_0,
# batch 1): model, prompt tokens, new tokens, timed runs
# the one-GPU greedy stream of the 7B decode model (tests/golden/make_greedy64_7b.py)
GREEDY64_FIXTURE = ROOT / "tests" / "golden" / "greedy64_7b_q8.json"

DECODE_MODELS = {
    "7b": ("LLAMA2_7B", 128, 256, 3,
           "Llama-2-7B shape, Q4_K layers, Q8_0 lm_head, fp16 embeddings and KV cache, ctx 2048"),
    "70b": ("LLAMA3_70B", 512, 128, 1,
            "Llama-3-70B shape (GQA 64/8), Q4_0 layers and lm_head, fp16 embeddings and KV cache, ctx 4096, batch 1"),
}


def decode_bench(args, world, rank, torch):
    """Full generation on a random-init model built on the device (T 0.8 /
    top-k 40 / top-p 0.95 / repeat penalty 1.1, fp16 KV cache): the 7B
    configuration (128-token prompt, 256 new tokens, median of 3 runs) or
    with --decode-model 70b the 70B one (512-token prompt, 128 new tokens).
    tok/s from the device time of the decode phase; e2e from the wall time of
    the public holo_model_generate call (prompt in, tokens out, prefill
    included).  With N ranks the model is row-sharded over the N GPUs (strong
    scaling: one model, one token stream); times are the maximum over the
    ranks."""
    from holo_b200 import model as hm
    from holo_b200.model import SamplerDesc, connect_peers, synthetic_model
    if args.decode_batch > 1:
        return decode_batch_bench(args, world, rank, torch)
    cfg_name, n_prompt, n_new, runs_n, desc = DECODE_MODELS[args.decode_model]
    cfg = dict(getattr(hm, cfg_name))
    act = hb.ACT_Q8 if args.act == "q8" else hb.ACT_F32
    want_cpu = rank == 0 and world == 1 and not args.no_cpu and args.decode_model == "7b"
    t0 = time.perf_counter()
    built = synthetic_model(cfg, seed=0, act_mode=act, kv_f16=True, keep_host=want_cpu, world=world, rank=rank)
    m, host = built if want_cpu else (built, None)
    if world > 1:
        connect_peers(m)
    build_s = time.perf_counter() - t0

    def max_over_ranks(*vals):
        if world == 1:
            return vals
        import torch.distributed as dist
        t = torch.tensor(vals, device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return tuple(float(v) for v in t.tolist())
    prompt = np.random.default_rng(0).integers(0, cfg["vocab"], size=n_prompt).astype(np.int32)
    s = SamplerDesc(0.8, 0.95, 40, 1.1, 64)
    m.generate(prompt, n_new, s, seed=0)            # warm-up (caches, clocks)
    runs = []
    for i in range(runs_n):
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        toks = m.generate(prompt, n_new, s, seed=i)
        wall = time.perf_counter() - w0
        pre_ms, dec_ms = m.last_timing()
        dec_ms, pre_ms, wall = max_over_ranks(dec_ms, pre_ms, wall)
        runs.append((dec_ms, pre_ms, wall, toks))
    first_tokens = runs[0][3]      # seed 0
    greedy = None
    if args.decode_model == "7b":
        # 64 greedy steps (the bench's prompt and penalty), against the
        # committed one-GPU stream: a sharded model is bit-identical to one GPU
        g64 = m.generate(prompt, 64, SamplerDesc(0.0, 0.95, 40, 1.1, 64), seed=0)
        fx = GREEDY64_FIXTURE
        want = json.loads(fx.read_text())["tokens"] if fx.exists() else None
        greedy = {"equal_1gpu": None if want is None else bool(np.array_equal(g64, np.array(want))),
                  "head": [int(t) for t in g64[:8]], "fixture": str(fx.relative_to(ROOT))}
    runs.sort(key=lambda r: r[0])
    dec_ms, pre_ms, wall, toks = runs[len(runs) // 2]
    tok_s = n_new / (dec_ms * 1e-3)
    bpt, wbytes = decode_bytes_per_token(cfg, n_prompt, n_new)
    peak, peak_kind = peaks()
    peak *= world                 # the shards stream from every GPU's HBM at once
    step_kernel = cfg["head_dim"] == 128 and os.environ.get("HOLO_STEP") != "graph"
    out = {
        "config": f"{desc}; prompt {n_prompt}, {n_new} new tokens, T 0.8 / top-k 40 / top-p 0.95 / rep 1.1"
                  + (f"; row-sharded over {world} GPUs" if world > 1 else ""),
        "model": args.decode_model, "scaling": "strong", "n_gpus": world,
        "act_mode": args.act, "value": round(tok_s, 1), "unit": "tokens/s", "ms_per_token": round(dec_ms / n_new, 4),
        "prefill_ms": round(pre_ms, 2), "prefill_tokens_s": round((n_prompt - 1) / (pre_ms * 1e-3), 1),
        "roofline": {"bound": "hbm", "bytes_per_token": int(bpt), "weight_bytes_per_token": int(wbytes),
                     "achieved": round(bpt * tok_s / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(bpt * tok_s / 1e9 / peak, 4), "peak_source": peak_kind},
        "e2e": {"value": round(n_new / wall, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * n_prompt,
                "d2h_bytes_per_step": 4 * n_new,
                "path": "holo_model_generate: prompt ids in, generated ids out, prefill included"},
        "gpu_launches_per_token": 2 if step_kernel else cfg["n_layers"] * 7 + 4,
        "runs": runs_n,
        "model_build_s": round(build_s, 1),
        "tokens_head_seed0": [int(t) for t in first_tokens[:8]],
    }
    if greedy is not None:
        out["greedy64_equal_1gpu"] = greedy["equal_1gpu"]
        out["greedy64"] = greedy
    if want_cpu and host is not None:
        out["cpu_baseline"] = decode_cpu_baseline(cfg, host, prompt, budget_s=args.cpu_budget)
    elif rank == 0 and world == 1 and not args.no_cpu:   # 70B: llm_forward is infeasible on the host
        out["cpu_baseline"] = decode_cpu_extrapolated(cfg, budget_s=args.cpu_budget)
    m.close()
    return out


PREFILL_SHAPES = [(14336, 4096), (4096, 14336)]
PREFILL_M = [64, 256, 512]


def c1_q8_0_bench(dev, torch, iters=20):
    """BASELINE configs[0]'s shape on the GPU: Q8_0 4096x4096 matvecs (16
    distinct matrices, 285 MB, larger than L2), Q8 activations: the batched
    call, one cuda_matvec_q8_0-style call a matrix in a graph, one isolated
    call, and the reference's own cuda_matmul_q8_0 (src/ai/cuda_ops.cu built
    for sm_100a) on the raw blocks.  GB/s of algorithmic bytes
    (17,858,560 a matvec)."""
    import ctypes as C
    lib = dev.lib
    stream = torch.cuda.ExternalStream(lib.cuda_get_stream())
    hbm, _ = peaks()
    n, r, c = 16, 4096, 4096
    Ws = [synth.quant_matrix(hb.Q8_0, r, c, s) for s in range(n)]
    mats = [dict(W=W, Wd=dev.upload_quant(W, hb.Q8_0, r, c), xd=dev.upload(synth.activation(c, s)),
                 yd=dev.alloc(4 * r)) for s, W in enumerate(Ws)]
    nbytes = algo_bytes(hb.Q8_0, r, c)
    dst = (C.c_void_p * n)(*[m["yd"] for m in mats])
    Mp = (C.c_void_p * n)(*[m["Wd"] for m in mats])
    xp = (C.c_void_p * n)(*[m["xd"] for m in mats])

    def graph(fn):
        fn()
        dev.sync()
        lib.cuda_capture_begin()
        fn()
        return lib.cuda_capture_end()

    def gtime(g, reps):
        for _ in range(3):
            lib.cuda_graph_launch(g)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            lib.cuda_graph_launch(g)
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    out = {"shape": "4096x4096 Q8_0 (BASELINE configs[0]), 16 distinct matrices, Q8 activations"}
    g = graph(lambda: lib.cuda_matvec_batch(n, dst, Mp, xp, hb.ACT_Q8))
    ms = gtime(g, iters)
    lib.cuda_graph_free(g)
    out["batch"] = {"gbs": round(n * nbytes / (ms * 1e-3) / 1e9, 1), "hbm_frac": round(n * nbytes / (ms * 1e-3) / 1e9 / hbm, 4),
                    "us_per_matvec": round(1e3 * ms / n, 3)}
    g = graph(lambda: [lib.cuda_matvec(m["yd"], m["Wd"], m["xd"], r, c, hb.Q8_0, hb.ACT_Q8, None) for m in mats])
    ms = gtime(g, iters)
    lib.cuda_graph_free(g)
    out["per_call_chain"] = {"gbs": round(n * nbytes / (ms * 1e-3) / 1e9, 1), "us_per_matvec": round(1e3 * ms / n, 3)}
    ts = []
    for m in mats[:8]:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        lib.cuda_matvec(m["yd"], m["Wd"], m["xd"], r, c, hb.Q8_0, hb.ACT_Q8, None)
        b.record(stream)
        ts.append((a, b))
    torch.cuda.synchronize()
    us = 1e3 * statistics.median([a.elapsed_time(b) for a, b in ts])
    out["isolated_call"] = {"us": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
    so = ROOT / "oracle" / "_ref" / "libholo_ref_cuda.so"
    if so.exists():
        ref = C.CDLL(str(so))
        ref.cuda_matmul_q8_0.argtypes = [C.c_void_p] * 3 + [C.c_int, C.c_int]
        raws = [dev.upload(m["W"]) for m in mats]
        dev.sync()
        for _ in range(2):
            for m, raw in zip(mats, raws):
                ref.cuda_matmul_q8_0(m["yd"], raw, m["xd"], r, c)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            for m, raw in zip(mats, raws):
                ref.cuda_matmul_q8_0(m["yd"], raw, m["xd"], r, c)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / 5
        out["reference_gpu_kernel"] = {"gbs": round(n * nbytes / (ms * 1e-3) / 1e9, 1),
                                       "what": "reference cuda_matmul_q8_0 (src/ai/cuda_ops.cu:1132-1155) for sm_100a"}
        for raw in raws:
            dev.free(raw)
    dev.check("c1 q8_0")
    for m in mats:
        for k in ("Wd", "xd", "yd"):
            dev.free(m[k])
    return out


def other_types_bench(dev, torch, iters=10):
    """Q6_K and F16 matvecs (the types real Q4_K_M files keep for some
    tensors): the tiled path (cuda_upload_quant, unit layout) against the raw
    GGUF path (cuda_malloc + cuda_memcpy_h2d of the blocks, as the reference's
    upload_tensor does), both through the reference entry points
    (cuda_matmul_q6_k / cuda_matmul_f16), fp32 activations.  Device time from
    CUDA events on the library stream over `iters` rotations of distinct
    matrices larger than L2 together; GB/s of GGUF weight bytes."""
    lib = dev.lib
    stream = torch.cuda.ExternalStream(lib.cuda_get_stream())
    hbm, _ = peaks()
    cases = [(hb.Q6_K, 4096, 11008, 4), (hb.Q6_K, 11008, 4096, 4), (hb.F16, 4096, 11008, 2)]
    out = []
    for gt, r, c, n in cases:
        fn = lib.cuda_matmul_q6_k if gt == hb.Q6_K else lib.cuda_matmul_f16
        mats = []
        for s in range(n):
            W = synth.quant_matrix(gt, r, c, s) if gt == hb.Q6_K else synth.f16_matrix(r, c, s).view(np.uint8).reshape(-1)
            raw = dev.alloc(W.nbytes)
            lib.cuda_memcpy_h2d(raw, W.ctypes.data, W.nbytes)
            mats.append((dev.upload_quant(W, gt, r, c), raw))
        xd, yd = dev.upload(synth.activation(c, 0)), dev.alloc(4 * r)
        wbytes = r * hb.row_bytes(gt, c)
        res = {"type": hb.TYPE_NAMES[gt], "rows": r, "cols": c}
        for label, k in (("tiled", 0), ("raw", 1)):
            for _ in range(2):
                for m in mats:
                    fn(yd, m[k], xd, r, c)
            dev.check("other types warm-up")
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(iters):
                for m in mats:
                    fn(yd, m[k], xd, r, c)
            e1.record(stream)
            e1.synchronize()
            dev.check("other types")
            us = e0.elapsed_time(e1) * 1e3 / (iters * len(mats))
            res[label] = {"us": round(us, 2), "gbs": round(wbytes / (us * 1e-6) / 1e9, 1),
                          "hbm_frac": round(wbytes / (us * 1e-6) / 1e9 / hbm, 4)}
        out.append(res)
        for m in mats:
            dev.free(m[0])
            dev.free(m[1])
        dev.free(xd)
        dev.free(yd)
    return out


def prefill_bench(dev, torch, iters=20):
    """C3: batched Q4_K matmul (cuda_matmul_quant_batched, tcgen05) for the
    prefill shapes and token counts; device time per call from CUDA events on
    the library stream over `iters` calls after 3 warm-up calls, inputs
    resident.  Roofline: dense tensor FLOPs against the measured bf16 peak
    (the kernel multiplies fp16 operands, same peak), and the weight bytes
    against HBM."""
    lib = dev.lib
    stream = torch.cuda.ExternalStream(lib.cuda_get_stream())
    peak_tf = None
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        peak_tf = float(json.loads(p.read_text())["bf16_tflops"])
    hbm, _ = peaks()
    out = []
    for n, k in PREFILL_SHAPES:
        W = synth.quant_matrix(hb.Q4_K, n, k, 0)
        Wd = dev.upload_quant(W, hb.Q4_K, n, k)
        for m in PREFILL_M:
            X = synth.activation(m * k, 0)
            Xd, Yd = dev.upload(X), dev.alloc(4 * m * n)
            for _ in range(3):
                lib.cuda_matmul_quant_batched(Yd, Wd, Xd, m, n, k)
            dev.check("prefill warm-up")
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(iters):
                lib.cuda_matmul_quant_batched(Yd, Wd, Xd, m, n, k)
            e1.record(stream)
            e1.synchronize()
            dev.check("prefill")
            us = e0.elapsed_time(e1) * 1e3 / iters
            flops = 2.0 * m * n * k
            tf = flops / (us * 1e-6) / 1e12
            wbytes = n * hb.row_bytes(hb.Q4_K, k)
            out.append({"N": n, "K": k, "M": m, "us": round(us, 2), "tflops": round(tf, 1),
                        "tensor_frac": round(tf / peak_tf, 4) if peak_tf else None,
                        "weight_gbs": round(wbytes / (us * 1e-6) / 1e9, 1),
                        "hbm_frac": round(wbytes / (us * 1e-6) / 1e9 / hbm, 4)})
            dev.free(Xd)
            dev.free(Yd)
        dev.free(Wd)
    return {"kernel": "cuda_matmul_quant_batched (tcgen05.mma kind::f16, fp32 accumulators in TMEM)",
            "peak_tflops": peak_tf, "peak_source": "measured bf16 (burst)", "cases": out,
            "timing": f"CUDA events on the library stream, {iters} calls after 3 warm-up, includes the "
                      "activation quantize/tile kernel and any K-split reduction"}


def decode_batch_bench(args, world, rank, torch):
    """Batched decode (BASELINE configs[4] batch 8 with --decode-model 70b):
    args.decode_batch independent prompts decoded together on one GPU
    (holo_model_generate_batch: each projection one tensor-core matmul with
    M = batch).  Under torchrun every rank runs its own batch (data-parallel
    replicas, weak scaling); value = all ranks' generated tokens / the slowest
    rank's decode time."""
    from holo_b200 import model as hm
    from holo_b200.model import SamplerDesc, synthetic_model
    cfg_name, n_prompt, n_new, _, desc = DECODE_MODELS[args.decode_model]
    cfg = dict(getattr(hm, cfg_name))
    B = args.decode_batch
    t0 = time.perf_counter()
    m = synthetic_model(cfg, seed=0, kv_f16=True, batch=B)
    build_s = time.perf_counter() - t0
    prompts = np.random.default_rng(rank).integers(0, cfg["vocab"], size=(B, n_prompt)).astype(np.int32)
    s = SamplerDesc(0.8, 0.95, 40, 1.1, 64)
    seeds = np.arange(B, dtype=np.int32) + 100 * rank
    m.generate_batch(prompts, n_new, s, seeds)            # warm-up (graph capture, caches)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    toks = m.generate_batch(prompts, n_new, s, seeds)
    wall = time.perf_counter() - w0
    pre_ms, dec_ms = m.last_timing()
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([dec_ms, pre_ms, wall], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dec_ms, pre_ms, wall = (float(v) for v in t.tolist())
    tok_s = world * B * n_new / (dec_ms * 1e-3)
    bpt, wbytes = decode_bytes_per_token(cfg, n_prompt, n_new)
    step_bytes = wbytes + B * (bpt - wbytes)          # weights once, the KV rows of every sequence
    peak, peak_kind = peaks()
    step_s = dec_ms * 1e-3 / n_new
    out = {
        "config": f"{desc}; batch {B}, prompt {n_prompt}, {n_new} new tokens a sequence, "
                  "T 0.8 / top-k 40 / top-p 0.95 / rep 1.1" + (f"; {world} data-parallel replicas" if world > 1 else ""),
        "model": args.decode_model, "batch": B, "scaling": "weak" if world > 1 else "n/a", "n_gpus": world,
        "value": round(tok_s, 1), "unit": "tokens/s (all sequences)", "ms_per_step": round(step_s * 1e3, 3),
        "prefill_ms": round(pre_ms, 1),
        "roofline": {"bound": "hbm", "bytes_per_step": int(step_bytes),
                     "achieved": round(step_bytes / step_s / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(step_bytes / step_s / 1e9 / peak, 4), "peak_source": peak_kind},
        "e2e": {"value": round(world * B * n_new / wall, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * B * n_prompt,
                "d2h_bytes_per_step": 4 * B * n_new, "path": "holo_model_generate_batch, prefill included"},
        "model_build_s": round(build_s, 1),
        "tokens_head_seq0": [int(t) for t in toks[0][:8]],
    }
    m.close()
    return out


def decode_cpu_baseline(cfg, host, prompt, budget_s):
    """The reference's llm_forward (src/ai/llm.c:1015) on the host cores with the
    same weights: seconds per token over a bounded sample of positions."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import holo_oracle
    try:
        ref = holo_oracle.Reference()
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}
    rm = holo_oracle.RefModel(ref, cfg, host)
    n, t0 = 0, time.perf_counter()
    for t in prompt:
        rm.forward(int(t))
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    rm.close()
    threads = os.cpu_count() or 1
    return {"value": round(n / dt, 4), "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"llm_forward for the first {n} prompt positions of the same model, {dt:.1f} s "
                      f"(Q4_K matvecs single-threaded as in the reference; OpenMP up to {threads} threads elsewhere)"}


def decode_cpu_extrapolated(cfg, budget_s, sample_rows=4096):
    """The reference's matmul_q (src/ai/llm.c:770-926) on the host cores over
    row samples (up to sample_rows rows, tens of MB: larger than the CPU's
    caches) of a model's seven per-layer matrix shapes and its output matrix,
    scaled to whole matrices and n_layers layers: tokens per second of the
    matvecs alone.  llm_forward end to end is infeasible at 70B (about a
    minute a token); attention and the elementwise work are left out, so the
    figure flatters the CPU.  matmul_q runs with its own threading (OpenMP for
    Q8_0/F32, one thread for Q4_0/Q4_K)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import holo_oracle
    try:
        ref = holo_oracle.Reference()
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}
    dim, ffn = cfg["dim"], cfg["ffn_dim"]
    q_dim, kv_dim = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    lt, ot = cfg["layer_type"], cfg["out_type"]
    shapes = [(lt, q_dim, dim), (lt, kv_dim, dim), (lt, kv_dim, dim), (lt, dim, q_dim), (lt, ffn, dim),
              (lt, ffn, dim), (lt, dim, ffn), (ot, cfg["vocab"], dim)]
    per_shape = budget_s / len(shapes)
    layer_s = out_s = 0.0
    for i, (gt, rows, cols) in enumerate(shapes):
        r = min(rows, sample_rows)
        W = synth.quant_matrix(gt, r, cols, seed=900 + i)
        x = synth.activation(cols, seed=900 + i)
        n, t0 = 0, time.perf_counter()
        while True:
            ref.matmul_q(gt, W, x, r, cols)
            n += 1
            if time.perf_counter() - t0 >= per_shape:
                break
        full = (time.perf_counter() - t0) / n * rows / r
        if i == len(shapes) - 1:
            out_s = full
        else:
            layer_s += full
    s_tok = layer_s * cfg["n_layers"] + out_s
    return {"value": round(1.0 / s_tok, 5), "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "reference",
            "sample": f"matmul_q on slices of up to {sample_rows} rows of the 7 layer shapes and the output "
                      f"matrix, scaled to whole matrices x {cfg['n_layers']} layers ({s_tok:.1f} s a token; "
                      f"matvecs only, attention left out)"}


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


def run_profile_decode(args):
    """Small decode case for ncu: the 7B model (--layers: only the first N
    layers, context 256, so a capture holds well under a GB), 2 prompt + 2 new
    tokens; the profiled generate is inside the NVTX range "profiled"."""
    import torch
    from holo_b200.model import LLAMA2_7B, SamplerDesc, synthetic_model
    dev = hb.Device(0, 1)
    cfg = dict(LLAMA2_7B)
    if args.layers:
        cfg.update(n_layers=args.layers, max_seq=256)
    m = synthetic_model(cfg, seed=0, act_mode=hb.ACT_Q8 if args.act == "q8" else hb.ACT_F32)
    s = SamplerDesc(0.8, 0.95, 40, 1.1, 64)
    p = np.array([1, 2], np.int32)
    m.generate(p, 2, s, seed=0)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("profiled")
    m.generate(p, 2, s, seed=0)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    dev.check("profile decode")
    print(json.dumps({"profile_decode": "llama2-7b q4_k", "layers": cfg["n_layers"], "steps": 3,
                      "kernels_per_step": 2}))
    m.close()


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


def run_profile_batch(args):
    """Small case for ncu: one cuda_matvec_batch call (one launch) over
    --profile-batch N distinct Q4_K 11008x4096 matrices (N = 8: 203 MB, the
    bench's per-launch group, larger than L2), --iters calls, no graph."""
    import ctypes as C
    n = args.profile_batch
    dev = hb.Device(0, 1)
    mats = []
    for s in range(n):
        W = synth.quant_matrix(hb.Q4_K, 11008, 4096, s)
        mats.append((dev.upload_quant(W, hb.Q4_K, 11008, 4096), dev.upload(synth.activation(4096, s)),
                     dev.alloc(4 * 11008)))
    dst = (C.c_void_p * n)(*[m[2] for m in mats])
    M = (C.c_void_p * n)(*[m[0] for m in mats])
    v = (C.c_void_p * n)(*[m[1] for m in mats])
    act = hb.ACT_Q8 if args.act == "q8" else hb.ACT_F32
    for _ in range(args.iters):
        dev.lib.cuda_matvec_batch(n, dst, M, v, act)
    dev.sync()
    dev.check("profile batch")
    print(json.dumps({"profile_batch": n, "act": args.act, "iters": args.iters,
                      "algorithmic_bytes_per_launch": n * algo_bytes(hb.Q4_K, 11008, 4096)}))


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
    ap.add_argument("--no-decode", action="store_true", help="skip the decode sub-benchmarks")
    ap.add_argument("--no-70b", action="store_true", help="skip the 70B decode sub-benchmarks")
    ap.add_argument("--profile-decode", action="store_true", help="small 7B decode case for ncu")
    ap.add_argument("--decode-only", action="store_true", help="only the decode sub-benchmark")
    ap.add_argument("--decode-model", choices=["7b", "70b"], default="7b", help="decode sub-benchmark model")
    ap.add_argument("--decode-batch", type=int, default=1,
                    help="sequences decoded together (batched engine; under torchrun: one batch per rank)")
    ap.add_argument("--layers", type=int, default=0, help="--profile-decode: first N layers only")
    ap.add_argument("--profile-prompt", type=int, default=0,
                    help="7B prompt passes of N positions (holo_model_prefill), --iters times, for ncu")
    ap.add_argument("--no-prefill", action="store_true", help="skip the tcgen05 prefill sub-benchmark")
    ap.add_argument("--prefill-only", action="store_true", help="only the prefill sub-benchmark")
    ap.add_argument("--profile-prefill", default=None,
                    help="e.g. 512:14336x4096 or 8:57344x8192:q4_0 (ncu case: M:NxK[:type], Q4_K by default)")
    ap.add_argument("--profile-case", default=None, help="e.g. q4_k:11008x4096 (ncu small case)")
    ap.add_argument("--profile-batch", type=int, default=0,
                    help="one cuda_matvec_batch over N Q4_K 11008x4096 matrices, --iters times (ncu case)")
    ap.add_argument("--iters", type=int, default=4)
    args = ap.parse_args()
    if args.profile_decode:
        run_profile_decode(args)
        return
    if args.profile_case:
        run_profile_case(args)
        return
    if args.profile_batch:
        run_profile_batch(args)
        return
    if args.profile_prompt:
        from holo_b200 import model as hm
        from holo_b200.model import synthetic_model
        hb.Device(0, 1)
        m = synthetic_model(dict(hm.LLAMA2_7B), seed=0, kv_f16=True)
        toks = np.random.default_rng(0).integers(0, 32000, size=args.profile_prompt).astype(np.int32)
        for _ in range(args.iters):
            m.reset()
            m.prefill(toks, want_logits=False)
        m.close()
        print(json.dumps({"profile_prompt": args.profile_prompt, "iters": args.iters}))
        return
    if args.profile_prefill:
        import torch
        fields = args.profile_prefill.split(":")
        m, nk = fields[0], fields[1]
        gt = {"q4_k": hb.Q4_K, "q4_0": hb.Q4_0, "q8_0": hb.Q8_0}[fields[2] if len(fields) > 2 else "q4_k"]
        n, k = (int(v) for v in nk.split("x"))
        m = int(m)
        dev = hb.Device(0, 1)
        Wd = dev.upload_quant(synth.quant_matrix(gt, n, k, 0), gt, n, k)
        Xd, Yd = dev.upload(synth.activation(m * k, 0)), dev.alloc(4 * m * n)
        for _ in range(args.iters):
            dev.lib.cuda_matmul_quant_batched(Yd, Wd, Xd, m, n, k)
        dev.check("profile prefill")
        print(json.dumps({"profile_prefill": args.profile_prefill, "iters": args.iters,
                          "flops_per_call": 2 * m * n * k}))
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
        if args.prefill_only:
            import torch
            torch.cuda.set_device(local_rank)
            d = prefill_bench(hb.Device(local_rank, world), torch)
            if rank == 0:
                print(json.dumps({"prefill": d}), flush=True)
        elif args.decode_only:
            import torch
            torch.cuda.set_device(local_rank)
            hb.Device(local_rank, world)
            args.no_cpu = True
            d = decode_bench(args, world, rank, torch)
            if rank == 0:
                print(json.dumps({"decode": d}), flush=True)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
