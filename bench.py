"""Benchmark of the batch backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload lr|gemv] [--impl ours|reference]

Workloads (synthetic seeded inputs of the stated shapes):
  lr    config 1: latent_reasoner int8 (RTN, --min-size 1), 1,048,576 rows of f32[8]
        with Bernoulli(0.5) entries (seed 1) per GPU; unit rows/s.
  gemv  config 2: int4 dequant GEMV, W [4096, 4096] codes uniform in [-8, 7],
        x f32 [4096] ~ N(0,1) (seed 2); unit GB/s of algorithmic bytes.

A step is one pass of the hot path over the whole per-GPU input. value is the
whole-job throughput with inputs resident in HBM (CUDA events on the launching
stream, max over ranks); e2e is the same metric through the C ABI with host
buffers, the copies inside the timed region. Under torchrun each rank runs the
same per-GPU workload (weak scaling, no collective on the data path).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # 74.4: 148 SMs x 128 FP32 lanes x FMA x 1965 MHz


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, gpu: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def flush_l2(buf) -> None:
    buf.add_(1.0)  # 256 MB write: larger than the 126 MB L2


# ---- config 1: latent_reasoner ----------------------------------------------------------------
LR_ROWS = 1 << 20


def lr_inputs(rows: int) -> np.ndarray:
    return np.random.default_rng(1).integers(0, 2, size=(rows, 8)).astype(np.float32)


def lr_flops(steps: np.ndarray) -> float:
    # per row: embed 2*16*8, per think step 2 matvecs 2*2*16*16 + adds/tanh/delta 64, readout + norms ~180
    return float(steps.shape[0] * (256 + 180) + 1088.0 * steps.sum())


def bench_lr(args, world, rank, local):
    import torch

    from technograd_b200 import _lib, tgir
    from technograd_b200.batch import Batch
    model = os.path.join(ROOT, "tests", "golden", "latent_reasoner.q8.tgir")
    m = tgir.load(model)
    rows = lr_inputs(LR_ROWS)
    _lib.init(0, [local])
    b = Batch(m)
    L = _lib.lib()
    d_in = torch.from_numpy(rows).cuda()
    d_out = torch.empty((LR_ROWS, 4), device="cuda")
    d_steps = torch.empty((LR_ROWS, 1), dtype=torch.int32, device="cuda")
    flush = torch.empty(64 << 20, device="cuda")
    stream = torch.cuda.current_stream()

    def step():
        _lib.check(L.tg_cuda_batch_device(b.handle, d_in.data_ptr(), LR_ROWS, d_out.data_ptr(), d_steps.data_ptr(),
                                          C.c_void_p(stream.cuda_stream)))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    clk = Clocks(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush_l2(flush)
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clocks = clk.stop()
    ms = [a.elapsed_time(z) for a, z in ev]
    t = max_over_ranks(sum(ms) / 1e3, world)
    steps_np = d_steps.cpu().numpy()
    value = world * LR_ROWS * args.steps / t
    flops = lr_flops(steps_np)
    achieved = flops / (t / args.steps) / 1e12
    # e2e: host buffers through tg_cuda_batch (H2D + kernel + D2H per step)
    out_h = np.empty((LR_ROWS, 4), np.float32)
    st_h = np.empty((LR_ROWS, 1), np.int32)
    for _ in range(2):
        _lib.check(L.tg_cuda_batch(b.handle, rows.ctypes.data, LR_ROWS, 8, out_h.ctypes.data, 4, st_h.ctypes.data, 1))
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _lib.check(L.tg_cuda_batch(b.handle, rows.ctypes.data, LR_ROWS, 8, out_h.ctypes.data, 4, st_h.ctypes.data, 1))
    te = max_over_ranks(time.perf_counter() - t0, world)
    e2e = {"value": world * LR_ROWS * args.steps / te, "unit": "rows/s", "h2d_bytes_per_step": rows.nbytes,
           "d2h_bytes_per_step": out_h.nbytes + st_h.nbytes}
    line = {
        "metric": "latent_reasoner int8 batch rows/s (config 1)", "value": value, "unit": "rows/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sum(ms) / len(ms),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config1 latent_reasoner int8 RTN --min-size 1", "rows_per_gpu": LR_ROWS,
                   "think_steps_mean": float(steps_np.mean()), "l2": "flushed between steps (256 MB write)"},
        "roofline": {"bound": "fp32", "achieved": achieved, "peak": FP32_NOMINAL_TFLOPS, "unit": "TFLOP/s",
                     "frac": achieved / FP32_NOMINAL_TFLOPS, "traffic": None,
                     "peak_source": "nominal FP32 SIMT (148 SMs x 128 lanes x FMA x 1965 MHz); not in MEASURED_PEAKS"},
        "e2e": e2e, "gpu_launches": args.steps, "clocks": clocks,
    }
    return line, m, rows


def cpu_baseline_lr(rows: np.ndarray, sample: int = LR_ROWS):
    """The reference's own `tgc batch -j auto` (oracle/_ref/tgc, compiled from its sources) on the host cores."""
    from oracle import tgo
    tgc = tgo.REF_TGC
    if not os.path.exists(tgc):
        return None
    model = os.path.join(ROOT, "tests", "golden", "latent_reasoner.q8.tgir")
    with tempfile.TemporaryDirectory() as d:
        inp = os.path.join(d, "rows.bin")
        rows[:sample].astype("<f4").tofile(inp)
        r = subprocess.run([tgc, "batch", model, inp, "-j", "auto", "-v", "-o", os.path.join(d, "out.bin")],
                           capture_output=True, text=True, check=True)
    mt = re.search(r"\[batch\] (\d+) row\(s\) in ([0-9.]+) ms .* on (\d+) thread", r.stderr)
    n, ms, th = int(mt.group(1)), float(mt.group(2)), int(mt.group(3))
    return {"value": n / (ms / 1e3), "unit": "rows/s", "cores": th, "kind": "reference",
            "sample": f"{n} rows of config 1, `tgc batch -j auto` binary I/O, [batch] event time"}


def reference_arm(args, world, rank):
    if rank != 0:
        return None
    rows = lr_inputs(LR_ROWS)
    vals = []
    base = None
    for _ in range(args.warmup):
        cpu_baseline_lr(rows)
    for _ in range(args.steps):
        base = cpu_baseline_lr(rows)
        if base is None:
            break
        vals.append(base["value"])
    if base is None:
        return {"impl": "reference", "unavailable": "oracle/_ref/tgc was not built (needs the reference sources)"}
    v = statistics.median(vals)
    base["value"] = v
    return {"impl": "reference", "metric": "latent_reasoner int8 batch rows/s (config 1)", "value": v,
            "unit": "rows/s", "n_gpus": 0, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1 latent_reasoner int8 RTN --min-size 1", "rows_per_gpu": LR_ROWS},
            "cpu_baseline": base, "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="lr")
    ap.add_argument("--impl", default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        line = reference_arm(args, world, rank)
        if rank == 0 and line:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    line, m, rows = bench_lr(args, world, rank, local)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_lr(rows)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
