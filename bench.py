"""Benchmark of the batch backend (one JSON line per workload on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload all|decode|lr|prefill|gemm|ssm] [--impl ours|reference]

With no --workload every config runs, one line each, in the order lr, gemm (M = 1, 16,
256, 4096), ssm, prefill, decode; the last line is config 5, the headline metric
BASELINE.json names. Workloads (seeded synthetic inputs of the
stated shapes):
  decode  config 5: Qwen3-0.6B architecture (28 layers, hidden 1024, 16/8 heads x 128,
          SwiGLU 3072, vocab 151936), random init N(0, 0.02), int4 GPTQ per output column
          against 256 seeded N(0,1) calibration rows per input width (the 3072-wide down
          projection RTN, as src/quant.c:346 does), greedy decode: 2048 sequences of 1024
          uniform-random ids, each continued by 257 argmax tokens (the prefill's plus 256
          decode steps over the KV cache). The 2048-sequence job is fixed: rank r of N takes
          2048/N sequences and runs them in waves of at most 512 (strong scaling); one step
          = one wave on every rank. Unit: generated tokens/s.
  lr      config 1: latent_reasoner int8 RTN (--min-size 1), 1,048,576 rows of f32[8]
          with Bernoulli(0.5) entries (seed 1) per GPU; unit rows/s.
  gemm    config 2: tg_cuda_matmul_q axis 0 (tg_matmul_qa) on W [4096, 4096] int4/int8
          codes and X^T [4096, M], --m 1,16,256,4096 (one JSON line per M), --bits 4|8;
          unit GEMMs/s, roofline HBM for M <= 16, bf16 tensor above.
  ssm     config 3: 4 selective-SSM blocks (d_model 256, d_inner 512, d_state 16, dt_rank
          16, conv 4), int8 RTN, 1024 sequences x 4096 steps of N(0,1) f32[256] (seed 3);
          unit tokens (sequence steps)/s.
  prefill config 4: the Qwen3-0.6B shape with int8 RTN weights (seed 4), 64 sequences x
          512 uniform-random ids, last-position logits; unit prompt tokens/s.

value: the device time of each step (CUDA events on the stream the library
launches on, first to last launch), summed over steps, max over ranks. e2e: the
same steps timed around the synchronous C-ABI call with host buffers (ids in,
tokens out). Under torchrun every rank runs its own shard, with no collective on
the data path.

--impl reference times the reference's own CPU implementation on the host cores (rank
0 only; other ranks exit without work) and prints config 5's line, or the --workload
given: its `tgc batch -j auto` (config 1), its tg_matmul_qa kernel (config 2), and its
VM -- load_module, quantize_param, plan, vm_run_into, compiled from its sources into
oracle/_ref -- on the config-3 program and on pieces of the config-4/5 Qwen3 forward at
the config's sequence length (oracle/refvm.py says how a forward is pieced). Nothing of
this repository's product (technograd_b200, libtgcuda) is imported on that path.
"""
from __future__ import annotations

import argparse
import ctypes as C
import faulthandler
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # 74.4: 148 SMs x 128 FP32 lanes x FMA x 1965 MHz
TOTAL_SEQS, PROMPT, NEW, WAVE = 2048, 1024, 257, 512
SMALL_SEQS = 8  # sequences per GPU of the small-wave decode line (its products: dequant GEMVs over int4 codes)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p)), "measured"
    return PEAKS_FALLBACK, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region. A timed region shorter than the 200 ms
    sampling period is bracketed by a sample taken before it (first()) and by untimed repeats
    of the same work after it (hold()), so the clocks it ran at are on record."""

    def __init__(self, gpu: int):
        self.t0 = time.perf_counter()
        self.held = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def first(self, timeout: float = 5.0) -> None:
        """Waits for the sampler's first row (nvidia-smi takes a moment to start)."""
        if self.p is None:
            return
        t = time.perf_counter()
        while time.perf_counter() - t < timeout:
            self.f.flush()
            with open(self.f.name) as g:
                if g.read().count("\n"):
                    return
            time.sleep(0.02)

    def hold(self, work, min_s: float = 1.0) -> None:
        """Repeats `work` (untimed) until the sampler has run for min_s seconds."""
        n = 0
        while time.perf_counter() - self.t0 < min_s:
            work()
            n += 1
        self.held = n

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [[x.strip() for x in r.split(",")] for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(r[1]) for r in rows) if v is not None]
        mx = [v for v in (num(r[2]) for r in rows) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
               "reasons": reasons, "samples": len(rows)}
        if self.held is not None:
            out["window"] = (f"a sample before the timed region, the region, and {self.held} untimed repeats of the "
                             "same work right after it")
        return out


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return world, rank, local



def shard_range(total: int, world: int, rank: int):
    from technograd_b200.shard import shard_range as f
    return f(total, world, rank)


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return float(x)
    from technograd_b200.shard import max_over_ranks as f
    return f(x, world)


class L2Flush:
    """Between timed calls: write a 256 MB buffer, then read another 256 MB one (both larger
    than the 126 MB L2). The read evicts the written lines, so their write-back happens here
    and not inside the next timed call, and the timed call finds no input of its own in L2."""

    NOTE = "flushed between calls: 256 MB written, then 256 MB read"

    def __init__(self):
        import torch
        self.w = torch.empty(64 << 20, device="cuda")
        self.r = torch.zeros(64 << 20, device="cuda")
        self.out = torch.empty((), device="cuda")

    def __call__(self):
        import torch
        self.w.fill_(1.0)
        torch.sum(self.r, dim=0, out=self.out)


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- the workloads as both arms name them (static: no measured values) --------------------------

METRICS = {
    "decode": ("int4 Qwen3-0.6B-shape greedy decode tokens/s (config 5)", "tokens/s"),
    "decode_small": ("int4 Qwen3-0.6B-shape greedy decode tokens/s, 8 sequences per GPU (config 5 shape, small wave)",
                     "tokens/s"),
    "prefill": ("int8 Qwen3-0.6B-shape batched prefill tokens/s (config 4)", "tokens/s"),
    "ssm": ("int8 stacked selective-SSM tokens/s (config 3)", "tokens/s"),
    "lr": ("latent_reasoner int8 batch rows/s (config 1)", "rows/s"),
}


def gemm_metric(bits: int, M: int):
    return f"int{bits} dequant GEMM [4096x4096] x [4096, M={M}] GEMMs/s (config 2)", "GEMM/s"


def workload_config(workload: str, args, M: int = 0) -> dict:
    """The line's `config`: what was run, identical in both arms for the same flags."""
    if workload == "decode":
        total, prompt, new, layers = args.seqs or TOTAL_SEQS, args.prompt or PROMPT, args.new or NEW, args.layers or 28
        full = (total, prompt, new, layers) == (TOTAL_SEQS, PROMPT, NEW, 28)
        return {"workload": "config5 int4 GPTQ Qwen3-0.6B-shape: 2048 seqs x 1024-token prompts + 256 decode steps"
                if full else f"REDUCED config5 shape (profiling): {total} seqs x {prompt} + {new - 1} steps, {layers} layers",
                "seqs": total, "prompt": prompt, "new_tokens_per_seq": new, "max_seqs_per_wave": WAVE,
                "parallelism": "sequences sharded over ranks, waves of <= 512 per GPU",
                "l2": "inputs larger than L2 (the KV cache, tens of GB, is streamed every decode step)"}
    if workload == "decode_small":
        per, prompt, new, layers = args.seqs or SMALL_SEQS, args.prompt or PROMPT, args.new or NEW, args.layers or 28
        full = (per, prompt, new, layers) == (SMALL_SEQS, PROMPT, NEW, 28)
        return {"workload": "config5 int4 GPTQ Qwen3-0.6B-shape, small wave: 8 seqs per GPU x 1024-token prompts + 256 "
                            "decode steps" if full else
                f"REDUCED config5 small wave: {per} seqs per GPU x {prompt} + {new - 1} steps, {layers} layers",
                "seqs_per_gpu": per, "prompt": prompt, "new_tokens_per_seq": new,
                "parallelism": "each rank its own sequences (one wave)",
                "l2": "inputs larger than L2 (the KV cache, up to 1.8 GB, and 0.3 GB of codes are streamed every decode step)"}
    if workload == "prefill":
        seqs, T, layers = args.seqs or PF_SEQS, args.prompt or PF_T, args.layers or 28
        return {"workload": "config4 int8 RTN Qwen3-0.6B-shape prefill: 64 seqs x 512 tokens, last-position logits"
                if (seqs, T, layers) == (PF_SEQS, PF_T, 28) else f"REDUCED config4 shape: {seqs} seqs x {T} tokens, {layers} layers",
                "seqs": seqs, "tokens_per_seq": T, "parallelism": "sequences sharded over ranks",
                "l2": "inputs larger than L2 (activations 64x512x3072 f32 and weights stream every layer)"}
    if workload == "ssm":
        seqs, T, blocks = args.seqs or SSM_SEQS, args.prompt or SSM_T, args.layers or 4
        return {"workload": "config3 4 SSM blocks d_model 256, d_inner 512, d_state 16, conv 4: 1024 seqs x 4096 steps"
                if (seqs, T, blocks) == (SSM_SEQS, SSM_T, 4) else f"REDUCED config3 shape: {seqs} seqs x {T} steps, {blocks} blocks",
                "seqs": seqs, "steps_per_seq": T, "parallelism": "sequences sharded over ranks",
                "l2": "inputs larger than L2 (4.3 GB in, 4.3 GB out per step)"}
    if workload == "lr":
        return {"workload": "config1 latent_reasoner int8 RTN --min-size 1", "rows_per_gpu": LR_ROWS,
                "parallelism": "each rank its own rows", "l2": "flushed between calls: 256 MB written, then 256 MB read"}
    if workload == "gemm":
        return {"workload": f"config2 M={M} int{args.bits}", "M": M, "N": GEMM_N, "K": GEMM_K,
                "parallelism": "replicas (each rank its own GEMM)",
                "step": "one call on each of the weight copies in turn",
                "l2": "inputs larger than L2: consecutive calls use different weight copies (together > 256 MB); the K "
                      "steps run as one CUDA graph"}
    raise ValueError(workload)


# ---- config 5: int4 GPTQ Qwen3-0.6B-shape greedy decode ----------------------------------------

def decode_ids(total: int, prompt: int) -> np.ndarray:
    return np.random.default_rng(5).integers(0, 151936, size=(total, prompt)).astype(np.float32)


def bench_decode(args, world, rank, local, small: bool = False):
    """Config 5: 2048 sequences over the ranks in waves of up to 512 per GPU; small: 8
    sequences per GPU in one wave, whose products run as dequant GEMVs over the int4 codes."""
    import torch

    from technograd_b200 import _lib, lm
    _lib.init(0, [local])
    torch.cuda.set_device(local)
    cfg = dict(lm.QWEN3_0_6B, layers=args.layers or lm.QWEN3_0_6B["layers"])
    total = (args.seqs or SMALL_SEQS) * world if small else args.seqs or TOTAL_SEQS
    prompt, new = args.prompt or PROMPT, args.new or NEW
    t0 = time.perf_counter()
    built = lm.DeviceBuilt(cfg, bits=4, method="gptq", seed=5)
    t_build = time.perf_counter() - t0
    lo, hi = shard_range(total, world, rank)
    shard = hi - lo
    wave = min(WAVE, shard)
    ids = decode_ids(total, prompt)[lo:hi]
    nwaves = (shard + wave - 1) // wave
    eng = lm.Engine(built, max_seqs=wave, max_len=prompt + new - 1, devices=[local])

    def step(i):
        w = i % nwaves
        return eng.generate(ids[w * wave:(w + 1) * wave], new)

    for i in range(args.warmup):
        step(i)
    # The timed steps run without the engine's per-kernel profiling events: an event between two
    # kernels of the captured decode step breaks their programmatic overlap and costs time of
    # its own. The breakdown and the roofline come from one profiled step of the same kind
    # right after the timed region.
    eng.profile(False)
    barrier(world)
    clk = Clocks(local)
    dev_ms, wall, launches = [], [], 0
    torch.cuda.nvtx.range_push("timed")  # lets a profiler restrict its launch list to the timed steps
    for i in range(args.steps):
        t = time.perf_counter()
        tok = step(args.warmup + i)
        wall.append(time.perf_counter() - t)
        s = eng.stats()
        dev_ms.append(s["device_ms"])
        launches += s["launches"]
    torch.cuda.nvtx.range_pop()
    barrier(world)
    clocks = clk.stop()
    eng.profile(True)
    step(args.warmup + args.steps)
    stats = [eng.stats()]
    eng.profile(False)
    t_dev = max_over_ranks(sum(dev_ms) / 1e3, world)
    t_wall = max_over_ranks(sum(wall), world)
    tokens_step = wave * new
    value = world * tokens_step * args.steps / t_dev
    pk, src = peaks()
    dec_bytes = sum(s["attn_decode_bytes"] for s in stats)
    dec_ms = sum(s["attn_decode_ms"] for s in stats)
    dec_launches = sum(s["attn_decode_launches"] for s in stats)
    achieved = dec_bytes / (dec_ms / 1e3) / 1e9
    gemm_tf = sum(s["gemm_flops"] for s in stats) / (sum(s["gemm_ms"] for s in stats) / 1e3) / 1e12
    pre_tf = sum(s["attn_prefill_flops"] for s in stats) / (sum(s["attn_prefill_ms"] for s in stats) / 1e3) / 1e12
    tot_ms = sum(s["device_ms"] for s in stats)  # the profiled step
    # the decode steps' products: the weight operands they read (int4 codes + scales for the
    # GEMVs of waves of up to 8 sequences, else the bf16 copies) per decode step, against HBM
    wb, wms = sum(s["decode_gemm_weight_bytes"] for s in stats), sum(s["decode_gemm_ms"] for s in stats)
    wl = "decode_small" if small else "decode"
    line = {
        "metric": METRICS[wl][0], "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sum(dev_ms) / len(dev_ms),
        "higher_is_better": True, "scaling": "weak" if small else "strong", "vs_baseline": None,
        "dtype": "f32 (bf16 hi/lo tensor-core split; f32 FMA in the small-wave GEMVs)",
        "data": "synthetic: random-init weights N(0,0.02), uniform-random prompt ids (seed 5)",
        "config": workload_config(wl, args),
        "breakdown": {"seqs_per_step_per_gpu": wave, "steps_for_full_job": nwaves,
                      "kv_cache": f"24-bit elements (bf16 + remainder byte, within 2^-16 of f32), "
                                  f"{wave * (prompt + new - 1) * cfg['layers'] * 8 * 128 * 6 / 1e9:.0f} GB per GPU at "
                                  f"{wave} seqs x {prompt + new - 1} positions",
                      "share_of_step": {"attn_decode": dec_ms / tot_ms, "gemm": sum(s["gemm_ms"] for s in stats) / tot_ms,
                                        "attn_prefill": sum(s["attn_prefill_ms"] for s in stats) / tot_ms},
                      "gemm_tflops": gemm_tf, "attn_prefill_tflops_f32": pre_tf, "build_s": t_build,
                      "decode_weights": {
                          "form": "int4 codes, dequant GEMVs" if wave <= 8 else "bf16 copies of the codes, tensor-core GEMMs",
                          "bytes_per_decode_step": wb / max(new - 1, 1), "ms_per_decode_step": wms / max(new - 1, 1),
                          "gbs": wb / max(wms, 1e-9) / 1e6, "frac_of_hbm": wb / max(wms, 1e-9) / 1e6 / pk["hbm_gbs"]},
                      "profiled_step_ms": tot_ms,
                      "profiled_step": "shares, TFLOP/s and the roofline: one step with per-kernel CUDA events right "
                                       "after the timed region (the timed steps run without them, so the decode "
                                       "step's kernels overlap by programmatic dependent launch)"},
        "roofline": {"kernel": "k_attn_decode (KV-cache attention)", "bound": "hbm", "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "peak_source": src,
                     # ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_attn_decode launch over 64
                     # sequences was 1.014x its algorithmic bytes; the bytes grow with sequences x keys
                     "traffic": 1.014 * dec_bytes / max(dec_launches, 1),
                     "traffic_source": "ncu dram read+write of a 64-sequence k_attn_decode launch (1.014x its "
                                       "algorithmic bytes), scaled to this launch's sequences x keys",
                     "bytes_per_launch": dec_bytes / max(dec_launches, 1),
                     "ms_per_launch": dec_ms / max(dec_launches, 1)},
        "e2e": {"value": world * tokens_step * args.steps / t_wall, "unit": "tokens/s",
                "h2d_bytes_per_step": wave * prompt * 4, "d2h_bytes_per_step": wave * new * 4},
        "gpu_launches": int(launches), "clocks": clocks,
    }
    if small:
        # a small wave's step is dominated by its products (the layers' GEMVs over int4 codes
        # and the LM head): their weight bytes per launch against HBM
        nl = sum(s["gemm_launches"] for s in stats)
        line["roofline"] = {"kernel": "gemv_dec (decode-step layer products over int4 codes) and the LM head's GEMM",
                            "bound": "hbm", "achieved": wb / max(wms, 1e-9) / 1e6, "peak": pk["hbm_gbs"], "unit": "GB/s",
                            "frac": wb / max(wms, 1e-9) / 1e6 / pk["hbm_gbs"], "peak_source": src, "traffic": None,
                            "bytes_per_launch": sum(s["gemm_weight_bytes"] for s in stats) / max(nl, 1),
                            "note": "latency-bound: about 10 us a launch for 1-4 MB of codes; the attention line of "
                                    "this step is in breakdown.attn_decode"}
        line["breakdown"]["attn_decode"] = {"gbs": achieved, "ms_per_launch": dec_ms / max(dec_launches, 1)}
    return line, built, tok


def ref_qwen3(T: int, bits: int, gptq: bool, seed: int):
    """The config-4/5 forward on the reference's own VM, in pieces (oracle/refvm.py)."""
    from oracle import refvm
    return refvm.Qwen3Pieces(T, bits, gptq, seed)


def ref_qwen3_line(P, per_seq_tokens: int, what: str) -> dict:
    """The rate the piece medians so far give: every host core runs one sequence's forward."""
    from oracle import refvm
    fwd = P.forward_seconds()
    n = {p: len(v) for p, v in P.times.items()}
    return {"value": P.threads * per_seq_tokens / fwd, "unit": "tokens/s", "cores": P.threads, "kind": "reference",
            "sample": f"{what}: the reference's VM (load_module, quantize_param, plan, vm_run_into from its own "
                      f"sources) on pieces of the Qwen3-0.6B-shape forward at T = {P.T}, one sequence per core on "
                      f"{P.threads} cores at once: one decoder layer's attention half, its gate/up half, its down "
                      f"projection, and the LM head on {refvm.HEAD_ROWS} of the {P.T} rows (timed {n['attn']}, "
                      f"{n['gate']}, {n['down']}, {n['head']} times, medians "
                      + ", ".join(f"{statistics.median(v):.2f}" for v in P.times.values()) +
                      f" s); one forward = 28 x (attn + gate + down) + {P.T // refvm.HEAD_ROWS} x head = {fwd:.0f} s "
                      f"per core; setup (writing, loading, quantizing the pieces) {P.setup_s:.0f} s, not timed",
            "forward_s_per_core": fwd}


def cpu_baseline_decode():
    """One pass over the pieces of a 1024-token forward (config 5: int4 GPTQ): the reference
    has no KV cache, so every generated token costs a forward of its whole prefix."""
    P = ref_qwen3(PROMPT, 4, True, 5)
    try:
        for piece in ("attn", "gate", "down", "head"):
            P.run(piece)
        return ref_qwen3_line(P, 1, "1 generated token per sequence at the prompt's 1024-token prefix "
                                    "(a lower bound of the cost: later tokens see up to 1280)")
    finally:
        P.close()


# ---- config 4: int8 RTN Qwen3-0.6B-shape batched prefill ---------------------------------------
PF_SEQS, PF_T = 64, 512


def bench_prefill(args, world, rank, local):
    import torch

    from technograd_b200 import _lib, lm
    _lib.init(0, [local])
    torch.cuda.set_device(local)
    cfg = dict(lm.QWEN3_0_6B, layers=args.layers or lm.QWEN3_0_6B["layers"])
    seqs, T = args.seqs or PF_SEQS, args.prompt or PF_T
    t0 = time.perf_counter()
    built = lm.DeviceBuilt(cfg, bits=8, method="rtn", seed=4)
    t_build = time.perf_counter() - t0
    lo, hi = shard_range(seqs, world, rank)
    shard = hi - lo
    ids = np.random.default_rng(4).integers(0, 151936, size=(seqs, T)).astype(np.float32)[lo:hi]
    eng = lm.Engine(built, max_seqs=shard, max_len=T, devices=[local])
    for _ in range(args.warmup):
        eng.forward(ids)
    # timed without the per-kernel profiling events; the breakdown and the roofline come from
    # one profiled forward right after the timed region
    eng.profile(False)
    barrier(world)
    clk = Clocks(local)
    dev_ms, wall, launches = [], [], 0
    torch.cuda.nvtx.range_push("timed")
    for _ in range(args.steps):
        t = time.perf_counter()
        eng.forward(ids)
        wall.append(time.perf_counter() - t)
        s = eng.stats()
        dev_ms.append(s["device_ms"])
        launches += s["launches"]
    torch.cuda.nvtx.range_pop()
    barrier(world)
    clocks = clk.stop()
    eng.profile(True)
    eng.forward(ids)
    stats = [eng.stats()]
    eng.profile(False)
    t_dev = max_over_ranks(sum(dev_ms) / 1e3, world)
    t_wall = max_over_ranks(sum(wall), world)
    tok = shard * T
    pk, src = peaks()
    gemm_ms = sum(s["gemm_ms"] for s in stats)
    gemm_fl = sum(s["gemm_flops"] for s in stats)
    achieved = gemm_fl / (gemm_ms / 1e3) / 1e12
    tot_ms = sum(s["device_ms"] for s in stats)  # the profiled forward
    line = {
        "metric": METRICS["prefill"][0], "value": world * tok * args.steps / t_dev,
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sum(dev_ms) / len(dev_ms),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (bf16 hi/lo tensor-core split)",
        "data": "synthetic: random-init weights N(0,0.02), uniform-random ids (seed 4)",
        "config": workload_config("prefill", args),
        "breakdown": {"seqs_per_gpu": shard,
                      "share_of_step": {"gemm": gemm_ms / tot_ms, "attn_prefill": sum(s["attn_prefill_ms"] for s in stats) / tot_ms},
                      "attn_prefill_tflops_f32": sum(s["attn_prefill_flops"] for s in stats) /
                      max(sum(s["attn_prefill_ms"] for s in stats) / 1e3, 1e-9) / 1e12, "build_s": t_build,
                      "profiled_step_ms": tot_ms,
                      "profiled_step": "shares, TFLOP/s and the roofline: one forward with per-kernel CUDA events "
                                       "right after the timed region (the timed forwards run without them)"},
        "roofline": {"kernel": "gemm_tc (tcgen05 dequant GEMM, all linear layers)", "bound": "tensor",
                     "achieved": achieved, "peak": pk["bf16_tflops_sustained"] if "bf16_tflops_sustained" in pk
                     else pk["bf16_tflops"], "unit": "TFLOP/s", "peak_source": src + " bf16 sustained",
                     "traffic": None, "flops_per_launch": gemm_fl / max(sum(s["gemm_launches"] for s in stats), 1)},
        "e2e": {"value": world * tok * args.steps / t_wall, "unit": "tokens/s", "h2d_bytes_per_step": ids.nbytes,
                "d2h_bytes_per_step": shard * cfg["vocab"] * 4},
        "gpu_launches": int(launches), "clocks": clocks,
    }
    line["roofline"]["frac"] = achieved / line["roofline"]["peak"]
    return line, built


def cpu_baseline_prefill():
    """One pass over the pieces of a 512-token forward (config 4: int8 RTN), the prefill of
    one sequence per core."""
    P = ref_qwen3(PF_T, 8, False, 4)
    try:
        for piece in ("attn", "gate", "down", "head"):
            P.run(piece)
        return ref_qwen3_line(P, PF_T, "a 512-token prefill per sequence")
    finally:
        P.close()


# ---- config 3: stacked selective-SSM blocks ------------------------------------------------------
SSM_SEQS, SSM_T = 1024, 4096
# DRAM bytes / algorithmic bytes of one k_ssm_scan launch, from ncu dram__bytes_read.sum +
# dram__bytes_write.sum (91.3 MB of 103.8 MB on 256 sequences x 512 channels: the g writes are
# partly still in L2 when the kernel ends)
SSM_SCAN_TRAFFIC_RATIO = 91.3 / 103.8


def ssm_inputs(seqs: int, T: int, lo: int, hi: int) -> np.ndarray:
    """Sequences [lo, hi) of the seeded N(0,1) input [seqs, T, 256] (seed 3), generated in
    blocks so a rank only materialises its own shard."""
    rng = np.random.default_rng(3)
    out = np.empty((hi - lo, T, 256), np.float32)
    for s in range(hi):
        row = rng.standard_normal((T, 256), dtype=np.float32)
        if s >= lo:
            out[s - lo] = row
    return out


def bench_ssm(args, world, rank, local):
    import torch

    from technograd_b200 import _lib, ssm
    _lib.init(0, [local])
    torch.cuda.set_device(local)
    cfg = dict(ssm.CONFIG3, blocks=args.layers or ssm.CONFIG3["blocks"])
    seqs, T = args.seqs or SSM_SEQS, args.prompt or SSM_T
    lo, hi = shard_range(seqs, world, rank)
    t0 = time.perf_counter()
    model = ssm.quantize_rtn_device(ssm.random_weights(cfg, seed=3), cfg, 8)
    u = ssm_inputs(seqs, T, lo, hi)
    t_build = time.perf_counter() - t0
    S = hi - lo
    eng = ssm.Engine(model, max_seqs=S, chunk=64, devices=[local])
    du = torch.from_numpy(u).cuda()
    dout = torch.empty_like(du)
    for _ in range(args.warmup):
        eng.forward_device(du.data_ptr(), S, T, dout.data_ptr())
    # timed without the per-kernel profiling events; the breakdown and the roofline come from
    # one profiled forward right after the timed region
    eng.profile(False)
    barrier(world)
    clk = Clocks(local)
    dev_ms, launches = [], 0
    torch.cuda.nvtx.range_push("timed")
    for _ in range(args.steps):
        eng.forward_device(du.data_ptr(), S, T, dout.data_ptr())
        s = eng.stats()
        dev_ms.append(s["device_ms"])
        launches += s["launches"]
    torch.cuda.nvtx.range_pop()
    barrier(world)
    clocks = clk.stop()
    eng.profile(True)
    eng.forward_device(du.data_ptr(), S, T, dout.data_ptr())
    stats = [eng.stats()]
    t_dev = max_over_ranks(sum(dev_ms) / 1e3, world)
    # e2e: host (pinned) rows in, host rows out, through tg_cuda_ssm_forward
    hu = torch.from_numpy(u).pin_memory()
    ho = torch.empty_like(hu).pin_memory()
    eng.profile(False)
    _lib.check(_lib.lib().tg_cuda_ssm_forward(eng.handle, hu.data_ptr(), S, T, ho.data_ptr()))
    barrier(world)
    wall = []
    for _ in range(args.steps):
        t1 = time.perf_counter()
        _lib.check(_lib.lib().tg_cuda_ssm_forward(eng.handle, hu.data_ptr(), S, T, ho.data_ptr()))
        wall.append(time.perf_counter() - t1)
    t_wall = max_over_ranks(sum(wall), world)
    tok = S * T
    scan_ms = sum(s["scan_ms"] for s in stats)
    gemm_ms = sum(s["gemm_ms"] for s in stats)
    tot_ms = sum(s["device_ms"] for s in stats)  # the profiled forward
    pk, src = peaks()
    scan_tf = sum(s["scan_flops"] for s in stats) / (scan_ms / 1e3) / 1e12
    gemm_tf = sum(s["gemm_flops"] for s in stats) / (gemm_ms / 1e3) / 1e12
    full = (seqs, T, cfg["blocks"]) == (SSM_SEQS, SSM_T, 4)
    # k_ssm_scan reads xs, z and the [dt | B | C] rows and writes g as bf16 hi/lo, per launch
    # (S sequences x one chunk of 64 steps)
    scan_bytes = float(S * 64 * (cfg["d_inner"] * 12 + (cfg["dt_rank"] + 2 * cfg["d_state"]) * 4))
    line = {
        "metric": METRICS["ssm"][0], "value": world * tok * args.steps / t_dev,
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sum(dev_ms) / len(dev_ms),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (bf16 hi/lo tensor-core split)",
        "data": "synthetic: random-init weights N(0,0.02) int8 RTN, inputs N(0,1) (seed 3)",
        "config": workload_config("ssm", args),
        "breakdown": {"seqs_per_gpu": S, "chunk": 64, "share_of_step": {"scan": scan_ms / tot_ms, "gemm": gemm_ms / tot_ms},
                      "gemm_tflops": gemm_tf, "build_s": t_build, "profiled_step_ms": tot_ms,
                      "profiled_step": "shares, TFLOP/s and the roofline: one forward with per-kernel CUDA events "
                                       "right after the timed region (the timed forwards run without them)"},
        "roofline": {"kernel": "k_ssm_scan (FP32 pipe + SFU)", "bound": "fp32", "achieved": scan_tf,
                     "peak": FP32_NOMINAL_TFLOPS, "unit": "TFLOP/s", "frac": scan_tf / FP32_NOMINAL_TFLOPS,
                     "peak_source": "nominal FP32 SIMT (148 SMs x 128 lanes x FMA x 1965 MHz); not in MEASURED_PEAKS",
                     "traffic": SSM_SCAN_TRAFFIC_RATIO * scan_bytes, "bytes_per_launch": scan_bytes,
                     "traffic_source": "ncu dram read+write of a 256-sequence k_ssm_scan launch (0.88x its algorithmic "
                                       "bytes), scaled to this launch's sequences"},
        "e2e": {"value": world * tok * args.steps / t_wall, "unit": "tokens/s", "h2d_bytes_per_step": u.nbytes,
                "d2h_bytes_per_step": u.nbytes},
        "gpu_launches": int(launches), "clocks": clocks,
    }
    return line, model


SSM_REF_T = 256


def cpu_baseline_ssm(S=None, runs: int = 1):
    """The config-3 program on the reference's own VM (oracle/refvm.py SsmSample): one
    sequence of SSM_REF_T steps per host core, all at once."""
    from oracle import refvm
    own = S is None
    S = S or refvm.SsmSample(SSM_REF_T)
    try:
        t = statistics.median([S.run() for _ in range(runs)])
        return {"value": S.threads * S.T / t, "unit": "tokens/s", "cores": S.threads, "kind": "reference",
                "sample": f"the reference's VM (load_module, quantize_param --bits 8 --min-size 1, plan, vm_run_into) "
                          f"on the config-3 program at full block widths, {S.T} steps per sequence, one sequence per "
                          f"core on {S.threads} cores at once, {t:.2f} s (a scan step costs the same at every position)"}
    finally:
        if own:
            S.close()


# ---- config 2: weight-only dequant GEMM microbench ---------------------------------------------
GEMM_N = GEMM_K = 4096
# DRAM bytes (read + write) of one gemm_tc launch, from an ncu capture: (M, bits) -> bytes
GEMM_TRAFFIC = {(256, 4): 12625920.0, (1, 4): 8438016.0}  # ncu dram read + write of one launch


def gemm_inputs(bits: int, M: int):
    """W codes uniform in [-8, 7] (int4) or [-127, 127] (int8), [N, K]; scale |N(0,0.02)|/7 or /127
    per output row; X [M, K] ~ N(0,1); seed 2. The reference op is tg_matmul_qa(o, q, bits, s, X^T, N, K, M)."""
    rng = np.random.default_rng(2)
    lo, hi = (-8, 8) if bits == 4 else (-127, 128)
    codes = rng.integers(lo, hi, size=GEMM_N * GEMM_K)
    if bits == 8:
        q = codes.astype(np.int8)
    else:  # element i in byte i/2, low nibble first (runtime/tg_rt.h:124-129)
        nib = (codes & 0xF).astype(np.uint8)
        q = (nib[0::2] | (nib[1::2] << 4)).view(np.int8)
    q = np.ascontiguousarray(q)
    s = (np.abs(rng.normal(0, 0.02, size=GEMM_N)) / (7 if bits == 4 else 127)).astype(np.float32)
    x = rng.standard_normal((M, GEMM_K), dtype=np.float32)
    return q, s, np.ascontiguousarray(x.T)  # b = X^T [K, M]


def gemm_cost(bits: int, M: int):
    N, K = GEMM_N, GEMM_K
    byts = N * K * bits // 8 + 4 * N + 4 * M * K + 4 * M * N
    return byts, 2.0 * M * N * K


def bench_gemm(args, world, rank, local, M: int, bits: int):
    import torch

    from technograd_b200 import _lib
    _lib.init(0, [local])
    torch.cuda.set_device(local)
    L = _lib.lib()
    q, s, b = gemm_inputs(bits, M)
    # copies of the weights, cycled step by step: together larger than the 126 MB L2, so no
    # step finds its codes in L2 (a flush between single calls would time the launch instead)
    ncopies = max(2, -(-(256 << 20) // q.nbytes))
    dq = torch.from_numpy(q).cuda().repeat(ncopies).view(ncopies, -1)
    ds, db = (torch.from_numpy(a).cuda() for a in (s, b))
    do = torch.empty((GEMM_N, M), device="cuda")
    flush = L2Flush()
    side = torch.cuda.Stream()
    torch.cuda.set_stream(side)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)

    def call(o_ptr, b_ptr, i=0):
        _lib.check(L.tg_cuda_matmul_q(0, o_ptr, b_ptr, dq[i % ncopies].data_ptr(), bits, ds.data_ptr(), GEMM_N, GEMM_K, M, sp))

    for i in range(max(args.warmup, 2)):  # the first calls allocate the library's scratch
        call(do.data_ptr(), db.data_ptr(), i)
    torch.cuda.synchronize()
    # a step is one call on each weight copy in turn (a stream of GEMMs, as a decoder issues
    # them); the K timed steps are captured as one CUDA graph so the per-call launch cost of
    # the host is not timed
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(args.steps * ncopies):
            call(do.data_ptr(), db.data_ptr(), i)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    clk = Clocks(local)
    clk.first()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush()
    torch.cuda.nvtx.range_push("timed")
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clk.hold(lambda: (graph.replay(), torch.cuda.synchronize()))
    barrier(world)
    clocks = clk.stop()
    ms = [e0.elapsed_time(e1) / args.steps] * args.steps
    t = max_over_ranks(sum(ms) / 1e3, world)
    del graph
    # e2e: activations from pinned host memory in, the product back to pinned host memory
    hb = torch.from_numpy(b).pin_memory()
    ho = torch.empty((GEMM_N, M)).pin_memory()
    db2, do2 = torch.empty_like(db), torch.empty_like(do)

    def e2e_call():
        db2.copy_(hb, non_blocking=True)
        call(do2.data_ptr(), db2.data_ptr())
        ho.copy_(do2, non_blocking=True)
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        e2e_call()
    barrier(world)
    wall = []
    for _ in range(args.steps):
        flush()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        e2e_call()
        wall.append(time.perf_counter() - t1)
    te = max_over_ranks(sum(wall), world)
    byts, flops = gemm_cost(bits, M)
    pk, src = peaks()
    per = sum(ms) / 1e3 / args.steps / ncopies  # one GEMM
    hbm = M <= 16
    if hbm:
        achieved, peak, unit = byts / per / 1e9, pk["hbm_gbs"], "GB/s"
    else:
        achieved, peak, unit = flops / per / 1e12, pk["bf16_tflops"], "TFLOP/s"
    path = ("gemv_bulk (code rows read coalesced into registers, CUDA cores, packed f32x2 FMAs)" if M <= 8 else
            "split_f32_t (activations -> bf16 hi/lo) + gemm_tc (tcgen05, codes expanded in the kernel)")
    line = {
        "metric": gemm_metric(bits, M)[0],
        "value": world * args.steps * ncopies / t, "unit": "GEMM/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": sum(ms) / len(ms), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"int{bits} codes, f32 activations and accumulation" + ("" if M <= 8 else " (bf16 hi/lo split)"),
        "data": "synthetic (seed 2)",
        "config": workload_config("gemm", args, M),
        "breakdown": {"path": path, "gemms_per_step": ncopies, "us_per_gemm": per * 1e6, "weight_copies": ncopies,
                      "weight_bytes_cycled": ncopies * q.nbytes, "algorithmic_bytes": byts, "flops": flops},
        "roofline": {"kernel": path, "bound": "hbm" if hbm else "tensor", "achieved": achieved, "peak": peak,
                     "unit": unit, "frac": achieved / peak, "peak_source": src + (" hbm_gbs" if hbm else " bf16 burst"),
                     "traffic": GEMM_TRAFFIC.get((M, bits)),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of the path's main "
                                       "kernel at this M" if (M, bits) in GEMM_TRAFFIC else None},
        "e2e": {"value": world * args.steps / te, "unit": "GEMM/s", "h2d_bytes_per_step": b.nbytes,
                "d2h_bytes_per_step": GEMM_N * M * 4,
                "step": "one GEMM through tg_cuda_matmul_q: activations in from pinned host memory, the product out"},
        # GEMV: one kernel; tensor cores: the activation split, the GEMM, and the fixed-order
        # split-K reduction when fewer than 74 output tiles would leave SMs idle
        "gpu_launches": args.steps * ncopies * (1 if M <= 8 else 2 + (32 * -(-M // (256 if M >= 256 else 128)) * 2 <= 148)),
        "clocks": clocks,
    }
    return line, (q, s, b)


def cpu_baseline_gemm(q, s, b, bits: int, M: int, budget_s: float = 10.0):
    """The reference's own tg_matmul_qa (runtime/tg_rt.h, compiled into oracle/_ref) on the host
    cores. `tgc batch` runs one GEMV per row (src/main.c:231-242) on -j auto threads, so the
    columns of b are split over threads; a bounded sample of columns is timed and scaled."""
    from oracle import tgo
    R = tgo.ref()
    kind, fn = ("reference", R.ref_matmul_qa) if R is not None else ("port", tgo.tgo().tgo_matmul_qa)
    threads = min(os.cpu_count() or 1, M)
    # calibrate: one column on one thread
    o1 = np.zeros(GEMM_N, np.float32)
    b1 = np.ascontiguousarray(b[:, :1])
    t0 = time.perf_counter()
    fn(tgo.f32p(o1), tgo.i8p(q), bits, tgo.f32p(s), tgo.f32p(b1), GEMM_N, GEMM_K, 1)
    per_col = time.perf_counter() - t0
    cols = max(threads, min(M, int(budget_s * threads / max(per_col, 1e-6))))
    cols -= cols % threads if cols >= threads else 0
    cols = max(cols, 1)
    chunks = np.array_split(np.arange(cols), threads)
    subs = [np.ascontiguousarray(b[:, c]) for c in chunks]
    outs = [np.zeros(GEMM_N * len(c), np.float32) for c in chunks]

    def work(i):
        n = len(chunks[i])
        if n:
            fn(tgo.f32p(outs[i]), tgo.i8p(q), bits, tgo.f32p(s), tgo.f32p(subs[i]), GEMM_N, GEMM_K, n)

    t0 = time.perf_counter()
    th = [threading.Thread(target=work, args=(i,)) for i in range(threads)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    dt = time.perf_counter() - t0
    return {"value": (cols / M) / dt, "unit": "GEMM/s", "cores": threads, "kind": kind,
            "sample": f"{cols} of the {M} activation columns on {threads} thread(s), {dt:.1f} s, scaled to the full GEMM"}


# ---- config 1: latent_reasoner -----------------------------------------------------------------
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
    m = tgir.load(os.path.join(ROOT, "tests", "golden", "latent_reasoner.q8.tgir"))
    rows = lr_inputs(LR_ROWS)
    _lib.init(0, [local])
    b = Batch(m)
    spec, why = b.specialized
    L = _lib.lib()
    d_in = torch.from_numpy(rows).cuda()
    d_out = torch.empty((LR_ROWS, 4), device="cuda")
    d_steps = torch.empty((LR_ROWS, 1), dtype=torch.int32, device="cuda")
    flush = L2Flush()
    stream = torch.cuda.current_stream()

    def step():
        _lib.check(L.tg_cuda_batch_device(b.handle, d_in.data_ptr(), LR_ROWS, d_out.data_ptr(), d_steps.data_ptr(),
                                          C.c_void_p(stream.cuda_stream)))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    clk = Clocks(local)
    clk.first()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        flush()
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    clk.hold(lambda: (step(), torch.cuda.synchronize()))
    barrier(world)
    clocks = clk.stop()
    ms = [a.elapsed_time(z) for a, z in ev]
    t = max_over_ranks(sum(ms) / 1e3, world)
    steps_np = d_steps.cpu().numpy()
    achieved = lr_flops(steps_np) / (t / args.steps) / 1e12
    out_h = np.empty((LR_ROWS, 4), np.float32)
    st_h = np.empty((LR_ROWS, 1), np.int32)

    def e2e() -> float:
        for _ in range(2):
            _lib.check(L.tg_cuda_batch(b.handle, rows.ctypes.data, LR_ROWS, 8, out_h.ctypes.data, 4, st_h.ctypes.data, 1))
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _lib.check(L.tg_cuda_batch(b.handle, rows.ctypes.data, LR_ROWS, 8, out_h.ctypes.data, 4, st_h.ctypes.data, 1))
        return max_over_ranks(time.perf_counter() - t0, world)

    te_pageable = e2e()  # the driver's plain buffers: through the library's staging buffers
    with _lib.HostRegistered(rows, out_h, st_h):  # page-locked once, outside the timed region
        te = e2e()
    line = {
        "metric": METRICS["lr"][0], "value": world * LR_ROWS * args.steps / t,
        "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sum(ms) / len(ms), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": workload_config("lr", args),
        "breakdown": {"think_steps_mean": float(steps_np.mean()),
                      "e2e_host_buffers": "page-locked with tg_cuda_host_register (direct DMA)",
                      "e2e_pageable_rows_per_s": world * LR_ROWS * args.steps / te_pageable,
                      "kernel": "generated for the program (NVRTC, sm_100a)" if spec else f"tape interpreter ({why})"},
        "roofline": {"kernel": "tg_rowvm (generated for the program)" if spec else "vm_kernel (tape interpreter)",
                     "bound": "fp32", "achieved": achieved, "peak": FP32_NOMINAL_TFLOPS,
                     "unit": "TFLOP/s", "frac": achieved / FP32_NOMINAL_TFLOPS, "traffic": None,
                     "peak_source": "nominal FP32 SIMT (148 SMs x 128 lanes x FMA x 1965 MHz); not in MEASURED_PEAKS"},
        "e2e": {"value": world * LR_ROWS * args.steps / te, "unit": "rows/s", "h2d_bytes_per_step": rows.nbytes,
                "d2h_bytes_per_step": out_h.nbytes + st_h.nbytes},
        "gpu_launches": args.steps, "clocks": clocks,
    }
    return line, rows


def cpu_baseline_lr(rows: np.ndarray):
    """The reference's own `tgc batch -j auto` (oracle/_ref/tgc, compiled from its sources) on the host cores."""
    from oracle import tgo
    tgc = tgo.REF_TGC
    if not os.path.exists(tgc):
        return None
    model = os.path.join(ROOT, "tests", "golden", "latent_reasoner.q8.tgir")
    with tempfile.TemporaryDirectory() as d:
        inp = os.path.join(d, "rows.bin")
        rows.astype("<f4").tofile(inp)
        r = subprocess.run([tgc, "batch", model, inp, "-j", "auto", "-v", "-o", os.path.join(d, "out.bin")],
                           capture_output=True, text=True, check=True)
    mt = re.search(r"\[batch\] (\d+) row\(s\) in ([0-9.]+) ms .* on (\d+) thread", r.stderr)
    n, ms, th = int(mt.group(1)), float(mt.group(2)), int(mt.group(3))
    return {"value": n / (ms / 1e3), "unit": "rows/s", "cores": th, "kind": "reference",
            "sample": f"{n} rows of config 1, `tgc batch -j auto` binary I/O, [batch] event time"}


# ---- the reference arm --------------------------------------------------------------------------

def reference_arm(args) -> list:
    """The reference's own CPU implementation of the path, timed on the host cores (no GPU,
    no process group, nothing of technograd_b200): the lines for --workload (config 5 by
    default), with the same metric, unit and config as this repository's arm."""
    wl = "decode" if args.workload == "all" else args.workload
    out = []

    def emit(metric, unit, cfg, scaling, vals, walls, base):
        v = statistics.median(vals)
        base = dict(base, value=v)
        out.append({"impl": "reference", "metric": metric, "value": v, "unit": unit, "n_gpus": 0, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": 1e3 * sum(walls) / len(walls), "higher_is_better": True,
                    "scaling": scaling, "vs_baseline": None, "dtype": "f32 (int8/int4 codes, f32 accumulation)",
                    "data": "synthetic", "config": cfg, "cpu_baseline": base,
                    "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})

    if wl == "lr":
        rows = lr_inputs(LR_ROWS)
        if cpu_baseline_lr(rows) is None:
            return [{"impl": "reference", "unavailable": "oracle/_ref/tgc was not built (needs the reference sources)"}]
        for _ in range(args.warmup):
            cpu_baseline_lr(rows)
        vals, walls, base = [], [], None
        for _ in range(args.steps):
            t = time.perf_counter()
            base = cpu_baseline_lr(rows)
            walls.append(time.perf_counter() - t)
            vals.append(base["value"])
        emit(*METRICS["lr"], workload_config("lr", args), "weak", vals, walls, base)
    elif wl == "gemm":
        for M in args.m:
            q, s, b = gemm_inputs(args.bits, M)
            for _ in range(args.warmup):
                cpu_baseline_gemm(q, s, b, args.bits, M, budget_s=0.5)
            vals, walls, base = [], [], None
            for _ in range(args.steps):
                t = time.perf_counter()
                base = cpu_baseline_gemm(q, s, b, args.bits, M, budget_s=1.0)
                walls.append(time.perf_counter() - t)
                vals.append(base["value"])
            emit(*gemm_metric(args.bits, M), workload_config("gemm", args, M), "weak", vals, walls, base)
    elif wl == "ssm":
        from oracle import refvm
        S = refvm.SsmSample(SSM_REF_T)
        try:
            for _ in range(args.warmup):
                S.run()
            vals, walls, base = [], [], None
            for _ in range(args.steps):
                t = time.perf_counter()
                base = cpu_baseline_ssm(S)
                walls.append(time.perf_counter() - t)
                vals.append(base["value"])
        finally:
            S.close()
        emit(*METRICS["ssm"], workload_config("ssm", args), "strong", vals, walls, base)
    else:
        from oracle import refvm
        pre = wl == "prefill"
        P = ref_qwen3(PF_T if pre else PROMPT, 8 if pre else 4, not pre, 4 if pre else 5)
        try:
            for i in range(args.warmup):
                P.run(refvm.PIECES[i % len(refvm.PIECES)])
            P.times = {p: [] for p in refvm.PIECES}
            walls = []
            # one piece per step, in turn; at least one of each, so a forward can be assembled
            for i in range(max(args.steps, len(refvm.PIECES))):
                walls.append(P.run(refvm.PIECES[i % len(refvm.PIECES)]))
            base = ref_qwen3_line(P, PF_T if pre else 1, "a 512-token prefill per sequence" if pre else
                                  "1 generated token per sequence at the prompt's 1024-token prefix (a lower bound "
                                  "of the cost: later tokens see up to 1280)")
        finally:
            P.close()
        emit(*METRICS[wl], workload_config(wl, args), "weak" if wl == "decode_small" else "strong", [base["value"]], walls,
             base)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="all", choices=["all", "decode", "decode_small", "lr", "prefill", "gemm", "ssm"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # shape overrides for small profiling captures; the line's config says when they were used
    ap.add_argument("--seqs", type=int, default=0)
    ap.add_argument("--prompt", type=int, default=0)
    ap.add_argument("--new", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0)
    # config 2: batch sizes (one JSON line per M) and code width
    ap.add_argument("--m", type=lambda v: [int(x) for x in v.split(",")], default=[1, 16, 256, 4096])
    ap.add_argument("--bits", type=int, default=4, choices=[4, 8])
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    faulthandler.enable()  # a fatal signal (abort, segfault) prints the Python stack of every thread
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return  # rank 0 alone times the reference; the others have no work
        for line in reference_arm(args):
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup()
    base = rank == 0 and world == 1 and not args.no_cpu_baseline
    order = ["lr", "gemm", "ssm", "prefill", "decode_small", "decode"] if args.workload == "all" else [args.workload]
    ref_decode = None  # the reference's per-token cost is the same for both decode lines: timed once
    for wl in order:
        lines = []
        if wl == "lr":
            line, rows = bench_lr(args, world, rank, local)
            if base:
                line["cpu_baseline"] = cpu_baseline_lr(rows)
            lines.append(line)
        elif wl == "gemm":
            for M in args.m:
                line, data = bench_gemm(args, world, rank, local, M, args.bits)
                if base:
                    line["cpu_baseline"] = cpu_baseline_gemm(*data, args.bits, M, budget_s=3.0)
                lines.append(line)
        elif wl == "ssm":
            line, _ = bench_ssm(args, world, rank, local)
            if base:
                line["cpu_baseline"] = cpu_baseline_ssm()
            lines.append(line)
        elif wl == "prefill":
            line, _ = bench_prefill(args, world, rank, local)
            if base:
                line["cpu_baseline"] = cpu_baseline_prefill()
            lines.append(line)
        else:
            line, _, _ = bench_decode(args, world, rank, local, small=wl == "decode_small")
            if base:
                ref_decode = ref_decode or cpu_baseline_decode()
                line["cpu_baseline"] = ref_decode
            lines.append(line)
        if rank == 0:
            for line in lines:
                print(json.dumps(line), flush=True)
        import gc

        import torch
        gc.collect()
        torch.cuda.empty_cache()
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
