"""The reference's own VM timed on the decoder configs (TEST / BASELINE INFRASTRUCTURE ONLY).

bench.py's reference arm and its cpu_baseline time the reference itself -- its parser,
planner, quantizer and VM (src/util.c load_module, src/plan.c, src/quant.c, src/vm.c
vm_run_into), compiled from its own sources into oracle/_ref/libtgref.so -- on the
Qwen3-0.6B-shape programs of configs 4 and 5, with nothing of this repository's
product on the path (no technograd_b200 import, no libtgcuda).

The reference has no KV cache: each generated token of config 5 is one forward of the
whole prefix (examples/qwen3/import.py:130-131 emits one program per sequence length,
run by src/vm.c:475-481), about 15 minutes of one core at a 1024-token prefix. So a
timed step runs one PIECE of that forward, cut from the program import.py emits at the
config's sequence length T, on every host core at once (one sequence per core, as
`tgc batch -j auto` runs rows):

  attn  one decoder layer's attention half: n = rmsnorm(h) * ln1; per KV head
        k = rotary(rmsnorm(n @ Wk) * kn), v = n @ Wv; per query head q = rotary(...),
        s = softmax((q @ transpose(k)) * scale + mask), o = (s @ v) @ Wo;
        h + (o0 + ... + o15)                                     (import.py:102-113)
  gate  the same layer's MLP up to its down projection: n = rmsnorm(h) * ln2;
        g = silu(n @ Wg) * (n @ Wu)                               (import.py:114-115)
  down  the rest of that line: h + g @ Wd                         (import.py:115)
  head  the LM head on HEAD_ROWS of the T rows: (rmsnorm(h) * lnf) @ LM
        (import.py:116; the reference applies it to every row before take(lastidx))

The 28 layers have identical shapes, and the head's cost is linear in its rows
(tg_matmul_qb computes each output row on its own, runtime/tg_rt.h:143-151), so one
forward costs 28 * (attn + gate + down) + (T / HEAD_ROWS) * head; the embedding gather
of T rows is left out (well under 0.1%). Splitting the MLP line in two keeps every
timed step near ten seconds. Weights are seeded N(0, 0.02) (norms 1), quantized
in process by the reference's quantize_param: config 5 int4 GPTQ against 256 seeded
N(0,1) rows per input width (inputs wider than 2048 by RTN, src/quant.c:346) -- except
the LM head, whose 1024 x 151,936 GPTQ sweep would take minutes of setup and whose
codes do not change the kernel's time, so it is RTN; config 4 int8 RTN. Rot stays f32
(--min-size 16385), as in the fixtures of tests/golden/make_golden.py.
"""
from __future__ import annotations

import ctypes as C
import math
import os
import statistics
import tempfile

import numpy as np

from . import tgo

QWEN3 = dict(layers=28, hidden=1024, nq=16, nkv=8, head_dim=128, ffn=3072, vocab=151936, theta=1e6)
HEAD_ROWS = 16
PIECES = ("attn", "gate", "down", "head")


def lib():
    R = tgo.ref()
    if R is None:
        return None
    R.ref_vm_load.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int]
    R.ref_vm_load.restype = C.c_void_p
    R.ref_vm_run.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_double)]
    R.ref_vm_run.restype = C.c_int
    return R


def _tables(T: int, HD: int, theta: float) -> dict:
    """cosT, sinT, Rot and the causal mask as import.py:74-86 writes them."""
    inv = theta ** (-(np.arange(0, HD, 2) / HD))
    ang = np.outer(np.arange(T), inv)
    rot = np.zeros((HD, HD), np.float32)
    for i in range(HD // 2):
        rot[i + HD // 2, i] = -1.0
        rot[i, i + HD // 2] = 1.0
    return {"cosT": np.concatenate([np.cos(ang), np.cos(ang)], axis=1),
            "sinT": np.concatenate([np.sin(ang), np.sin(ang)], axis=1), "Rot": rot,
            "mask": np.where(np.arange(T)[None, :] <= np.arange(T)[:, None], 0.0, -1e9)}


def emit_piece(piece: str, T: int, outdir: str, seed: int, cfg: dict = QWEN3) -> str:
    """Write the piece's program and its file() weights under outdir; return the .tg path."""
    D, NQ, NKV, HD, FF, V = (cfg[k] for k in ("hidden", "nq", "nkv", "head_dim", "ffn", "vocab"))
    rng = np.random.default_rng(seed)
    wdir = os.path.join(outdir, "w")
    os.makedirs(wdir, exist_ok=True)
    lines = [f"model qwen3_{piece}", ""]

    def par(name, arr):
        np.asarray(arr, dtype="<f4").tofile(os.path.join(wdir, name + ".bin"))
        lines.append(f'param {name} : f32[{", ".join(map(str, np.shape(arr)))}] = file("w/{name}.bin")')

    def g(*shape):
        return rng.standard_normal(size=shape, dtype=np.float32) * np.float32(0.02)

    if piece == "attn":
        tab = _tables(T, HD, cfg["theta"])
        par("ln1", np.ones(D)), par("qn", np.ones(HD)), par("kn", np.ones(HD))
        for name in ("cosT", "sinT", "Rot", "mask"):
            par(name, tab[name])
        for h in range(NQ):
            par(f"Wq_{h}", g(D, HD)), par(f"Wo_{h}", g(HD, D))
        for j in range(NKV):
            par(f"Wk_{j}", g(D, HD)), par(f"Wv_{j}", g(D, HD))
        lines += ["", f"def rotary(x: f32[{T}, {HD}]) -> f32[{T}, {HD}]:", "    return x * cosT + (x @ Rot) * sinT", "",
                  f"def forward(h: f32[{T}, {D}]) -> f32[{T}, {D}]:", "    n = rmsnorm(h) * ln1"]
        for j in range(NKV):
            lines += [f"    k{j} = rotary(rmsnorm(n @ Wk_{j}) * kn)", f"    v{j} = n @ Wv_{j}"]
        grp, scale = NQ // NKV, 1.0 / math.sqrt(HD)
        for h in range(NQ):
            lines += [f"    q{h} = rotary(rmsnorm(n @ Wq_{h}) * qn)",
                      f"    s{h} = softmax((q{h} @ transpose(k{h // grp})) * {scale:.9g} + mask)",
                      f"    o{h} = (s{h} @ v{h // grp}) @ Wo_{h}"]
        lines.append(f"    return h + ({' + '.join(f'o{h}' for h in range(NQ))})")
    elif piece == "gate":
        par("ln2", np.ones(D)), par("Wg", g(D, FF)), par("Wu", g(D, FF))
        lines += ["", f"def forward(h: f32[{T}, {D}]) -> f32[{T}, {FF}]:", "    n = rmsnorm(h) * ln2",
                  "    return silu(n @ Wg) * (n @ Wu)"]
    elif piece == "down":
        par("Wd", g(FF, D))
        lines += ["", f"def forward(h: f32[{T}, {D}], g: f32[{T}, {FF}]) -> f32[{T}, {D}]:", "    return h + g @ Wd"]
    elif piece == "head":
        par("lnf", np.ones(D)), par("LM", g(D, V))
        lines += ["", f"def forward(h: f32[{HEAD_ROWS}, {D}]) -> f32[{HEAD_ROWS}, {V}]:",
                  "    return (rmsnorm(h) * lnf) @ LM"]
    else:
        raise ValueError(piece)
    path = os.path.join(outdir, f"{piece}.tg")
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return path


# ---- config 3: the stacked selective-SSM program ---------------------------------------------

SSM3 = dict(blocks=4, d_model=256, d_inner=512, d_state=16, dt_rank=16)


def ssm_weights(cfg: dict, seed: int) -> dict:
    """Projections and conv weights ~ N(0, 0.02); norms 1; a = 1..d_state per channel; d = 1;
    the dt bias the inverse softplus of dt log-uniform in [1e-3, 1e-1] (config 3's init)."""
    rng = np.random.default_rng(seed)
    B, DM, DI, DS, R = (cfg[k] for k in ("blocks", "d_model", "d_inner", "d_state", "dt_rank"))

    def g(*s):
        return rng.standard_normal(size=s, dtype=np.float32) * np.float32(0.02)

    w = {"nf": np.ones(DM, np.float32)}
    for b in range(B):
        w[f"nw_{b}"] = np.ones(DM, np.float32)
        w[f"Wx_{b}"], w[f"Wz_{b}"] = g(DM, DI), g(DM, DI)
        for i in range(4):
            w[f"cw{i}_{b}"] = g(DI)
        w[f"cb_{b}"] = g(DI)
        w[f"Wr_{b}"], w[f"WB_{b}"], w[f"WC_{b}"] = g(DI, R), g(DI, DS), g(DI, DS)
        w[f"Wdt_{b}"] = g(R, DI)
        dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), size=DI))
        w[f"bdt_{b}"] = (dt + np.log(-np.expm1(-dt))).astype(np.float32)
        w[f"A_{b}"] = np.tile(np.arange(1, DS + 1, dtype=np.float32), (DI, 1))
        w[f"D_{b}"] = np.ones(DI, np.float32)
        w[f"Wo_{b}"] = g(DI, DM)
    return w


def emit_ssm(cfg: dict, w: dict, outdir: str, T: int) -> str:
    """The config-3 program in the reference's language: per block one scan over the steps
    with the state h and the last three conv inputs as carries (include/tg_cuda.h
    tg_cuda_ssm_desc states the arithmetic)."""
    B, DM, DI, DS, R = (cfg[k] for k in ("blocks", "d_model", "d_inner", "d_state", "dt_rank"))
    os.makedirs(os.path.join(outdir, "w"), exist_ok=True)
    tables = {"Zh": np.zeros((DI, DS), np.float32), "Zc": np.zeros(DI, np.float32)}
    for name, arr in list(w.items()) + list(tables.items()):
        np.asarray(arr, dtype="<f4").tofile(os.path.join(outdir, "w", name + ".bin"))
    lines = ["model ssm", ""]

    def par(name, *shape):
        lines.append(f'param {name} : f32[{", ".join(map(str, shape))}] = file("w/{name}.bin")')

    par("nf", DM), par("Zh", DI, DS), par("Zc", DI)
    for b in range(B):
        par(f"nw_{b}", DM), par(f"Wx_{b}", DM, DI), par(f"Wz_{b}", DM, DI)
        for i in range(4):
            par(f"cw{i}_{b}", DI)
        par(f"cb_{b}", DI), par(f"Wr_{b}", DI, R), par(f"WB_{b}", DI, DS), par(f"WC_{b}", DI, DS)
        par(f"Wdt_{b}", R, DI), par(f"bdt_{b}", DI), par(f"A_{b}", DI, DS), par(f"D_{b}", DI), par(f"Wo_{b}", DI, DM)
    lines += ["", f"def forward(u0: f32[{T}, {DM}]) -> f32[{T}, {DM}]:"]
    for b in range(B):
        lines += [f"    h{b} = Zh", f"    c1_{b} = Zc", f"    c2_{b} = Zc", f"    c3_{b} = Zc",
                  f"    scan h{b}, c1_{b}, c2_{b}, c3_{b} over ut in u{b}:",
                  f"        n = rmsnorm(ut) * nw_{b}",
                  f"        xi = n @ Wx_{b}",
                  f"        z = n @ Wz_{b}",
                  f"        xc = c3_{b} * cw0_{b} + c2_{b} * cw1_{b} + c1_{b} * cw2_{b} + xi * cw3_{b} + cb_{b}",
                  f"        c3_{b} = c2_{b}",
                  f"        c2_{b} = c1_{b}",
                  f"        c1_{b} = xi",
                  "        xs = silu(xc)",
                  f"        dt = softplus((xs @ Wr_{b}) @ Wdt_{b} + bdt_{b})",
                  f"        bt = xs @ WB_{b}",
                  f"        ct = xs @ WC_{b}",
                  f"        e = exp(-(reshape(dt, {DI}, 1) * A_{b}))",
                  f"        h{b} = e * h{b} + (1 - e) / A_{b} * outer(xs, bt)",
                  f"        y = h{b} @ ct + D_{b} * xs",
                  f"        emit u{b + 1} = ut + (y * silu(z)) @ Wo_{b}"]
    lines.append(f"    return rmsnorm(u{B}) * nf")
    path = os.path.join(outdir, "ssm.tg")
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return path



class SsmSample:
    """Config 3 on the reference's VM: the program of emit_ssm at T steps per sequence, int8
    RTN (`tgc quantize --bits 8 --min-size 1`: every projection), one sequence per host
    core. A scan step costs the same at every position, so T steps stand for any length."""

    def __init__(self, T: int, seed: int = 3):
        import time
        t0 = time.perf_counter()
        self.T = T
        self.dir = tempfile.TemporaryDirectory(prefix="tg_refvm_")
        self.R = lib()
        path = emit_ssm(SSM3, ssm_weights(SSM3, seed), self.dir.name, T)
        self.mod = self.R.ref_vm_load(path.encode(), 8, 0, 1, 0)
        self.threads = os.cpu_count() or 1
        self.setup_s = time.perf_counter() - t0

    def run(self) -> float:
        sec = (C.c_double * 1)()
        self.threads = self.R.ref_vm_run(self.mod, self.threads, 1, sec)
        return sec[0]

    def close(self):
        self.dir.cleanup()


class Qwen3Pieces:
    """The pieces of one config's forward: written, loaded and quantized by the reference
    once (setup, not timed), then timed on demand."""

    def __init__(self, T: int, bits: int, gptq: bool, seed: int):
        import time
        t0 = time.perf_counter()
        self.T, self.bits, self.gptq, self.seed = T, bits, gptq, seed
        self.dir = tempfile.TemporaryDirectory(prefix="tg_refvm_")
        self.R = lib()
        self.mods = {}
        for i, p in enumerate(PIECES):
            path = emit_piece(p, T, os.path.join(self.dir.name, p), seed + i)
            self.mods[p] = self.R.ref_vm_load(path.encode(), bits, 1 if gptq and p != "head" else 0,
                                              QWEN3["head_dim"] ** 2 + 1, 256)
        self.threads = os.cpu_count() or 1
        self.times = {p: [] for p in PIECES}
        self.setup_s = time.perf_counter() - t0

    def run(self, piece: str) -> float:
        """The piece on one row per host core, all at once: its wall time (seconds)."""
        sec = (C.c_double * 1)()
        self.threads = self.R.ref_vm_run(self.mods[piece], self.threads, 1, sec)
        self.times[piece].append(sec[0])
        return sec[0]

    def forward_seconds(self) -> float:
        """One full forward on every core at once, from the medians of the pieces timed so far."""
        med = {p: statistics.median(v) for p, v in self.times.items()}
        return QWEN3["layers"] * (med["attn"] + med["gate"] + med["down"]) + (self.T / HEAD_ROWS) * med["head"]

    def close(self):
        self.dir.cleanup()
