"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference sources (it builds oracle/_ref with
oracle/Makefile): `python tests/golden/make_golden.py`. Every fixture is an
output of the reference's own code -- the `tgc` binary compiled from its
sources, or its runtime/tg_rt.h kernels and src/quant.c quantizer behind
oracle/ref_harness.c -- on seeded inputs. The tests compare the CPU oracle and
the CUDA library against these files; nothing at test time reads the reference.

Fixtures:
  latent_reasoner.{f32,q8}.tgir    `tgc ir` / `tgc quantize --bits 8 --min-size 1` of examples/latent_reasoner.tg
  lr_rows.csv                      2000 rows of f32[8], entries Bernoulli(0.5) (numpy default_rng(1))
  lr_{f32,q8}_out.csv              `tgc batch ... -j 1` text output: 4 values and the think steps per row
  ops.tgir, ops_expected.txt       tests/cases/ops.tg and the reference's own ops.expected
  kernels.npz                      tg_matmul_qa/qb, tg_matmul, rmsnorm, softmax on seeded shapes
  quant.npz                        quantize_param (RTN int8/int4 on both axes, GPTQ int4 with a Hessian)
  nano/                            a Qwen3-structured program (examples/qwen3/import.py layout) at toy
                                   sizes: weights, quantized TGIR (int8 RTN, int4 RTN, int4 GPTQ) and
                                   `tgc batch` logits of 4 sequences
  nano_ssm/                        a stacked selective-SSM program at toy sizes, quantized int8 and
                                   int4, with `tgc batch` outputs
  programs/                        `tgc ir` (or `tgc quantize`) of the reference's own test and
                                   example programs, seeded rows (the inputs tests/run.sh uses
                                   first) and `tgc batch` outputs: control flow (PROGRAMS), the
                                   sparse and memory ops (SPARSE_MEMORY), every other stateless one
                                   (SMALL)

`python make_golden.py PART ...` regenerates only the named parts (PARTS).
"""
from __future__ import annotations

import gzip
import math
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _reference() -> str:
    """The reference checkout: $TG_REFERENCE, else a `reference` directory beside this repository."""
    for d in (os.environ.get("TG_REFERENCE"), os.path.join(os.path.dirname(ROOT), "reference")):
        if d and os.path.exists(os.path.join(d, "src", "vm.c")):
            return d
    sys.exit("make_golden.py: set TG_REFERENCE to the reference checkout (no src/vm.c found)")


REF = _reference()
sys.path.insert(0, ROOT)

from oracle import tgo  # noqa: E402
from oracle.refvm import emit_ssm  # noqa: E402


def sh(*args, **kw) -> str:
    return subprocess.run([str(a) for a in args], check=True, capture_output=True, text=True, **kw).stdout


def latent_reasoner(tgc: str) -> None:
    src = os.path.join(REF, "examples", "latent_reasoner.tg")
    with open(os.path.join(HERE, "latent_reasoner.f32.tgir"), "w") as f:
        f.write(sh(tgc, "ir", src))
    q8 = os.path.join(HERE, "latent_reasoner.q8.tgir")
    sh(tgc, "quantize", src, "--bits", "8", "--min-size", "1", "-o", q8)
    rows = np.random.default_rng(1).integers(0, 2, size=(2000, 8)).astype(np.float32)
    rp = os.path.join(HERE, "lr_rows.csv")
    np.savetxt(rp, rows, fmt="%g", delimiter=",")
    for tag, model in (("f32", os.path.join(HERE, "latent_reasoner.f32.tgir")), ("q8", q8)):
        sh(tgc, "batch", model, rp, "-j", "1", "-o", os.path.join(HERE, f"lr_{tag}_out.csv"))


def ops(tgc: str) -> None:
    with open(os.path.join(HERE, "ops.tgir"), "w") as f:
        f.write(sh(tgc, "ir", os.path.join(REF, "tests", "cases", "ops.tg")))
    shutil.copy(os.path.join(REF, "tests", "cases", "ops.expected"), os.path.join(HERE, "ops_expected.txt"))


def kernels() -> None:
    R = tgo.ref()
    rng = np.random.default_rng(7)
    out = {}
    cases = [(0, 8, 5, 7, 1), (0, 4, 5, 7, 3), (0, 8, 33, 65, 2), (0, 4, 64, 96, 4), (0, 4, 17, 31, 1),
             (1, 8, 3, 9, 11), (1, 4, 2, 13, 17), (1, 4, 5, 64, 40), (1, 8, 1, 128, 24)]
    for idx, (axis, bits, m, k, n) in enumerate(cases):
        lim = 127 if bits == 8 else 8
        codes = rng.integers(-lim, lim if bits == 8 else 8, size=m * k if axis == 0 else k * n)
        if bits == 4:
            codes[0] = -8  # the int4 code TGIR cannot carry (src/ir.c:499-501)
        from technograd_b200.tgir import pack_codes
        q = np.ascontiguousarray(pack_codes(codes, bits))
        s = (np.abs(rng.normal(0, 0.02, size=m if axis == 0 else n)) / 7).astype(np.float32)
        act = rng.normal(0, 1, size=k * n if axis == 0 else m * k).astype(np.float32)
        o = tgo.matmul_q(R, "ref_", axis, act, q, bits, s, m, k, n)
        out[f"mq{idx}_meta"] = np.array([axis, bits, m, k, n])
        out[f"mq{idx}_codes"] = codes.astype(np.int8)
        out[f"mq{idx}_q"], out[f"mq{idx}_s"], out[f"mq{idx}_act"], out[f"mq{idx}_o"] = q, s, act, o
    a = rng.normal(0, 1, size=(7, 13)).astype(np.float32)
    b = rng.normal(0, 1, size=(13, 5)).astype(np.float32)
    o = np.zeros((7, 5), np.float32)
    R.ref_matmul(tgo.f32p(o), tgo.f32p(a), tgo.f32p(b), 7, 13, 5)
    out.update(mm_a=a, mm_b=b, mm_o=o)
    x = rng.normal(0, 3, size=(6, 37)).astype(np.float32)
    rn = np.zeros_like(x)
    sm = np.zeros_like(x)
    R.ref_rmsnorm(tgo.f32p(rn), tgo.f32p(x), 6, 37)
    R.ref_softmax(tgo.f32p(sm), tgo.f32p(x), 6, 37)
    out.update(row_x=x, rms_o=rn, softmax_o=sm)
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **out)


def quant() -> None:
    R = tgo.ref()
    rng = np.random.default_rng(11)
    out = {}
    cases = [("r8a0", 8, 0, (24, 40), False), ("r8a1", 8, 1, (40, 24), False), ("r4a0", 4, 0, (17, 33), False),
             ("r4a1", 4, 1, (33, 17), False), ("g4a1", 4, 1, (48, 20), True), ("g8a0", 8, 0, (12, 48), True),
             ("zero", 4, 0, (4, 16), False)]
    for name, bits, axis, shape, gptq in cases:
        w = rng.normal(0, 0.02, size=shape).astype(np.float32)
        if name == "zero":
            w[1] = 0.0  # an all-zero channel takes the 1e-8 scale (src/quant.c:188)
        H = None
        if gptq:
            K = shape[1 - axis]
            x = rng.normal(0, 1, size=(64, K)).astype(np.float32)
            H = np.zeros((K, K))
            tgo.tgo().tgo_hessian_add(H.ctypes.data_as(tgo.DP), tgo.f32p(x), 64, K)
            out[name + "_x"] = x
        q, s = tgo.quantize(R, "ref_", w, axis, bits, H)
        out[name + "_meta"] = np.array([bits, axis, *shape, int(gptq)])
        out[name + "_w"], out[name + "_q"], out[name + "_s"] = w, q, s
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **out)


# ---- a Qwen3-structured program at toy sizes ---------------------------------------------------
NANO = dict(layers=2, hidden=32, nq=4, nkv=2, head_dim=8, ffn=48, vocab=96, theta=1e6, T=6)


def nano_weights(cfg: dict, seed: int) -> dict:
    rng = np.random.default_rng(seed)
    D, L, NQ, NKV, HD, FF, V = (cfg[k] for k in ("hidden", "layers", "nq", "nkv", "head_dim", "ffn", "vocab"))
    g = lambda *s: rng.normal(0, 0.02, size=s).astype(np.float32)  # noqa: E731
    nw = lambda n: (1 + rng.normal(0, 0.1, size=n)).astype(np.float32)  # noqa: E731
    w = {"E": rng.normal(0, 1.0, size=(V, D)).astype(np.float32), "LM": g(D, V), "lnf": nw(D)}
    for l in range(L):
        w[f"ln1_{l}"], w[f"ln2_{l}"], w[f"qn_{l}"], w[f"kn_{l}"] = nw(D), nw(D), nw(HD), nw(HD)
        for h in range(NQ):
            w[f"Wq_{l}_{h}"], w[f"Wo_{l}_{h}"] = g(D, HD), g(HD, D)
        for j in range(NKV):
            w[f"Wk_{l}_{j}"], w[f"Wv_{l}_{j}"] = g(D, HD), g(D, HD)
        w[f"Wg_{l}"], w[f"Wu_{l}"], w[f"Wd_{l}"] = g(D, FF), g(D, FF), g(FF, D)
    return w


def emit_qwen3(cfg: dict, w: dict, outdir: str, T: int) -> str:
    """The program examples/qwen3/import.py:51-131 emits, for random weights: per-head rank-2
    matmuls, rotate-half RoPE through cos/sin tables and a Rot matrix, a -1e9 causal mask, the
    LM head on every row and take(lastidx)."""
    D, L, NQ, NKV, HD, FF, V = (cfg[k] for k in ("hidden", "layers", "nq", "nkv", "head_dim", "ffn", "vocab"))
    os.makedirs(os.path.join(outdir, "w"), exist_ok=True)
    tables = {}
    inv = cfg["theta"] ** (-(np.arange(0, HD, 2) / HD))
    ang = np.outer(np.arange(T), inv)
    tables["cosT"] = np.concatenate([np.cos(ang), np.cos(ang)], axis=1)
    tables["sinT"] = np.concatenate([np.sin(ang), np.sin(ang)], axis=1)
    rot = np.zeros((HD, HD), np.float32)
    for i in range(HD // 2):
        rot[i + HD // 2, i] = -1.0
        rot[i, i + HD // 2] = 1.0
    tables["Rot"] = rot
    tables["mask"] = np.where(np.arange(T)[None, :] <= np.arange(T)[:, None], 0.0, -1e9)
    tables["lastidx"] = np.array([T - 1], np.float32)
    for name, arr in list(w.items()) + list(tables.items()):
        np.asarray(arr, dtype="<f4").tofile(os.path.join(outdir, "w", name + ".bin"))
    lines = ["model qwen3", ""]

    def par(name, *shape):
        lines.append(f'param {name} : f32[{", ".join(map(str, shape))}] = file("w/{name}.bin")')

    par("E", V, D), par("LM", D, V), par("lnf", D), par("cosT", T, HD), par("sinT", T, HD)
    par("Rot", HD, HD), par("mask", T, T), par("lastidx", 1)
    for l in range(L):
        par(f"ln1_{l}", D), par(f"ln2_{l}", D), par(f"qn_{l}", HD), par(f"kn_{l}", HD)
        for h in range(NQ):
            par(f"Wq_{l}_{h}", D, HD), par(f"Wo_{l}_{h}", HD, D)
        for j in range(NKV):
            par(f"Wk_{l}_{j}", D, HD), par(f"Wv_{l}_{j}", D, HD)
        par(f"Wg_{l}", D, FF), par(f"Wu_{l}", D, FF), par(f"Wd_{l}", FF, D)
    lines += ["", f"def rotary(x: f32[{T}, {HD}]) -> f32[{T}, {HD}]:",
              "    return x * cosT + (x @ Rot) * sinT", "",
              f"def forward(ids: f32[{T}]) -> f32[{V}]:", "    h = take(E, ids)"]
    grp = NQ // NKV
    scale = 1.0 / math.sqrt(HD)
    for l in range(L):
        lines.append(f"    n = rmsnorm(h) * ln1_{l}")
        for j in range(NKV):
            lines.append(f"    k{j} = rotary(rmsnorm(n @ Wk_{l}_{j}) * kn_{l})")
            lines.append(f"    v{j} = n @ Wv_{l}_{j}")
        terms = []
        for h in range(NQ):
            j = h // grp
            lines.append(f"    q{h} = rotary(rmsnorm(n @ Wq_{l}_{h}) * qn_{l})")
            lines.append(f"    s{h} = softmax((q{h} @ transpose(k{j})) * {scale:.9g} + mask)")
            lines.append(f"    o{h} = (s{h} @ v{j}) @ Wo_{l}_{h}")
            terms.append(f"o{h}")
        lines.append(f"    h = h + ({' + '.join(terms)})")
        lines.append(f"    n = rmsnorm(h) * ln2_{l}")
        lines.append(f"    h = h + (silu(n @ Wg_{l}) * (n @ Wu_{l})) @ Wd_{l}")
    lines.append("    logits = (rmsnorm(h) * lnf) @ LM")
    lines.append(f"    return reshape(take(logits, lastidx), {V})")
    path = os.path.join(outdir, "qwen3.tg")
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return path


def nano(tgc: str) -> None:
    cfg = NANO
    T = cfg["T"]
    out = os.path.join(HERE, "nano")
    os.makedirs(out, exist_ok=True)
    w = nano_weights(cfg, 4)
    rng = np.random.default_rng(5)
    ids = rng.integers(0, cfg["vocab"], size=(4, T)).astype(np.float32)
    calib = rng.integers(0, cfg["vocab"], size=(16, T)).astype(np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        prog = emit_qwen3(cfg, w, tmp, T)
        np.savetxt(os.path.join(tmp, "ids.csv"), ids, fmt="%d", delimiter=",")
        np.savetxt(os.path.join(tmp, "calib.csv"), calib, fmt="%d", delimiter=",")
        minsz = str(cfg["head_dim"] ** 2 + 1)  # Rot (HD x HD) stays f32, every linear weight is quantized
        variants = {"q8": ["--bits", "8"], "q4": ["--bits", "4"],
                    "q4gptq": ["--bits", "4", "--method", "gptq", "--calib", os.path.join(tmp, "calib.csv")]}
        for tag, flags in variants.items():
            qp = os.path.join(tmp, f"{tag}.tgir")
            sh(tgc, "quantize", prog, "--min-size", minsz, *flags, "-o", qp)
            with open(qp, "rb") as f, open(os.path.join(out, f"{tag}.tgir.gz"), "wb") as raw:
                with gzip.GzipFile(fileobj=raw, mode="wb", mtime=0) as g:
                    g.write(f.read())
            sh(tgc, "batch", qp, os.path.join(tmp, "ids.csv"), "-j", "1", "-o", os.path.join(out, f"{tag}_logits.csv"))
        shutil.copy(os.path.join(tmp, "ids.csv"), os.path.join(out, "ids.csv"))
        with open(os.path.join(out, "config.txt"), "w") as f:
            f.write(" ".join(f"{k}={v}" for k, v in cfg.items()) + "\n")


# ---- stacked selective-SSM blocks (config 3) at toy sizes -------------------------------------
NANO_SSM = dict(blocks=2, d_model=16, d_inner=32, d_state=4, dt_rank=4, T=10)


def ssm_weights(cfg: dict, seed: int) -> dict:
    """Projections, conv weights ~ N(0, 0.02) (the config's init); norms 1 + N(0, 0.1) so they
    matter; a = 1..d_state per channel (a positive decay rate, as exp(A_log) of Mamba's
    init); d = 1; the dt bias the inverse softplus of dt log-uniform in [1e-3, 1e-1]."""
    rng = np.random.default_rng(seed)
    B, DM, DI, DS, R = (cfg[k] for k in ("blocks", "d_model", "d_inner", "d_state", "dt_rank"))
    g = lambda *s: rng.normal(0, 0.02, size=s).astype(np.float32)  # noqa: E731
    w = {"nf": (1 + rng.normal(0, 0.1, size=DM)).astype(np.float32)}
    for b in range(B):
        w[f"nw_{b}"] = (1 + rng.normal(0, 0.1, size=DM)).astype(np.float32)
        w[f"Wx_{b}"], w[f"Wz_{b}"] = g(DM, DI), g(DM, DI)
        for i in range(4):
            w[f"cw{i}_{b}"] = g(DI)
        w[f"cb_{b}"] = g(DI)
        w[f"Wr_{b}"], w[f"WB_{b}"], w[f"WC_{b}"] = g(DI, R), g(DI, DS), g(DI, DS)
        w[f"Wdt_{b}"] = g(R, DI)
        dt = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), size=DI))
        w[f"bdt_{b}"] = (dt + np.log(-np.expm1(-dt))).astype(np.float32)  # softplus^-1(dt)
        w[f"A_{b}"] = np.tile(np.arange(1, DS + 1, dtype=np.float32), (DI, 1))
        w[f"D_{b}"] = np.ones(DI, np.float32)
        w[f"Wo_{b}"] = g(DI, DM)
    return w


def nano_ssm(tgc: str) -> None:
    cfg = NANO_SSM
    T = cfg["T"]
    out = os.path.join(HERE, "nano_ssm")
    os.makedirs(out, exist_ok=True)
    w = ssm_weights(cfg, 6)
    rows = np.round(np.random.default_rng(7).normal(0, 1, size=(6, T * cfg["d_model"])), 4).astype(np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        prog = emit_ssm(cfg, w, tmp, T)
        np.savetxt(os.path.join(tmp, "u.csv"), rows, fmt="%.9g", delimiter=",")
        for tag, flags in (("q8", ["--bits", "8"]), ("q4", ["--bits", "4"])):
            qp = os.path.join(tmp, f"{tag}.tgir")
            sh(tgc, "quantize", prog, "--min-size", "1", *flags, "-o", qp)
            shutil.copy(qp, os.path.join(out, f"{tag}.tgir"))
            sh(tgc, "batch", qp, os.path.join(tmp, "u.csv"), "-j", "1", "-o", os.path.join(out, f"{tag}_out.csv"))
        shutil.copy(os.path.join(tmp, "u.csv"), os.path.join(out, "u.csv"))
        with open(os.path.join(out, "config.txt"), "w") as f:
            f.write(" ".join(f"{k}={v}" for k, v in cfg.items()) + "\n")


# The reference's control-flow test programs: scan carries and stacked outputs, think
# loops (`until` and learned halting), gradients through loops (lowered into the IR by
# the compiler), and rope + windowed attention. name -> (source, rows, value range)
PROGRAMS = {
    "scan": ("tests/scan/scan.tg", 300, 2.0),
    "halt": ("tests/think/halt.tg", 400, 3.0),
    "nested_grad": ("tests/scan/nested_grad.tg", 300, 1.0),
    "window": ("tests/attn/window.tg", 200, 1.5),
}
# the inputs tests/run.sh:45 runs these programs on, prepended to the random rows
RUN_SH_ROWS = {
    "scan": [[1, 2, 3, 4, 5, 6, 7, 8, 1, 0.5, -1, 2]],
    "halt": [[1, 1], [0, 0]],
    "nested_grad": [[0.1, 0.2, 0.3, -0.4, 0.5, 0.1, -0.2, 0.3]],
}


def programs(tgc: str) -> None:
    out = os.path.join(HERE, "programs")
    os.makedirs(out, exist_ok=True)
    for name, (src, n, span) in PROGRAMS.items():
        ir = os.path.join(out, f"{name}.tgir")
        with open(ir, "w") as f:
            f.write(sh(tgc, "ir", os.path.join(REF, src)))
        from technograd_b200 import tgir
        per = tgir.load(ir).per
        rng = np.random.default_rng(sum(map(ord, name)))
        rows = rng.uniform(-span, span, size=(n, per)).astype(np.float32)
        rows = np.round(rows, 3)  # text rows that read back exactly as the same f32
        if name in RUN_SH_ROWS:
            rows = np.concatenate([np.array(RUN_SH_ROWS[name], np.float32), rows])
        rp = os.path.join(out, f"{name}_rows.csv")
        np.savetxt(rp, rows, fmt="%.9g", delimiter=",")
        sh(tgc, "batch", ir, rp, "-j", "1", "-o", os.path.join(out, f"{name}_out.csv"))


# Programs of the reference's tests with the ops of the sparse and memory models: name ->
# (source, rows, how rows are drawn, quantize flags or None for `tgc ir`)
SPARSE_MEMORY = {
    "topk": ("tests/memory/topk.tg", 200, "ties", None),
    "topk_pad": ("tests/memory/topk_pad.tg", 100, "ties", None),
    "memscan": ("tests/memory/scan.tg", 200, "uniform", None),
    "sufmatch": ("tests/memory/sufmatch.tg", 200, "tokens", None),
    "mlp_f32": ("tests/quant/mlp.tg", 300, "sparse", None),
    "mlp_q8": ("tests/quant/mlp.tg", 300, "sparse", ["--bits", "8"]),
    "mlp_q4": ("tests/quant/mlp.tg", 300, "sparse", ["--bits", "4"]),
    "memscan_grad": ("tests/memory/scan_grad.tg", 200, "uniform", None),
    "memscan4": ("tests/memory/scan4.tg", 200, "uniform", None),
    "broadcast": ("tests/native/broadcast.tg", 200, "uniform", None),
}
# tests/run.sh:33-48: the inputs the reference's own suite runs these programs on
SPARSE_MEMORY_ROWS = {
    "topk": [[0, 5, 3, 4, -1, 2, 0, 0, 0, 0, 0, 0, 6, 5, 4, 3, 2, 1]],
    "topk_pad": [[2, 3, 1]],
    "memscan": [list(np.round(np.arange(-1.1, 1.25, 0.1), 1))],
    "sufmatch": [[1, 5, 2, 6, 3, 5, 1, 6, 2, 5, 3, 6, 1, -1, 2, 5, 3, 6, 9, 7, 1, 6, 2, 5]],
    "memscan_grad": [list(np.round(np.arange(-1.1, 1.25, 0.1), 1))],
    "memscan4": [list(np.round(np.arange(-1.1, 1.25, 0.1), 1))],
    "broadcast": [[1, 2, 3, 0.5, -1, 2, 0] + list(np.round(np.arange(-1, 1.35, 0.1), 1))],
}


def sparse_memory(tgc: str) -> None:
    from technograd_b200 import tgir
    out = os.path.join(HERE, "programs")
    os.makedirs(out, exist_ok=True)
    for name, (src, n, kind, qflags) in SPARSE_MEMORY.items():
        ir = os.path.join(out, f"{name}.tgir")
        if qflags is None:
            with open(ir, "w") as f:
                f.write(sh(tgc, "ir", os.path.join(REF, src)))
        else:
            sh(tgc, "quantize", os.path.join(REF, src), *qflags, "-o", ir)
        m = tgir.load(ir)
        rng = np.random.default_rng(sum(map(ord, name)))
        if kind == "ties":  # small integers: many equal values, and a NaN now and then
            rows = rng.integers(-3, 4, size=(n, m.per)).astype(np.float32)
            rows[rng.uniform(size=rows.shape) < 0.05] = np.nan
        elif kind == "tokens":  # token ids with repeats and breaks (negative ids)
            rows = rng.integers(-1, 7, size=(n, m.per)).astype(np.float32)
        elif kind == "sparse":  # x f32[16], then 3 (index, value) pairs into a 64-row table
            rows = np.round(rng.uniform(-1.5, 1.5, size=(n, m.per)), 3).astype(np.float32)
            idx = rng.integers(-3, 68, size=(n, 3)).astype(np.float32) + np.round(rng.uniform(-0.45, 0.45, size=(n, 3)), 2)
            val = np.round(rng.uniform(-2, 2, size=(n, 3)), 3)
            val[rng.uniform(size=val.shape) < 0.15] = 0.0  # padding
            rows[:, 16::2], rows[:, 17::2] = idx, val
        else:
            rows = np.round(rng.uniform(-1.5, 1.5, size=(n, m.per)), 3).astype(np.float32)
        if name in SPARSE_MEMORY_ROWS:
            rows = np.concatenate([np.array(SPARSE_MEMORY_ROWS[name], np.float32), rows])
        rp = os.path.join(out, f"{name}_rows.csv")
        np.savetxt(rp, rows, fmt="%.9g", delimiter=",")
        sh(tgc, "batch", ir, rp, "-j", "1", "-o", os.path.join(out, f"{name}_out.csv"))


# The other stateless programs of the reference's tests and examples: name -> (source, rows,
# how rows are drawn). Imports and file() params are resolved by `tgc ir`.
SMALL = {
    "xor": ("examples/xor.tg", 100, "bits"),
    "newton": ("examples/newton.tg", 200, "positive"),
    "use_import": ("examples/use_import.tg", 200, "uniform"),
    "bcast": ("tests/bcast/broadcast.tg", 200, "uniform"),
    "file_param": ("tests/cases/file_param.tg", 200, "uniform"),
    "multi_input": ("tests/cases/multi_input.tg", 200, "uniform"),
    "nested": ("tests/cases/nested.tg", 200, "uniform"),
    "cycle": ("tests/imports/cycle.tg", 100, "uniform"),
    "diamond": ("tests/imports/diamond.tg", 100, "uniform"),
    "take_along": ("tests/memory/take_along.tg", 200, "take"),
    "native_matmul": ("tests/native/matmul.tg", 200, "uniform"),
}  # tests/par/wide.tg is left out: its TGIR (a large param for the parallel-matmul test) is 16 MB
# tests/run.sh:26-47,334,427-428: the inputs the reference's own suite runs them on (a
# program's inputs concatenated, as `tgc batch` reads a row)
SMALL_ROWS = {
    "xor": [[0, 0], [1, 0], [0, 1], [1, 1]],
    "newton": [[2, 9, 16]],
    "use_import": [[1, -1, 2, -2]],
    "bcast": [[0.1, -0.2, 0.3, 1, 2, -1, 0, 0, 0, -3, 0.5, 0.25]],
    "file_param": [[1, 2]],
    "multi_input": [[1, 2, 3, 0.5]],
    "nested": [[0.3, -0.7]],
    "cycle": [[10, 20]],
    "diamond": [[10, 20]],
    "take_along": [[1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 3, 0, -1, 1, 4, 2]],
    "native_matmul": [[1, 2, 3, 4, 5, 6, 7] + [round(0.1 * i, 1) for i in range(1, 36)] + [1, -1, 2, -2, 0.5, 0.5, 1, 2, 3]],
}


def small_programs(tgc: str) -> None:
    from technograd_b200 import tgir
    out = os.path.join(HERE, "programs")
    os.makedirs(out, exist_ok=True)
    for name, (src, n, kind) in SMALL.items():
        ir = os.path.join(out, f"{name}.tgir")
        with open(ir, "w") as f:
            f.write(sh(tgc, "ir", os.path.join(REF, src)))
        m = tgir.load(ir)
        rng = np.random.default_rng(sum(map(ord, name)))
        if kind == "bits":
            rows = rng.integers(0, 2, size=(n, m.per)).astype(np.float32)
        elif kind == "positive":  # square roots by a think loop: 0.001 .. 100
            rows = np.round(10 ** rng.uniform(-3, 2, size=(n, m.per)), 4).astype(np.float32)
        elif kind == "take":  # 12 values, then 6 indices, some out of range or fractional
            vals = np.round(rng.uniform(-5, 5, size=(n, 12)), 3)
            idx = rng.integers(-2, 7, size=(n, 6)) + np.round(rng.uniform(-0.45, 0.45, size=(n, 6)), 2)
            rows = np.concatenate([vals, idx], axis=1).astype(np.float32)
        else:
            rows = np.round(rng.uniform(-1.5, 1.5, size=(n, m.per)), 3).astype(np.float32)
        if name in SMALL_ROWS:
            rows = np.concatenate([np.array(SMALL_ROWS[name], np.float32), rows])
        rp = os.path.join(out, f"{name}_rows.csv")
        np.savetxt(rp, rows, fmt="%.9g", delimiter=",")
        sh(tgc, "batch", ir, rp, "-j", "1", "-o", os.path.join(out, f"{name}_out.csv"))


PARTS = {"latent_reasoner": latent_reasoner, "ops": ops, "kernels": kernels, "quant": quant, "nano": nano,
         "nano_ssm": nano_ssm, "programs": programs, "sparse_memory": sparse_memory, "small_programs": small_programs}


def main() -> None:
    """python make_golden.py [PART ...]: every fixture, or only the named parts."""
    tgo.build()
    tgc = tgo.REF_TGC
    if not os.path.exists(tgc) or tgo.ref() is None:
        sys.exit("oracle/_ref was not built: the reference sources are needed")
    for part in sys.argv[1:] or list(PARTS):
        if part not in PARTS:
            sys.exit(f"unknown part {part!r}; parts: {', '.join(PARTS)}")
        f = PARTS[part]
        f() if part in ("kernels", "quant") else f(tgc)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
