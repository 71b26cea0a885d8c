"""TGIR files of the Qwen3 program (TEST INFRASTRUCTURE ONLY).

Writes the quantized program examples/qwen3/import.py:90-132 emits, in the form the
reference's `tgc quantize` writes it (src/ir.c ir_write): the params in declaration order
(E, LM, lnf, cosT, sinT, Rot, mask, lastidx, then per layer ln1, ln2, qn, kn, the query
heads' Wq/Wo, the KV heads' Wk/Wv, Wg, Wu, Wd), the input ids, and the block the compiler
lowers the program to, instruction for instruction (tests/test_qwen3_tgir.py checks the
block against a TGIR the reference wrote, tests/golden/nano/q4.tgir.gz). It exists so the
tests can give the streaming loader a full-size quantized Qwen3 file (~0.6 G codes) without
running the reference's quantizer over 600 M weights: numbers are printed as ir_write
prints them (%.9g of the f32 value; integers as integers), the many ones through a token
table chunk by chunk.
"""
from __future__ import annotations

import math

import numpy as np


def _tok(x: float, integer: bool) -> bytes:
    return (("%d" % int(x)) if integer else ("%.9g" % float(x))).encode()


def _write_numbers(f, a, chunk: int = 1 << 22) -> None:
    """Writes the numbers of a, each preceded by spaces, as ir_write prints them (integers as
    integers, the rest %.9g of the f32 value). `a` is an array, or (index array, values):
    the numbers values[index], which a large param of few distinct values (the synthetic
    embedding) is given as. Integer arrays of a small range and indexed values go through
    a fixed-width token table, chunk by chunk, so memory stays bounded."""
    if isinstance(a, tuple):
        idx, vals = np.asarray(a[0]).ravel(), np.asarray(a[1], np.float32)
        toks = [_tok(v, False) for v in vals]
    else:
        a = np.asarray(a).ravel()
        integer = np.issubdtype(a.dtype, np.integer)
        if not integer or a.size == 0 or int(a.max()) - int(a.min()) >= 4096:
            if not integer:
                a = a.astype(np.float32)
            f.write(b"".join(b" " + _tok(x, integer) for x in a.tolist()))
            return
        lo = int(a.min())
        toks = [_tok(v, True) for v in range(lo, int(a.max()) + 1)]
        idx = a
    w = max(len(t) for t in toks) + 1
    table = np.full((len(toks), w), ord(" "), np.uint8)
    for i, t in enumerate(toks):
        table[i, w - len(t):] = np.frombuffer(t, np.uint8)
    for s in range(0, idx.size, chunk):
        part = idx[s:s + chunk]
        f.write(table[part if isinstance(a, tuple) else part.astype(np.int64) - lo].tobytes())


def _shape(shape) -> str:
    return "(f32" + "".join(f" {d}" for d in shape) + ")"


def tables(T: int, HD: int, theta: float) -> dict:
    """cosT, sinT, Rot, the causal mask and lastidx as import.py:74-86 writes them."""
    inv = theta ** (-(np.arange(0, HD, 2) / HD))
    ang = np.outer(np.arange(T), inv)
    rot = np.zeros((HD, HD), np.float32)
    for i in range(HD // 2):
        rot[i + HD // 2, i] = -1.0
        rot[i, i + HD // 2] = 1.0
    return {"cosT": np.concatenate([np.cos(ang), np.cos(ang)], axis=1).astype(np.float32),
            "sinT": np.concatenate([np.sin(ang), np.sin(ang)], axis=1).astype(np.float32), "Rot": rot,
            "mask": np.where(np.arange(T)[None, :] <= np.arange(T)[:, None], 0.0, -1e9).astype(np.float32),
            "lastidx": np.array([T - 1], np.float32)}


def param_names(cfg: dict) -> list:
    L, NQ, NKV = cfg["layers"], cfg["nq"], cfg["nkv"]
    names = ["E", "LM", "lnf", "cosT", "sinT", "Rot", "mask", "lastidx"]
    for l in range(L):
        names += [f"ln1_{l}", f"ln2_{l}", f"qn_{l}", f"kn_{l}"]
        for h in range(NQ):
            names += [f"Wq_{l}_{h}", f"Wo_{l}_{h}"]
        for j in range(NKV):
            names += [f"Wk_{l}_{j}", f"Wv_{l}_{j}"]
        names += [f"Wg_{l}", f"Wu_{l}", f"Wd_{l}"]
    return names


def param_shape(cfg: dict, name: str, T: int) -> tuple:
    D, HD, FF, V = cfg["hidden"], cfg["head_dim"], cfg["ffn"], cfg["vocab"]
    base = name.split("_")[0]
    return {"E": (V, D), "LM": (D, V), "lnf": (D,), "cosT": (T, HD), "sinT": (T, HD), "Rot": (HD, HD), "mask": (T, T),
            "lastidx": (1,), "ln1": (D,), "ln2": (D,), "qn": (HD,), "kn": (HD,), "Wq": (D, HD), "Wo": (HD, D),
            "Wk": (D, HD), "Wv": (D, HD), "Wg": (D, FF), "Wu": (D, FF), "Wd": (FF, D)}[base]


def block(cfg: dict, T: int, first: int) -> list:
    """The program's instructions as the compiler lowers them: (id, shape, op, args)."""
    L, D, NQ, NKV, HD, FF, V = (cfg[k] for k in ("layers", "hidden", "nq", "nkv", "head_dim", "ffn", "vocab"))
    grp = NQ // NKV
    scale = "%.9g" % float(np.float32(1.0 / math.sqrt(HD)))
    out = []
    nxt = [first]

    def op(shape, name, *args):
        v = f"%{nxt[0]}"
        nxt[0] += 1
        out.append((v, shape, name, args))
        return v

    def rotary(x, w):  # rotary(rmsnorm(x) * w) of import.py:96-97,104,108
        b = op((T, HD), "rmsnorm", x)
        c = op((T, HD), "mul", b, w)
        d = op((T, HD), "mul", c, "cosT")
        e = op((T, HD), "matmul", c, "Rot")
        f = op((T, HD), "mul", e, "sinT")
        return op((T, HD), "add", d, f)

    h = op((T, D), "take", "E", "ids")
    for l in range(L):
        n = op((T, D), "mul", op((T, D), "rmsnorm", h), f"ln1_{l}")
        k, v = [], []
        for j in range(NKV):
            k.append(rotary(op((T, HD), "matmul", n, f"Wk_{l}_{j}"), f"kn_{l}"))
            v.append(op((T, HD), "matmul", n, f"Wv_{l}_{j}"))
        heads = []
        for hh in range(NQ):
            j = hh // grp
            q = rotary(op((T, HD), "matmul", n, f"Wq_{l}_{hh}"), f"qn_{l}")
            s = op((T, T), "matmul", q, op((HD, T), "transpose", k[j]))
            s = op((T, T), "add", op((T, T), "mul", s, op((), "const", scale)), "mask")
            o = op((T, HD), "matmul", op((T, T), "softmax", s), v[j])
            heads.append(op((T, D), "matmul", o, f"Wo_{l}_{hh}"))
        acc = heads[0]
        for x in heads[1:]:
            acc = op((T, D), "add", acc, x)
        h = op((T, D), "add", h, acc)
        n = op((T, D), "mul", op((T, D), "rmsnorm", h), f"ln2_{l}")
        g = op((T, FF), "silu", op((T, FF), "matmul", n, f"Wg_{l}"))
        u = op((T, FF), "matmul", n, f"Wu_{l}")
        h = op((T, D), "add", h, op((T, D), "matmul", op((T, FF), "mul", g, u), f"Wd_{l}"))
    r = op((T, D), "mul", op((T, D), "rmsnorm", h), "lnf")
    lg = op((T, V), "matmul", r, "LM")
    op((V,), "reshape", op((1, V), "take", lg, "lastidx"))
    return out


def write(path: str, cfg: dict, T: int, f32: dict, quant: dict) -> None:
    """f32: name -> values, or (index array, values) (E, lnf and the per-layer norms; the
    tables are made here unless given); quant: name -> (codes [rows*cols] as integers, scales [channels], bits), every
    linear weight quantized per output column (axis 1), as `tgc quantize` leaves them."""
    tab = tables(T, cfg["head_dim"], cfg["theta"])
    names = param_names(cfg)
    with open(path, "wb") as f:
        f.write(b"(tgir 1\n  (model qwen3)\n")
        for name in names:
            shape = param_shape(cfg, name, T)
            f.write(f"  (param {name} {_shape(shape)}\n".encode())
            if name in quant:
                codes, scales, bits = quant[name]
                f.write(f"    (quant {bits} 1\n      (scale".encode())
                _write_numbers(f, np.asarray(scales, np.float32))
                f.write(b")\n      (codes")
                _write_numbers(f, codes)
                f.write(b")))\n")
            else:
                vals = f32[name] if name in f32 else tab[name]
                f.write(b"    (data")
                _write_numbers(f, vals if isinstance(vals, tuple) else np.asarray(vals, np.float32))
                f.write(b"))\n")
        f.write(f"  (input ids {_shape((T,))})\n  (block\n".encode())
        for v, shape, name, args in block(cfg, T, len(names) + 1):
            inner = f"({name} {args[0]})" if name == "const" else f"({name} {' '.join(args)})"
            f.write(f"    ({v} {_shape(shape)} {inner})\n".encode())
        f.write(f"  )\n  (output %{len(names) + len(block(cfg, T, len(names) + 1))}))\n".encode())
