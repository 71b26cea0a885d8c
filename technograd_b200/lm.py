"""Decoder LMs of the Qwen3 import (examples/qwen3/import.py) over libtgcuda.

A model is a dict of the program's params by name, as import.py writes them:
E [V, D], LM [D, V], lnf, and per layer l: ln1_l, ln2_l, qn_l, kn_l,
Wq_l_h / Wo_l_h per query head, Wk_l_j / Wv_l_j per KV head, Wg_l, Wu_l, Wd_l.
Linear weights are quantized per output column (axis 1, x @ W, src/ops.c:310-320)
as `tgc quantize` does; `Quantized` keeps them in the reference packing, and
`desc()` concatenates the per-head params along the output axis for the C ABI.
"""
from __future__ import annotations

import ctypes as C
import gzip
import math

import numpy as np

from . import _lib, tgir

QWEN3_0_6B = dict(layers=28, hidden=1024, nq=16, nkv=8, head_dim=128, ffn=3072, vocab=151936, theta=1e6)


class QParam:
    """One quantized param in the reference format: codes (packed) and one scale per channel."""

    def __init__(self, q: np.ndarray, s: np.ndarray, bits: int, shape: tuple):
        self.q, self.s, self.bits, self.shape = np.ascontiguousarray(q, np.int8), np.ascontiguousarray(s, np.float32), bits, shape

    def codes(self) -> np.ndarray:
        n = self.shape[0] * self.shape[1]
        return tgir.unpack_codes(self.q, self.bits, n).reshape(self.shape)


class Model:
    """A quantized Qwen3-structured program: f32 params plus QParams for the linear weights."""

    def __init__(self, cfg: dict, bits: int, f32: dict, q: dict):
        self.cfg, self.bits, self.f32, self.q = dict(cfg), bits, f32, q

    # ---- the C descriptor -------------------------------------------------------------
    def desc(self):
        c = self.cfg
        L, D, NQ, NKV, HD, FF, V = (c[k] for k in ("layers", "hidden", "nq", "nkv", "head_dim", "ffn", "vocab"))
        keep = []

        def f32p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return a.ctypes.data_as(_lib.FP)

        def qmat(q: np.ndarray, scales: np.ndarray):  # packed codes
            q = np.ascontiguousarray(q, np.int8)
            s = np.ascontiguousarray(scales, np.float32)
            keep.extend([q, s])
            m = _lib.QMat()
            m.q = q.ctypes.data_as(C.POINTER(C.c_byte))
            m.s = s.ctypes.data_as(_lib.FP)
            return m

        def packed_rows(p: QParam) -> np.ndarray | None:  # [rows, packed bytes per row], or None
            per = p.shape[1] * self.bits // 8
            if self.bits == 4 and p.shape[1] % 2:
                return None  # a row ends inside a byte
            return p.q[:p.shape[0] * per].reshape(p.shape[0], per)

        def cat(names, axis):  # per-head params joined along the column (1) or row (0) axis
            ps = [self.q[n] for n in names]
            s = np.concatenate([p.s for p in ps])
            rows = [packed_rows(p) for p in ps]
            if all(r is not None for r in rows):  # join the packed bytes as they are
                return qmat(np.concatenate(rows, axis=axis).ravel(), s)
            return qmat(tgir.pack_codes(np.concatenate([p.codes() for p in ps], axis=axis), self.bits), s)

        def cat_cols(names):  # per-head [D, HD] params -> [D, n*HD], scales concatenated
            return cat(names, 1)

        d = _lib.LmDesc()
        d.layers, d.hidden, d.nq, d.nkv, d.head_dim, d.ffn, d.vocab = L, D, NQ, NKV, HD, FF, V
        d.bits = self.bits
        d.eps = 1e-6
        d.attn_scale = float(np.float32(float(f"{1.0 / math.sqrt(HD):.9g}")))  # the program's printed constant
        d.rope_theta = float(c["theta"])
        d.embed = f32p(self.f32["E"])
        d.final_norm = f32p(self.f32["lnf"])
        d.lm_head = qmat(self.q["LM"].q, self.q["LM"].s)
        arrs = {k: (_lib.FP * L)() for k in ("ln1", "ln2", "qn", "kn")}
        mats = {k: (_lib.QMat * L)() for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")}
        for l in range(L):
            for k in ("ln1", "ln2", "qn", "kn"):
                arrs[k][l] = f32p(self.f32[f"{k}_{l}"])
            mats["wq"][l] = cat_cols([f"Wq_{l}_{h}" for h in range(NQ)])
            mats["wk"][l] = cat_cols([f"Wk_{l}_{j}" for j in range(NKV)])
            mats["wv"][l] = cat_cols([f"Wv_{l}_{j}" for j in range(NKV)])
            mats["wo"][l] = cat([f"Wo_{l}_{h}" for h in range(NQ)], 0)  # [NQ*HD, D], scales [NQ*D]
            for k, n in (("wg", "Wg"), ("wu", "Wu"), ("wd", "Wd")):
                mats[k][l] = qmat(self.q[f"{n}_{l}"].q, self.q[f"{n}_{l}"].s)
        for k, v in arrs.items():
            setattr(d, k, C.cast(v, _lib.FPP))
        for k, v in mats.items():
            setattr(d, k, C.cast(v, _lib.QP))
        keep.extend(list(arrs.values()) + list(mats.values()))
        return d, keep

    @classmethod
    def from_tgir(cls, path: str, cfg: dict) -> "Model":
        """A `tgc quantize`d Qwen3 program. A plain file is read through a memory map with
        its number lists parsed straight into arrays and the quantized params kept as their
        packed codes (tgir.load), so a full-size model loads in memory proportional to its
        codes; a .gz file is decompressed first."""
        if path.endswith(".gz"):
            with gzip.open(path, "rb") as f:
                m = tgir.read(f.read())
        else:
            m = tgir.load(path)
        f32, q, bits = {}, {}, 0
        for v in m.vals:
            if v.kind != _lib.PARAM:
                continue
            if v.qbits:
                if v.qaxis != 1:
                    raise ValueError(f"{v.name}: expected a column-quantized (x @ W) param")
                q[v.name] = QParam(v.q, v.qs, v.qbits, v.shape)
                bits = v.qbits
            else:
                f32[v.name] = v.data.reshape(v.shape)
        return cls(cfg, bits, f32, q)


def random_weights(cfg: dict, seed: int, norm_jitter: float = 0.0) -> dict:
    """Random-init weights of the architecture: linear weights ~ N(0, 0.02); norms 1 (+ jitter)."""
    rng = np.random.default_rng(seed)
    L, D, NQ, NKV, HD, FF, V = (cfg[k] for k in ("layers", "hidden", "nq", "nkv", "head_dim", "ffn", "vocab"))

    def g(*s):
        return rng.standard_normal(size=s, dtype=np.float32) * np.float32(0.02)

    def nw(n):
        return (1 + norm_jitter * rng.standard_normal(n)).astype(np.float32)

    w = {"E": g(V, D), "LM": g(D, V), "lnf": nw(D)}
    for l in range(L):
        w[f"ln1_{l}"], w[f"ln2_{l}"], w[f"qn_{l}"], w[f"kn_{l}"] = nw(D), nw(D), nw(HD), nw(HD)
        for h in range(NQ):
            w[f"Wq_{l}_{h}"], w[f"Wo_{l}_{h}"] = g(D, HD), g(HD, D)
        for j in range(NKV):
            w[f"Wk_{l}_{j}"], w[f"Wv_{l}_{j}"] = g(D, HD), g(D, HD)
        w[f"Wg_{l}"], w[f"Wu_{l}"], w[f"Wd_{l}"] = g(D, FF), g(D, FF), g(FF, D)
    return w


def is_linear(name: str) -> bool:
    return name == "LM" or name.split("_")[0] in ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd")


def quantize_rtn_device(w: dict, cfg: dict, bits: int) -> Model:
    """RTN-quantize every linear weight on the device (tg_cuda_quantize_rtn, bit-exact
    with src/quant.c's RTN), axis 1 as the program uses them."""
    import torch
    L = _lib.lib()
    f32, q = {}, {}
    for name, a in w.items():
        if not is_linear(name):
            f32[name] = a
            continue
        rows, cols = a.shape
        n = rows * cols
        dw = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        dq = torch.empty(n if bits == 8 else (n + 1) // 2, dtype=torch.int8, device="cuda")
        ds = torch.empty(cols, dtype=torch.float32, device="cuda")
        _lib.check(L.tg_cuda_quantize_rtn(dw.data_ptr(), rows, cols, 1, bits, dq.data_ptr(), ds.data_ptr(), None))
        q[name] = QParam(dq.cpu().numpy(), ds.cpu().numpy(), bits, (rows, cols))
    return Model(cfg, bits, f32, q)


class Engine:
    """A model loaded on the selected GPUs."""

    def __init__(self, model, max_seqs: int, max_len: int, gpus: int = 0, devices=None):
        _lib.init(gpus, devices)
        self.model = model
        d, keep = model.desc()
        h = C.c_void_p()
        _lib.check(_lib.lib().tg_cuda_lm_load(C.byref(d), max_seqs, max_len, C.byref(h)))
        del keep
        self.handle = h
        self.V = model.cfg["vocab"]

    def __del__(self):
        if getattr(self, "handle", None):
            _lib.lib().tg_cuda_lm_free(self.handle)
            self.handle = None

    def forward(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.float32)
        S, T = ids.shape
        out = np.empty((S, self.V), np.float32)
        _lib.check(_lib.lib().tg_cuda_lm_forward(self.handle, ids.ctypes.data, S, T, out.ctypes.data))
        return out

    def generate(self, ids: np.ndarray, nnew: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.float32)
        S, T = ids.shape
        tok = np.empty((S, nnew), np.int32)
        _lib.check(_lib.lib().tg_cuda_lm_generate(self.handle, ids.ctypes.data, S, T, nnew, tok.ctypes.data))
        return tok

    def profile(self, on: bool) -> None:
        _lib.check(_lib.lib().tg_cuda_lm_profile(self.handle, 1 if on else 0))

    def stats(self) -> dict:
        st = _lib.LmStats()
        _lib.check(_lib.lib().tg_cuda_lm_get_stats(self.handle, C.byref(st)))
        return {f: getattr(st, f) for f, _ in st._fields_}


class Gptq:
    """tg_cuda_gptq_prepare over seeded calibration rows (HOST memory)."""

    def __init__(self, calib: np.ndarray):
        calib = np.ascontiguousarray(calib, np.float32)
        h = C.c_void_p()
        _lib.check(_lib.lib().tg_cuda_gptq_prepare(calib.ctypes.data, calib.shape[0], calib.shape[1], C.byref(h)))
        self.h, self.K = h, calib.shape[1]

    def __del__(self):
        if getattr(self, "h", None):
            _lib.lib().tg_cuda_gptq_free(self.h)
            self.h = None


def quantize_device(w, bits: int, gptq: "Gptq | None", out_q=None, out_s=None):
    """Quantize a device f32 [in, out] matrix per output column (axis 1); GPTQ when a
    calibration of the right width is given and in <= 2048 (src/quant.c:346), else RTN."""
    import torch
    rows, cols = w.shape
    n = rows * cols
    q = out_q if out_q is not None else torch.empty(n if bits == 8 else (n + 1) // 2, dtype=torch.int8, device=w.device)
    s = out_s if out_s is not None else torch.empty(cols, dtype=torch.float32, device=w.device)
    L = _lib.lib()
    if gptq is not None and gptq.K == rows and rows <= 2048:
        _lib.check(L.tg_cuda_quantize_gptq(gptq.h, w.data_ptr(), rows, cols, 1, bits, q.data_ptr(), s.data_ptr(), None))
    else:
        _lib.check(L.tg_cuda_quantize_rtn(w.data_ptr(), rows, cols, 1, bits, q.data_ptr(), s.data_ptr(), None))
    return q, s


class DeviceBuilt:
    """A Qwen3-shaped model generated and quantized on the device, kept as the C
    descriptor's concatenated per-layer matrices (host copies for tg_cuda_lm_load).

    Random init: linear weights and the embedding ~ N(0, 0.02), norm weights 1.
    Calibration: 256 seeded N(0,1) rows per input width; every param of that width
    shares them. Per-head params are column blocks of one matrix (q/k/v) or row
    blocks quantized one head at a time (o_proj, whose scales are per head)."""

    def __init__(self, cfg: dict, bits: int = 4, method: str = "gptq", seed: int = 5, ncal: int = 256):
        import torch
        self.cfg, self.bits = dict(cfg), bits
        L, D, NQ, NKV, HD, FF, V = (cfg[k] for k in ("layers", "hidden", "nq", "nkv", "head_dim", "ffn", "vocab"))
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)

        def randn(*shape):
            return torch.randn(*shape, generator=gen, device="cuda", dtype=torch.float32) * 0.02

        cal = {}
        if method == "gptq":
            rng = np.random.default_rng(seed)
            cal = {K: Gptq(rng.standard_normal((ncal, K)).astype(np.float32)) for K in sorted({D, HD})}

        def quant(w):
            q, s = quantize_device(w, bits, cal.get(w.shape[0]))
            return q.cpu().numpy(), s.cpu().numpy()

        self.E = randn(V, D).cpu().numpy()
        self.lnf = np.ones(D, np.float32)
        self.lm = quant(randn(D, V))
        self.layers = []
        for _ in range(L):
            lay = {"ln1": np.ones(D, np.float32), "ln2": np.ones(D, np.float32), "qn": np.ones(HD, np.float32),
                   "kn": np.ones(HD, np.float32)}
            lay["wq"], lay["wk"], lay["wv"] = quant(randn(D, NQ * HD)), quant(randn(D, NKV * HD)), quant(randn(D, NKV * HD))
            wo = randn(NQ * HD, D)
            per = HD * D if bits == 8 else HD * D // 2
            qo = torch.empty(NQ * per, dtype=torch.int8, device="cuda")
            so = torch.empty(NQ * D, dtype=torch.float32, device="cuda")
            for h in range(NQ):
                quantize_device(wo[h * HD:(h + 1) * HD].contiguous(), bits, cal.get(HD), qo[h * per:(h + 1) * per],
                                so[h * D:(h + 1) * D])
            lay["wo"] = (qo.cpu().numpy(), so.cpu().numpy())
            lay["wg"], lay["wu"], lay["wd"] = quant(randn(D, FF)), quant(randn(D, FF)), quant(randn(FF, D))
            self.layers.append(lay)
        torch.cuda.synchronize()
        del cal

    def desc(self):
        c = self.cfg
        keep = []

        def f32p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return a.ctypes.data_as(_lib.FP)

        def qmat(qs):
            q, s = (np.ascontiguousarray(qs[0], np.int8), np.ascontiguousarray(qs[1], np.float32))
            keep.extend([q, s])
            m = _lib.QMat()
            m.q, m.s = q.ctypes.data_as(C.POINTER(C.c_byte)), s.ctypes.data_as(_lib.FP)
            return m

        L = c["layers"]
        d = _lib.LmDesc()
        d.layers, d.hidden, d.nq, d.nkv, d.head_dim, d.ffn, d.vocab = (c[k] for k in (
            "layers", "hidden", "nq", "nkv", "head_dim", "ffn", "vocab"))
        d.bits, d.eps = self.bits, 1e-6
        d.attn_scale = float(np.float32(float(f"{1.0 / math.sqrt(c['head_dim']):.9g}")))
        d.rope_theta = float(c["theta"])
        d.embed, d.final_norm, d.lm_head = f32p(self.E), f32p(self.lnf), qmat(self.lm)
        arrs = {k: (_lib.FP * L)() for k in ("ln1", "ln2", "qn", "kn")}
        mats = {k: (_lib.QMat * L)() for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")}
        for l, lay in enumerate(self.layers):
            for k in arrs:
                arrs[k][l] = f32p(lay[k])
            for k in mats:
                mats[k][l] = qmat(lay[k])
        for k, v in arrs.items():
            setattr(d, k, C.cast(v, _lib.FPP))
        for k, v in mats.items():
            setattr(d, k, C.cast(v, _lib.QP))
        keep.extend(list(arrs.values()) + list(mats.values()))
        return d, keep

