"""Stacked selective-SSM blocks (config 3) over libtgcuda.

A model is a dict of the program's params by name, as tests/golden/make_golden.py
emit_ssm writes them: nf, and per block b: nw_b, Wx_b, Wz_b, cw0_b..cw3_b, cb_b,
Wr_b, WB_b, WC_b, Wdt_b, bdt_b, A_b, D_b, Wo_b. The matrices are quantized per
output column (axis 1, x @ W, src/ops.c:310-320) as `tgc quantize --min-size 1`
does; the arithmetic is stated in include/tg_cuda.h (tg_cuda_ssm_desc).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib, tgir
from .lm import QParam

CONFIG3 = dict(blocks=4, d_model=256, d_inner=512, d_state=16, dt_rank=16)
MATS = ("Wx", "Wz", "Wr", "WB", "WC", "Wdt", "Wo")
FIELDS = dict(Wx="w_x", Wz="w_z", Wr="w_r", WB="w_b", WC="w_c", Wdt="w_dt", Wo="w_o")


def random_weights(cfg: dict, seed: int) -> dict:
    """Projections and conv weights ~ N(0, 0.02); norms 1; a = 1..d_state per channel
    (the positive decay rates exp(A_log) of Mamba's init); d = 1; dt bias = the inverse
    softplus of dt log-uniform in [1e-3, 1e-1]."""
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


class Model:
    """f32 params plus QParams for the seven matrices of every block."""

    def __init__(self, cfg: dict, bits: int, f32: dict, q: dict):
        self.cfg, self.bits, self.f32, self.q = dict(cfg), bits, f32, q

    @classmethod
    def from_tgir(cls, path: str, cfg: dict) -> "Model":
        with open(path, encoding="utf-8") as f:
            m = tgir.read(f.read())
        f32, q, bits = {}, {}, 0
        for v in m.vals:
            if v.kind != _lib.PARAM or not v.name:
                continue
            if v.qbits:
                if v.qaxis != 1:
                    raise ValueError(f"{v.name}: expected a column-quantized (x @ W) param")
                q[v.name] = QParam(v.q, v.qs, v.qbits, v.shape)
                bits = v.qbits
            else:
                f32[v.name] = v.data.reshape(v.shape)
        return cls(cfg, bits, f32, q)

    def desc(self):
        c = self.cfg
        B = c["blocks"]
        keep = []

        def f32p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return a.ctypes.data_as(_lib.FP)

        def qmat(p: QParam):
            qq, s = np.ascontiguousarray(p.q, np.int8), np.ascontiguousarray(p.s, np.float32)
            keep.extend([qq, s])
            m = _lib.QMat()
            m.q, m.s = qq.ctypes.data_as(C.POINTER(C.c_byte)), s.ctypes.data_as(_lib.FP)
            return m

        d = _lib.SsmDesc()
        d.blocks, d.d_model, d.d_inner, d.d_state, d.dt_rank = (c[k] for k in (
            "blocks", "d_model", "d_inner", "d_state", "dt_rank"))
        d.bits, d.eps = self.bits, 1e-6
        d.final_norm = f32p(self.f32["nf"])
        arrs = {k: (_lib.FP * B)() for k in ("norm", "conv_w", "conv_b", "dt_b", "d", "a")}
        mats = {k: (_lib.QMat * B)() for k in FIELDS.values()}
        for b in range(B):
            arrs["norm"][b] = f32p(self.f32[f"nw_{b}"])
            arrs["conv_w"][b] = f32p(np.stack([self.f32[f"cw{i}_{b}"] for i in range(4)]))
            arrs["conv_b"][b] = f32p(self.f32[f"cb_{b}"])
            arrs["dt_b"][b] = f32p(self.f32[f"bdt_{b}"])
            arrs["d"][b] = f32p(self.f32[f"D_{b}"])
            arrs["a"][b] = f32p(self.f32[f"A_{b}"])
            for n, field in FIELDS.items():
                mats[field][b] = qmat(self.q[f"{n}_{b}"])
        for k, v in arrs.items():
            setattr(d, k, C.cast(v, _lib.FPP))
        for k, v in mats.items():
            setattr(d, k, C.cast(v, _lib.QP))
        keep.extend(list(arrs.values()) + list(mats.values()))
        return d, keep


def quantize_rtn_device(w: dict, cfg: dict, bits: int) -> Model:
    """RTN-quantize the matrices on the device (tg_cuda_quantize_rtn, bit-exact with
    src/quant.c), per output column as the program uses them."""
    import torch
    L = _lib.lib()
    f32, q = {}, {}
    for name, a in w.items():
        if name.split("_")[0] not in MATS:
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

    def __init__(self, model: Model, max_seqs: int, chunk: int = 64, gpus: int = 0, devices=None):
        _lib.init(gpus, devices)
        self.model = model
        d, keep = model.desc()
        h = C.c_void_p()
        _lib.check(_lib.lib().tg_cuda_ssm_load(C.byref(d), max_seqs, chunk, C.byref(h)))
        del keep
        self.handle = h
        self.DM = model.cfg["d_model"]

    def __del__(self):
        if getattr(self, "handle", None):
            _lib.lib().tg_cuda_ssm_free(self.handle)
            self.handle = None

    def forward(self, u: np.ndarray) -> np.ndarray:
        """u [nseq, T, d_model] f32 (host) -> the program's output rows, same shape."""
        u = np.ascontiguousarray(u, np.float32)
        S, T, _ = u.shape
        out = np.empty_like(u)
        _lib.check(_lib.lib().tg_cuda_ssm_forward(self.handle, u.ctypes.data, S, T, out.ctypes.data))
        return out

    def forward_device(self, u_ptr: int, nseq: int, T: int, out_ptr: int) -> None:
        _lib.check(_lib.lib().tg_cuda_ssm_forward_device(self.handle, u_ptr, nseq, T, out_ptr))

    def profile(self, on: bool) -> None:
        _lib.check(_lib.lib().tg_cuda_ssm_profile(self.handle, 1 if on else 0))

    def stats(self) -> dict:
        st = _lib.SsmStats()
        _lib.check(_lib.lib().tg_cuda_ssm_get_stats(self.handle, C.byref(st)))
        return {f: getattr(st, f) for f, _ in st._fields_}
