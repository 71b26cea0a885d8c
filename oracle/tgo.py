"""ctypes access to the CPU oracle (TEST INFRASTRUCTURE ONLY).

libtgo.so is the C restatement of the reference arithmetic (oracle/tgo.c);
libtgref.so (optional, built only where the reference sources exist) is the
reference's own kernels and quantizer behind oracle/ref_harness.c. Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline leg import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TGO = os.path.join(HERE, "_build", "libtgo.so")
REF = os.path.join(HERE, "_ref", "libtgref.so")
REF_TGC = os.path.join(HERE, "_ref", "tgc")

_tgo = None
_ref = None

FP = C.POINTER(C.c_float)
BP = C.POINTER(C.c_byte)
DP = C.POINTER(C.c_double)


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def tgo() -> C.CDLL:
    global _tgo
    if _tgo is None:
        if not os.path.exists(TGO):
            build()
        L = C.CDLL(TGO)
        L.tgo_qget.argtypes = [BP, C.c_int, C.c_long]
        L.tgo_qget.restype = C.c_int
        for n in ("tgo_matmul",):
            getattr(L, n).argtypes = [FP, FP, FP, C.c_int, C.c_int, C.c_int]
        L.tgo_matmul_qa.argtypes = [FP, BP, C.c_int, FP, FP, C.c_int, C.c_int, C.c_int]
        L.tgo_matmul_qb.argtypes = [FP, FP, BP, C.c_int, FP, C.c_int, C.c_int, C.c_int]
        L.tgo_rmsnorm.argtypes = [FP, FP, C.c_int, C.c_int]
        L.tgo_softmax.argtypes = [FP, FP, C.c_int, C.c_int]
        L.tgo_unary.argtypes = [C.c_int, FP, FP, C.c_int]
        L.tgo_rand.argtypes = [C.c_uint, C.c_float, FP, C.c_long]
        L.tgo_quantize.argtypes = [FP, C.c_int, C.c_int, C.c_int, C.c_int, DP, BP, FP]
        L.tgo_quantize.restype = C.c_int
        L.tgo_hessian_add.argtypes = [DP, FP, C.c_int, C.c_int]
        L.tgo_program_arena.argtypes = [C.c_void_p]
        L.tgo_program_arena.restype = C.c_long
        L.tgo_program_run.argtypes = [C.c_void_p, FP, FP, C.POINTER(C.c_int), FP, FP]
        L.tgo_program_run.restype = C.c_int
        L.tgo_lm_forward.argtypes = [C.c_void_p, FP, C.c_int, FP]
        L.tgo_lm_forward.restype = C.c_int
        L.tgo_matmul_qb_mt.argtypes = [FP, FP, BP, C.c_int, FP, C.c_int, C.c_int, C.c_int, C.c_int]
        L.tgo_lm_forward_mt.argtypes = [C.c_void_p, FP, C.c_int, FP, C.c_int]
        L.tgo_lm_forward_mt.restype = C.c_int
        L.tgo_ssm_forward.argtypes = [C.c_void_p, FP, C.c_int, FP]
        L.tgo_ssm_forward.restype = C.c_int
        _tgo = L
    return _tgo


def ref():
    """The reference's own kernels, or None where oracle/_ref was not built."""
    global _ref
    if _ref is None and os.path.exists(REF):
        L = C.CDLL(REF)
        L.ref_matmul.argtypes = [FP, FP, FP, C.c_int, C.c_int, C.c_int]
        L.ref_matmul_qa.argtypes = [FP, BP, C.c_int, FP, FP, C.c_int, C.c_int, C.c_int]
        L.ref_matmul_qb.argtypes = [FP, FP, BP, C.c_int, FP, C.c_int, C.c_int, C.c_int]
        L.ref_rmsnorm.argtypes = [FP, FP, C.c_int, C.c_int]
        L.ref_softmax.argtypes = [FP, FP, C.c_int, C.c_int]
        L.ref_qget.argtypes = [BP, C.c_int, C.c_int]
        L.ref_quantize.argtypes = [FP, C.c_int, C.c_int, C.c_int, C.c_int, DP, BP, FP]
        _ref = L
    return _ref


def f32p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(FP)


def i8p(a: np.ndarray):
    assert a.dtype == np.int8 and a.flags.c_contiguous
    return a.ctypes.data_as(BP)


def matmul_q(lib, prefix: str, axis: int, act: np.ndarray, q: np.ndarray, bits: int, s: np.ndarray, m: int, k: int,
             n: int) -> np.ndarray:
    """tg_matmul_qa (axis 0: act is b [k, n]) or tg_matmul_qb (axis 1: act is a [m, k])."""
    o = np.zeros(m * n, np.float32)
    act = np.ascontiguousarray(act, np.float32).ravel()
    if axis == 0:
        getattr(lib, prefix + "matmul_qa")(f32p(o), i8p(q), bits, f32p(s), f32p(act), m, k, n)
    else:
        getattr(lib, prefix + "matmul_qb")(f32p(o), f32p(act), i8p(q), bits, f32p(s), m, k, n)
    return o.reshape(m, n)


def quantize(lib, prefix: str, w: np.ndarray, axis: int, bits: int, H: np.ndarray | None = None):
    rows, cols = w.shape
    C_, K = (rows, cols) if axis == 0 else (cols, rows)
    n = rows * cols
    q = np.zeros(n if bits == 8 else (n + 1) // 2, np.int8)
    s = np.zeros(C_, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    Hp = None
    if H is not None:
        H = np.ascontiguousarray(H, np.float64).copy()
        Hp = H.ctypes.data_as(DP)
    getattr(lib, prefix + "quantize")(f32p(w), rows, cols, axis, bits, Hp, i8p(q), f32p(s))
    return q, s


def program_run(prog, rows: np.ndarray, margins: bool = False):
    """Run a flattened program (technograd_b200.tgir.CProgram) row by row on the CPU.
    Returns (out, steps) or, with margins, (out, steps, min |delta - eps| per think loop)."""
    L = tgo()
    m = prog.module
    rows = np.ascontiguousarray(rows, np.float32).reshape(-1, m.per)
    arena = np.zeros(L.tgo_program_arena(C.addressof(prog.c)), np.float32)
    out = np.zeros((rows.shape[0], m.nout), np.float32)
    steps = np.zeros((rows.shape[0], max(m.nthink, 1)), np.int32)
    marg = np.zeros((rows.shape[0], max(m.nthink, 1)), np.float32)
    for r in range(rows.shape[0]):
        rc = L.tgo_program_run(C.addressof(prog.c), f32p(rows[r]), out[r].ctypes.data_as(FP),
                               steps[r].ctypes.data_as(C.POINTER(C.c_int)), f32p(arena), marg[r].ctypes.data_as(FP))
        if rc:
            raise RuntimeError("oracle: program uses an op the oracle does not implement")
    if margins:
        return out, steps[:, :m.nthink], marg[:, :m.nthink]
    return out, steps[:, :m.nthink]


def ssm_forward(desc, u: np.ndarray) -> np.ndarray:
    """tgo_ssm_forward over every sequence of u [S, T, d_model]."""
    L = tgo()
    u = np.ascontiguousarray(u, np.float32)
    out = np.zeros_like(u)
    for s in range(u.shape[0]):
        L.tgo_ssm_forward(C.addressof(desc), f32p(u[s]), u.shape[1], out[s].ctypes.data_as(FP))
    return out
