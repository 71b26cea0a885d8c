"""ctypes binding of libtgcuda (include/tg_cuda.h).

The structures mirror the header field for field. Loading fails loudly when
the library is missing: the package has no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libtgcuda.so")

OK, EINVAL, ENODEV, ECUDA, EUNSUPPORTED, ENOMEM, EFAULT, EDEVICE = 0, -1, -2, -3, -4, -5, -6, -7

# enum Op of the reference (src/tg.h:68-112), the numbering of TG_CUDA_OP_*
OPS = ["const", "add", "sub", "mul", "div", "max", "min", "neg", "tanh", "relu", "sigmoid", "exp", "sqrt",
       "gelu", "silu", "softplus", "log", "matmul", "softmax", "rmsnorm", "sum", "mean", "transpose", "outer",
       "step", "spmm", "spmm_t", "spmm_dx", "active", "take", "take_t", "spmm_tc", "sin", "cos", "reshape",
       "floor", "sum_to", "topk", "memscan", "memscan_t", "sufmatch", "think", "scan"]
OP = {name: i for i, name in enumerate(OPS)}
PARAM, INPUT, TMP, STATE = 0, 1, 2, 3

# Every entry point include/tg_cuda.h declares.
SYMBOLS = ["tg_cuda_error", "tg_cuda_init", "tg_cuda_ngpus", "tg_cuda_selftest_wait", "tg_cuda_selftest_gemm", "tg_cuda_shutdown", "tg_cuda_matmul_q",
           "tg_cuda_matmul_qb_noalloc",
           "tg_cuda_quantize_rtn", "tg_cuda_gptq_prepare", "tg_cuda_quantize_gptq", "tg_cuda_gptq_free", "tg_cuda_load", "tg_cuda_batch", "tg_cuda_batch_device", "tg_cuda_free",
           "tg_cuda_host_register", "tg_cuda_host_unregister",
           "tg_cuda_model_jit", "tg_cuda_program_kernel", "tg_cuda_batcher_new", "tg_cuda_batcher_run",
           "tg_cuda_batcher_stats", "tg_cuda_batcher_free",
           "tg_cuda_lm_load", "tg_cuda_lm_forward", "tg_cuda_lm_generate", "tg_cuda_lm_free", "tg_cuda_lm_profile",
           "tg_cuda_lm_get_stats", "tg_cuda_ssm_load", "tg_cuda_ssm_forward", "tg_cuda_ssm_forward_device",
           "tg_cuda_ssm_free", "tg_cuda_ssm_profile", "tg_cuda_ssm_get_stats"]


class TgCudaError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"tg_cuda status {status}: {msg}")
        self.status = status


class Value(C.Structure):
    _fields_ = [("kind", C.c_int), ("rank", C.c_int), ("dim", C.c_int * 4), ("data", C.POINTER(C.c_float)),
                ("qbits", C.c_int), ("qaxis", C.c_int), ("q", C.POINTER(C.c_byte)), ("qs", C.POINTER(C.c_float)),
                ("index", C.c_int)]


class Scan(C.Structure):
    _fields_ = [("T", C.c_int), ("reverse", C.c_int), ("tid", C.c_int),
                ("nc", C.c_int), ("c", C.POINTER(C.c_int)), ("init", C.POINTER(C.c_int)), ("next", C.POINTER(C.c_int)),
                ("nx", C.c_int), ("x", C.POINTER(C.c_int)), ("xt", C.POINTER(C.c_int)),
                ("ny", C.c_int), ("y", C.POINTER(C.c_int)), ("ys", C.POINTER(C.c_int))]


class Ins(C.Structure):
    _fields_ = [("op", C.c_int), ("out", C.c_int), ("a", C.c_int * 3), ("na", C.c_int), ("k", C.c_float),
                ("init", C.c_int), ("maxit", C.c_int), ("eps", C.c_float), ("yield_", C.c_int), ("tid", C.c_int),
                ("halt", C.c_int), ("hthr", C.c_float), ("body", C.c_int), ("nbody", C.c_int), ("scan", C.c_int)]


class Program(C.Structure):
    _fields_ = [("nval", C.c_int), ("val", C.POINTER(Value)), ("nins", C.c_int), ("ins", C.POINTER(Ins)),
                ("ntop", C.c_int), ("nscan", C.c_int), ("scans", C.POINTER(Scan)), ("ninputs", C.c_int),
                ("inputs", C.POINTER(C.c_int)), ("output", C.c_int), ("nthink", C.c_int), ("nupd", C.c_int)]


class QMat(C.Structure):
    _fields_ = [("q", C.POINTER(C.c_byte)), ("s", C.POINTER(C.c_float))]


FP = C.POINTER(C.c_float)
FPP = C.POINTER(FP)
QP = C.POINTER(QMat)


class LmDesc(C.Structure):
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("nq", C.c_int), ("nkv", C.c_int), ("head_dim", C.c_int),
                ("ffn", C.c_int), ("vocab", C.c_int), ("bits", C.c_int), ("eps", C.c_float),
                ("attn_scale", C.c_float), ("rope_theta", C.c_double), ("embed", FP), ("final_norm", FP),
                ("lm_head", QMat), ("ln1", FPP), ("ln2", FPP), ("qn", FPP), ("kn", FPP),
                ("wq", QP), ("wk", QP), ("wv", QP), ("wo", QP), ("wg", QP), ("wu", QP), ("wd", QP)]


class SsmDesc(C.Structure):
    _fields_ = [("blocks", C.c_int), ("d_model", C.c_int), ("d_inner", C.c_int), ("d_state", C.c_int),
                ("dt_rank", C.c_int), ("bits", C.c_int), ("eps", C.c_float), ("final_norm", FP), ("norm", FPP),
                ("conv_w", FPP), ("conv_b", FPP), ("dt_b", FPP), ("d", FPP), ("a", FPP),
                ("w_x", QP), ("w_z", QP), ("w_r", QP), ("w_b", QP), ("w_c", QP), ("w_dt", QP), ("w_o", QP)]


class SsmStats(C.Structure):
    _fields_ = [("device_ms", C.c_double), ("launches", C.c_long), ("gemm_ms", C.c_double), ("gemm_flops", C.c_double),
                ("gemm_launches", C.c_long), ("scan_ms", C.c_double), ("scan_flops", C.c_double),
                ("scan_launches", C.c_long)]


class LmStats(C.Structure):
    _fields_ = [("device_ms", C.c_double), ("launches", C.c_long), ("attn_decode_ms", C.c_double),
                ("attn_decode_bytes", C.c_double), ("attn_decode_launches", C.c_long), ("attn_prefill_ms", C.c_double),
                ("attn_prefill_flops", C.c_double), ("gemm_ms", C.c_double), ("gemm_flops", C.c_double),
                ("gemm_launches", C.c_long), ("gemm_weight_bytes", C.c_double),
                ("decode_gemm_ms", C.c_double), ("decode_gemm_weight_bytes", C.c_double)]


_lib = None


def lib() -> C.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libtgcuda is not built ({LIB_PATH}); run __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        vp, i, l = C.c_void_p, C.c_int, C.c_long
        sigs = {
            "tg_cuda_error": ([], C.c_char_p),
            "tg_cuda_init": ([i, C.POINTER(i)], i),
            "tg_cuda_ngpus": ([], i),
            "tg_cuda_selftest_wait": ([C.c_longlong, C.POINTER(i)], i),
            "tg_cuda_selftest_gemm": ([i, C.POINTER(vp), i, C.POINTER(vp), i, i, C.POINTER(i), C.POINTER(i), i, i, i, i,
                                       vp, vp, vp, C.c_long, vp, vp, vp], i),
            "tg_cuda_shutdown": ([], None),
            "tg_cuda_matmul_q": ([i, vp, vp, vp, i, vp, i, i, i, vp], i),
            "tg_cuda_matmul_qb_noalloc": ([vp, vp, vp, i, vp, i, i, i, vp], i),
            "tg_cuda_quantize_rtn": ([vp, i, i, i, i, vp, vp, vp], i),
            "tg_cuda_gptq_prepare": ([vp, i, i, C.POINTER(vp)], i),
            "tg_cuda_quantize_gptq": ([vp, vp, i, i, i, i, vp, vp, vp], i),
            "tg_cuda_gptq_free": ([vp], None),
            "tg_cuda_load": ([C.POINTER(Program), C.POINTER(vp)], i),
            "tg_cuda_batch": ([vp, vp, l, i, vp, i, vp, i], i),
            "tg_cuda_batch_device": ([vp, vp, l, vp, vp, vp], i),
            "tg_cuda_free": ([vp], None),
            "tg_cuda_host_register": ([vp, C.c_size_t], i),
            "tg_cuda_host_unregister": ([vp], i),
            "tg_cuda_model_jit": ([vp, C.c_char_p, i], i),
            "tg_cuda_batcher_new": ([vp, i, i, C.POINTER(vp)], i),
            "tg_cuda_batcher_run": ([vp, vp, vp, vp], i),
            "tg_cuda_batcher_stats": ([vp, C.POINTER(l), C.POINTER(l)], i),
            "tg_cuda_batcher_free": ([vp], None),
            "tg_cuda_program_kernel": ([C.POINTER(Program), C.c_char_p, l, C.POINTER(l), i], i),
            "tg_cuda_lm_load": ([C.POINTER(LmDesc), i, i, C.POINTER(vp)], i),
            "tg_cuda_lm_forward": ([vp, vp, l, i, vp], i),
            "tg_cuda_lm_generate": ([vp, vp, l, i, i, vp], i),
            "tg_cuda_lm_free": ([vp], None),
            "tg_cuda_lm_profile": ([vp, i], i),
            "tg_cuda_lm_get_stats": ([vp, C.POINTER(LmStats)], i),
            "tg_cuda_ssm_load": ([C.POINTER(SsmDesc), i, i, C.POINTER(vp)], i),
            "tg_cuda_ssm_forward": ([vp, vp, l, i, vp], i),
            "tg_cuda_ssm_forward_device": ([vp, vp, l, i, vp], i),
            "tg_cuda_ssm_free": ([vp], None),
            "tg_cuda_ssm_profile": ([vp, i], i),
            "tg_cuda_ssm_get_stats": ([vp, C.POINTER(SsmStats)], i),
        }
        for name, (args, res) in sigs.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        raise TgCudaError(status, lib().tg_cuda_error().decode(errors="replace"))


def init(ngpus: int = 0, devices=None) -> int:
    L = lib()
    if devices:
        arr = (C.c_int * len(devices))(*devices)
        check(L.tg_cuda_init(len(devices), arr))
    else:
        check(L.tg_cuda_init(ngpus, None))
    return L.tg_cuda_ngpus()


class HostRegistered:
    """Page-locks numpy arrays for direct DMA by tg_cuda_batch for the length of a `with`
    block (tg_cuda_host_register / tg_cuda_host_unregister)."""

    def __init__(self, *arrays):
        self.arrays = [a for a in arrays if a is not None and a.nbytes]
        self.done = []

    def __enter__(self):
        try:
            for a in self.arrays:
                if not a.flags.c_contiguous:
                    raise ValueError("tg_cuda_host_register: the array must be C-contiguous")
                check(lib().tg_cuda_host_register(a.ctypes.data, a.nbytes))
                self.done.append(a)
        except BaseException as e:
            self.__exit__(type(e), e, e.__traceback__)  # releases what was registered, keeps e
            raise
        return self

    def __exit__(self, exc_type, exc, tb):
        # every range is released even if one fails; a failure is raised only when no other
        # exception is already leaving the block
        first = None
        while self.done:
            try:
                check(lib().tg_cuda_host_unregister(self.done.pop().ctypes.data))
            except TgCudaError as e:
                first = first or e
        if first is not None and exc_type is None:
            raise first
        return False
