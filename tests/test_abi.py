"""The C ABI: the library loads and exports every entry point include/tg_cuda.h
declares; calls that need a device fail cleanly without one."""
import ctypes as C
import os
import re

import pytest

from technograd_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_header_and_binding_agree():
    hdr = open(os.path.join(ROOT, "include", "tg_cuda.h")).read()
    declared = set(re.findall(r"\b(tg_cuda_\w+)\s*\(", hdr))
    assert declared == set(_lib.SYMBOLS)


def test_library_exports_every_symbol():
    L = _lib.lib()
    for name in _lib.SYMBOLS:
        assert hasattr(L, name), name


def test_op_numbering_matches_header():
    hdr = open(os.path.join(ROOT, "include", "tg_cuda.h")).read()
    body = hdr[hdr.index("TG_CUDA_OP_CONST"):hdr.index("TG_CUDA_OP_COUNT")]
    names = [n.lower() for n in re.findall(r"TG_CUDA_OP_(\w+)", body)]
    assert names == _lib.OPS


def test_no_device_is_an_error_not_a_crash():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = _lib.lib()
    rc = L.tg_cuda_init(0, None)
    assert rc == _lib.ENODEV
    assert L.tg_cuda_error()
    assert L.tg_cuda_ngpus() == 0


def test_host_register_checks_arguments_first():
    """No GPU needed: a NULL or empty range is EINVAL, a range before tg_cuda_init is
    ENODEV, an unknown pointer cannot be unregistered."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = _lib.lib()
    assert L.tg_cuda_host_register(None, 64) == _lib.EINVAL
    buf = (C.c_char * 64)()
    assert L.tg_cuda_host_register(C.addressof(buf), 0) == _lib.EINVAL
    assert L.tg_cuda_host_register(C.addressof(buf), 64) == _lib.ENODEV
    assert L.tg_cuda_host_unregister(C.addressof(buf)) == _lib.EINVAL
