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


class _FakeHostLib:
    """tg_cuda_host_register / unregister stand-ins that record the ranges and fail on request."""

    def __init__(self, fail_register_at=None, fail_unregister=False):
        self.calls, self.fail_register_at, self.fail_unregister, self.live = 0, fail_register_at, fail_unregister, set()

    def tg_cuda_host_register(self, p, n):
        self.calls += 1
        if self.calls == self.fail_register_at:
            return _lib.EINVAL
        self.live.add(p)
        return _lib.OK

    def tg_cuda_host_unregister(self, p):
        self.live.discard(p)
        return _lib.EINVAL if self.fail_unregister else _lib.OK

    def tg_cuda_error(self):
        return b"fake failure"


@pytest.mark.parametrize("fail_register_at,fail_unregister", [(None, False), (2, False), (None, True)])
def test_host_registered_releases_every_range(monkeypatch, fail_register_at, fail_unregister):
    """No GPU needed: HostRegistered releases every range it registered, when a registration
    fails part way, when an unregistration fails, and when the block raises; a failing
    unregistration does not replace an exception leaving the block."""
    import numpy as np
    fake = _FakeHostLib(fail_register_at, fail_unregister)
    monkeypatch.setattr(_lib, "lib", lambda: fake)
    arrays = [np.zeros(4, np.float32) for _ in range(3)]
    if fail_register_at or fail_unregister:
        with pytest.raises(_lib.TgCudaError):
            with _lib.HostRegistered(*arrays):
                pass
    else:
        with _lib.HostRegistered(*arrays):
            assert len(fake.live) == 3
    assert not fake.live
    fake.calls, fake.fail_register_at = 0, None
    with pytest.raises(KeyError):
        with _lib.HostRegistered(*arrays):
            raise KeyError("inside the block")
    assert not fake.live
