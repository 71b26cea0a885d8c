"""Failure detection on the GPU without a GPU fault: every tcgen05 kernel's mbarrier waits
are bounded; here a kernel waits on a barrier that nothing arrives on, with a short
limit, and must give up, report the timeout in its status word and leave the context
usable (tg_cuda_selftest_wait)."""
import ctypes as C

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import _lib, tgir

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives(cuda):
    status = C.c_int(-1)
    rc = cuda.tg_cuda_selftest_wait(2_000_000, C.byref(status))  # ~1 ms of SM cycles
    assert rc == _lib.EDEVICE, cuda.tg_cuda_error().decode()
    assert status.value == 1  # ST_TIMEOUT_FULL
    assert b"gave up" in cuda.tg_cuda_error()
    # the context still runs kernels: a small tensor-core GEMM against the oracle
    import torch
    rng = np.random.default_rng(9)
    m, k, n = 256, 256, 64
    codes = rng.integers(-8, 8, size=m * k)
    q = tgir.pack_codes(codes, 4)
    s = (np.abs(rng.normal(0, 0.02, size=m)) / 7).astype(np.float32)
    b = rng.normal(size=k * n).astype(np.float32)
    dq, ds, db = (torch.from_numpy(a).cuda() for a in (q, s, b))
    o = torch.empty((m, n), device="cuda")
    _lib.check(cuda.tg_cuda_matmul_q(0, o.data_ptr(), db.data_ptr(), dq.data_ptr(), 4, ds.data_ptr(), m, k, n, None))
    torch.cuda.synchronize()
    want = tgo.matmul_q(tgo.tgo(), "tgo_", 0, b, q, 4, s, m, k, n)
    np.testing.assert_allclose(o.cpu().numpy(), want, rtol=1e-3, atol=1e-4)


def test_selftest_rejects_bad_limits(cuda):
    status = C.c_int(-1)
    assert cuda.tg_cuda_selftest_wait(0, C.byref(status)) == _lib.EINVAL
    assert cuda.tg_cuda_selftest_wait(10**12, C.byref(status)) == _lib.EINVAL
