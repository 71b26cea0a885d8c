"""tg_cuda_matmul_qb_noalloc: the small-batch x @ W GEMV for callers that may not
allocate device memory (GPU).

It must agree with tg_cuda_matmul_q, the entry point that allocates its scratch,
and with the CPU oracle's x @ W (the reference's tg_matmul_qb arithmetic), within
the float tolerance of the other GPU tests (1e-3 relative + 1e-4 absolute), on two
calls in a row: the second call reuses the fixed scratch the first one left
behind. The large shapes make the fixed array decide the split count: m*n = 2^19
leaves room for two K splits where four CTAs per SM would want three, and
m*n = 2^20 fills the array to its last float with a single split. This file is
collected last so that a failure here never hides another test's result."""
import numpy as np
import pytest
import torch

from oracle import tgo
from technograd_b200 import _lib, tgir

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-3, 1e-4


def _case(rng, bits, m, k, n):
    codes = rng.integers(-8 if bits == 4 else -127, 8 if bits == 4 else 128, size=k * n)
    q = torch.from_numpy(np.ascontiguousarray(tgir.pack_codes(codes, bits))).cuda()
    s = torch.from_numpy((np.abs(rng.normal(0, 0.02, n)) / 7).astype(np.float32)).cuda()
    a = torch.from_numpy(rng.normal(0, 1, size=m * k).astype(np.float32)).cuda()
    return q, s, a


@pytest.mark.parametrize("bits,m,k,n", [(4, 1, 1024, 3072), (8, 5, 3072, 1024), (4, 8, 1024, 2048), (4, 3, 200, 24),
                                        (4, 8, 4096, 1 << 16), (4, 8, 1024, 1 << 17), (8, 1, 256, 1 << 20)])
def test_no_alloc_matches_allocating_entry_point(cuda, bits, m, k, n):
    L = _lib.lib()
    rng = np.random.default_rng(100 + m)
    want = torch.empty(m * n, device="cuda")
    got = [torch.full((m * n,), float("nan"), device="cuda") for _ in range(2)]
    for call in range(2):  # two calls in a row, fresh inputs each time
        q, s, a = _case(rng, bits, m, k, n)
        _lib.check(L.tg_cuda_matmul_q(1, want.data_ptr(), a.data_ptr(), q.data_ptr(), bits, s.data_ptr(), m, k, n, None))
        _lib.check(L.tg_cuda_matmul_qb_noalloc(got[call].data_ptr(), a.data_ptr(), q.data_ptr(), bits, s.data_ptr(), m, k,
                                               n, None))
        torch.cuda.synchronize()
        mine = got[call].cpu().numpy()
        np.testing.assert_allclose(mine, want.cpu().numpy(), rtol=RTOL, atol=ATOL)
        # the oracle: the reference's x @ W arithmetic on the CPU (threaded, bit-identical to the scalar form)
        oracle = np.zeros(m * n, np.float32)
        qh, sh, ah = q.cpu().numpy(), s.cpu().numpy(), a.cpu().numpy()
        tgo.tgo().tgo_matmul_qb_mt(tgo.f32p(oracle), tgo.f32p(ah), tgo.i8p(qh), bits, tgo.f32p(sh), m, k, n, 0)
        np.testing.assert_allclose(mine, oracle, rtol=RTOL, atol=ATOL)


def test_no_alloc_rejects_sizes_beyond_its_scratch(cuda):
    L = _lib.lib()
    buf = torch.zeros(16, device="cuda")
    p = buf.data_ptr()
    assert L.tg_cuda_matmul_qb_noalloc(p, p, p, 4, p, 9, 64, 64, None) == _lib.EINVAL      # batch above 8
    assert b"maximum of 8" in L.tg_cuda_error()
    assert L.tg_cuda_matmul_qb_noalloc(p, p, p, 4, p, 8, 64, 1 << 18, None) == _lib.EINVAL  # m*n above 1,048,576
    assert b"exceeds" in L.tg_cuda_error()
