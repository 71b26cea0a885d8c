"""tg_cuda_matmul_q and tg_cuda_quantize_rtn against the oracle (GPU).

Tolerance for the float kernels: |gpu - oracle| <= 1e-4 + 1e-3 |oracle|
(north_star: 1e-3 relative / 1e-4 absolute of the reference's f32 dequant
path). The one-thread-per-output path and the quantizer are bit-exact."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from oracle import tgo
from technograd_b200 import tgir

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-3, 1e-4


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gpu_matmul_q(L, axis, act, q, bits, s, m, k, n):
    o = torch.empty(m * n, dtype=torch.float32, device="cuda")
    da, dq, ds = dev(act.astype(np.float32)), dev(q.view(np.int8)), dev(s.astype(np.float32))
    rc = L.tg_cuda_matmul_q(axis, o.data_ptr(), da.data_ptr(), dq.data_ptr(), bits, ds.data_ptr(), m, k, n, None)
    assert rc == 0, L.tg_cuda_error()
    torch.cuda.synchronize()
    return o.cpu().numpy().reshape(m, n)


def test_matmul_q_golden(cuda, golden):
    z = np.load(os.path.join(golden, "kernels.npz"))
    i = 0
    while f"mq{i}_meta" in z:
        axis, bits, m, k, n = (int(v) for v in z[f"mq{i}_meta"])
        o = gpu_matmul_q(cuda, axis, z[f"mq{i}_act"], z[f"mq{i}_q"], bits, z[f"mq{i}_s"], m, k, n)
        np.testing.assert_allclose(o, z[f"mq{i}_o"], rtol=RTOL, atol=ATOL, err_msg=f"case {i}")
        i += 1


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("axis,m,k,n", [
    (0, 4096, 4096, 1), (0, 4096, 4096, 16), (0, 1000, 512, 3), (0, 257, 96, 8), (0, 64, 4096, 256),
    (1, 1, 1024, 3072), (1, 5, 3072, 1024), (1, 8, 1024, 2048), (1, 3, 200, 24), (1, 300, 256, 512),
    (0, 33, 70, 5), (1, 7, 33, 31),
])
def test_matmul_q_vs_oracle(cuda, axis, m, k, n, bits):
    rng = np.random.default_rng(2)
    lim = 8 if bits == 4 else 127
    codes = rng.integers(-lim, lim if bits == 8 else 8, size=m * k if axis == 0 else k * n)
    q = tgir.pack_codes(codes, bits)
    s = (np.abs(rng.normal(0, 0.02, size=m if axis == 0 else n)) / (7 if bits == 4 else 127)).astype(np.float32)
    act = rng.normal(0, 1, size=k * n if axis == 0 else m * k).astype(np.float32)
    want = tgo.matmul_q(tgo.tgo(), "tgo_", axis, act, q, bits, s, m, k, n)
    got = gpu_matmul_q(cuda, axis, act, q, bits, s, m, k, n)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("axis,m,k,n", [
    (0, 128, 64, 128), (0, 200, 72, 130), (1, 130, 200, 136), (1, 9, 64, 128), (0, 4096, 4096, 256),
    (1, 2048, 1024, 3072), (0, 1024, 4096, 4096),
    # narrow batches (32-column tiles, split K) and ragged rows / columns of the code operand
    (0, 4096, 4096, 9), (0, 300, 1024, 32), (0, 129, 128, 17), (0, 1000, 512, 40), (0, 4096, 1024, 33),
])
def test_matmul_q_tensor_cores_vs_oracle(cuda, axis, m, k, n, bits):
    """Batches above 8 take the tcgen05 GEMM; large shapes are checked on sampled outputs."""
    rng = np.random.default_rng(4)
    lim = 8 if bits == 4 else 127
    codes = rng.integers(-lim, lim if bits == 8 else 8, size=m * k if axis == 0 else k * n)
    q = tgir.pack_codes(codes, bits)
    s = (np.abs(rng.normal(0, 0.02, size=m if axis == 0 else n)) / (7 if bits == 4 else 127)).astype(np.float32)
    act = rng.normal(0, 1, size=k * n if axis == 0 else m * k).astype(np.float32)
    got = gpu_matmul_q(cuda, axis, act, q, bits, s, m, k, n)
    if m * n * k <= 1 << 26:
        want = tgo.matmul_q(tgo.tgo(), "tgo_", axis, act, q, bits, s, m, k, n)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
        return
    # sample: for axis 0 a few batch columns j (full GEMVs), for axis 1 a few rows i
    pick = rng.choice(n if axis == 0 else m, size=6, replace=False)
    for j in pick:
        if axis == 0:
            b = act.reshape(k, n)[:, j].copy()
            want = tgo.matmul_q(tgo.tgo(), "tgo_", 0, b, q, bits, s, m, k, 1)[:, 0]
            np.testing.assert_allclose(got[:, j], want, rtol=RTOL, atol=ATOL)
        else:
            a = act.reshape(m, k)[j].copy()
            want = tgo.matmul_q(tgo.tgo(), "tgo_", 1, a, q, bits, s, 1, k, n)[0]
            np.testing.assert_allclose(got[j], want, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,k,n", [
    # gemv_bulk: rows per CTA chosen for one wave (1 ... 16 warps), ragged last CTA, ragged
    # last register block of a row, every batch width
    (1, 4096, 1), (2, 32, 1), (3, 1056, 2), (147, 4096, 1), (148, 4096, 3), (149, 2048, 4), (4097, 4096, 1),
    (4096, 4096, 5), (1000, 1056, 6), (300, 3072, 7), (16384, 1024, 8), (64, 25600, 1), (9, 12800, 2),
    # activations too large for shared memory twice: gemv_rows
    (256, 32768, 1), (100, 16384, 2),
])
def test_gemv_axis0_vs_oracle(cuda, m, k, n, bits):
    rng = np.random.default_rng(m + k + n)
    lim = 8 if bits == 4 else 127
    codes = rng.integers(-lim, lim if bits == 8 else 8, size=m * k)
    q = tgir.pack_codes(codes, bits)
    s = (np.abs(rng.normal(0, 0.02, size=m)) / (7 if bits == 4 else 127)).astype(np.float32)
    act = rng.normal(0, 1, size=k * n).astype(np.float32)
    want = tgo.matmul_q(tgo.tgo(), "tgo_", 0, act, q, bits, s, m, k, n)
    got = gpu_matmul_q(cuda, 0, act, q, bits, s, m, k, n)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    assert np.array_equal(got, gpu_matmul_q(cuda, 0, act, q, bits, s, m, k, n))  # fixed summation order


@pytest.mark.parametrize("bits", [4, 8])
def test_gemv_axis0_activation_range(cuda, bits):
    """Activations from 1e-30 to 1e30 (the decode divides them by powers of two up to 2^12
    while staging: exact outside the subnormal range, and below it the loss is far under
    the absolute tolerance)."""
    rng = np.random.default_rng(17)
    m, k, n = 512, 2048, 1
    codes = rng.integers(-7, 8, size=m * k)
    q = tgir.pack_codes(codes, bits)
    s = np.full(m, 1e-3, np.float32)
    for scale in (1e-30, 1e-6, 1.0, 1e20, 1e30):
        act = (rng.normal(0, 1, size=k * n) * scale).astype(np.float32)
        want = tgo.matmul_q(tgo.tgo(), "tgo_", 0, act, q, bits, s, m, k, n)
        got = gpu_matmul_q(cuda, 0, act, q, bits, s, m, k, n)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL * min(scale, 1.0))


def test_matmul_q_edge_cases(cuda):
    # code -8 everywhere, k = 1, and a row count that is not a multiple of anything
    for axis, bits, m, k, n in ((0, 4, 3, 1, 1), (1, 4, 1, 1, 2), (0, 4, 5, 64, 2), (1, 8, 2, 5, 3)):
        codes = np.full(m * k if axis == 0 else k * n, -8 if bits == 4 else -127)
        q = tgir.pack_codes(codes, bits)
        s = np.linspace(0.5, 1.5, m if axis == 0 else n).astype(np.float32)
        act = np.random.default_rng(3).normal(size=k * n if axis == 0 else m * k).astype(np.float32)
        want = tgo.matmul_q(tgo.tgo(), "tgo_", axis, act, q, bits, s, m, k, n)
        got = gpu_matmul_q(cuda, axis, act, q, bits, s, m, k, n)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)


def test_matmul_q_rejects_bad_arguments(cuda):
    o = torch.empty(4, device="cuda")
    assert cuda.tg_cuda_matmul_q(2, o.data_ptr(), o.data_ptr(), o.data_ptr(), 4, o.data_ptr(), 1, 1, 1, None) == -1
    assert cuda.tg_cuda_matmul_q(0, o.data_ptr(), o.data_ptr(), o.data_ptr(), 5, o.data_ptr(), 1, 1, 1, None) == -1
    assert cuda.tg_cuda_matmul_q(0, None, o.data_ptr(), o.data_ptr(), 4, o.data_ptr(), 1, 1, 1, None) == -1
    assert b"bad arguments" in cuda.tg_cuda_error() or b"NULL" in cuda.tg_cuda_error()


@pytest.mark.parametrize("bits,axis,shape", [(8, 0, (64, 300)), (8, 1, (300, 64)), (4, 0, (33, 129)), (4, 1, (129, 33)),
                                             (4, 1, (1024, 256)), (8, 0, (7, 5))])
def test_quantize_rtn_bit_exact(cuda, bits, axis, shape):
    rng = np.random.default_rng(9)
    w = rng.normal(0, 0.02, size=shape).astype(np.float32)
    w[0] = 0.0 if axis == 0 else w[0]
    q_want, s_want = tgo.quantize(tgo.tgo(), "tgo_", w, axis, bits)
    dw = dev(w)
    dq = torch.zeros(q_want.size, dtype=torch.int8, device="cuda")
    ds = torch.zeros(s_want.size, dtype=torch.float32, device="cuda")
    rc = cuda.tg_cuda_quantize_rtn(dw.data_ptr(), shape[0], shape[1], axis, bits, dq.data_ptr(), ds.data_ptr(), None)
    assert rc == 0, cuda.tg_cuda_error()
    torch.cuda.synchronize()
    assert np.array_equal(dq.cpu().numpy(), q_want)
    assert np.array_equal(ds.cpu().numpy().view(np.uint32), s_want.view(np.uint32))


@pytest.mark.parametrize("bits,axis,shape,ncal", [(4, 1, (256, 96), 64), (8, 0, (40, 128), 256), (4, 0, (33, 64), 20),
                                                  (4, 1, (1024, 384), 256)])
def test_quantize_gptq_bit_exact(cuda, bits, axis, shape, ncal):
    """Device GPTQ against the oracle restatement of src/quant.c (itself pinned to the
    reference's quantize_param in test_oracle.py). ncal < K makes H rank-deficient:
    the 1% dampening keeps it positive definite, as in the reference."""
    rng = np.random.default_rng(17)
    w = rng.normal(0, 0.02, size=shape).astype(np.float32)
    K = shape[1 - axis]
    x = rng.normal(0, 1, size=(ncal, K)).astype(np.float32)
    x[:, 3] = 0.0  # an input never active: its weights are zeroed (src/quant.c:274-277)
    H = np.zeros((K, K))
    tgo.tgo().tgo_hessian_add(H.ctypes.data_as(tgo.DP), tgo.f32p(x), ncal, K)
    q_want, s_want = tgo.quantize(tgo.tgo(), "tgo_", w, axis, bits, H)
    h = C.c_void_p()
    assert cuda.tg_cuda_gptq_prepare(x.ctypes.data, ncal, K, C.byref(h)) == 0, cuda.tg_cuda_error()
    dw = dev(w)
    dq = torch.zeros(q_want.size, dtype=torch.int8, device="cuda")
    ds = torch.zeros(s_want.size, dtype=torch.float32, device="cuda")
    rc = cuda.tg_cuda_quantize_gptq(h, dw.data_ptr(), shape[0], shape[1], axis, bits, dq.data_ptr(), ds.data_ptr(), None)
    assert rc == 0, cuda.tg_cuda_error()
    torch.cuda.synchronize()
    cuda.tg_cuda_gptq_free(h)
    assert np.array_equal(ds.cpu().numpy().view(np.uint32), s_want.view(np.uint32))
    assert np.array_equal(dq.cpu().numpy(), q_want)
