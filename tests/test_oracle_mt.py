"""The threaded, vectorised oracle (oracle/tgo_mt.c) against the scalar restatement
(oracle/tgo.c, pinned to the reference in test_oracle.py) and the reference's own
tg_matmul_qb: the same bits, not a tolerance. CPU only.

tgo_lm_forward_mt is what the full-shape decoder parity tests run, because the scalar
restatement needs ~20 minutes per 1024-token forward."""
import ctypes as C

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import lm

SMALL = dict(layers=2, hidden=256, nq=4, nkv=2, head_dim=128, ffn=512, vocab=1000, theta=1e6)


def _model(cfg, bits, seed):
    """A Qwen3-structured model quantized per output column by the oracle's RTN (CPU)."""
    w = lm.random_weights(cfg, seed=seed, norm_jitter=0.1)
    w["E"] = np.random.default_rng(seed + 1).standard_normal(w["E"].shape).astype(np.float32)
    f32, q = {}, {}
    for name, a in w.items():
        if lm.is_linear(name):
            codes, s = tgo.quantize(tgo.tgo(), "tgo_", a, 1, bits)
            q[name] = lm.QParam(codes, s, bits, a.shape)
        else:
            f32[name] = a
    return lm.Model(cfg, bits, f32, q)


@pytest.mark.parametrize("bits,m,k,n", [(4, 1, 64, 96), (4, 7, 130, 45), (8, 5, 33, 200), (4, 9, 256, 1000), (8, 1, 7, 3)])
def test_matmul_qb_mt_is_bit_exact(bits, m, k, n):
    rng = np.random.default_rng(m * 1000 + n)
    codes = rng.integers(-8 if bits == 4 else -127, 8 if bits == 4 else 128, size=k * n)
    from technograd_b200.tgir import pack_codes
    q = np.ascontiguousarray(pack_codes(codes, bits))
    s = rng.random(n).astype(np.float32)
    a = rng.standard_normal(m * k).astype(np.float32)
    want = tgo.matmul_q(tgo.tgo(), "tgo_", 1, a, q, bits, s, m, k, n)
    got = np.zeros((m, n), np.float32)
    for threads in (1, 3):
        got[:] = np.nan
        tgo.tgo().tgo_matmul_qb_mt(tgo.f32p(got), tgo.f32p(a), tgo.i8p(q), bits, tgo.f32p(s), m, k, n, threads)
        assert np.array_equal(got, want)
    R = tgo.ref()
    if R is not None:
        assert np.array_equal(got, tgo.matmul_q(R, "ref_", 1, a, q, bits, s, m, k, n))


@pytest.mark.parametrize("bits,nkv", [(4, 2), (8, 4)])
def test_lm_forward_mt_is_bit_exact(bits, nkv):
    cfg = dict(SMALL, nkv=nkv)
    model = _model(cfg, bits, seed=20 + bits)
    d, keep = model.desc()
    L = tgo.tgo()
    rng = np.random.default_rng(bits)
    # T = 1 (one key), 5, 33 (a key block and a bit), 77 (query blocks of 16 with a partial one), 130
    for T in (1, 5, 33, 77, 130):
        ids = rng.integers(0, cfg["vocab"], size=T).astype(np.float32)
        ids[0] = -2.0  # out of range: a zero embedding row, as take() gives
        want = np.zeros(cfg["vocab"], np.float32)
        L.tgo_lm_forward(C.addressof(d), tgo.f32p(ids), T, tgo.f32p(want))
        for threads in (1, 4):
            got = np.full(cfg["vocab"], np.nan, np.float32)
            assert L.tgo_lm_forward_mt(C.addressof(d), tgo.f32p(ids), T, tgo.f32p(got), threads) == 0
            assert np.array_equal(got, want), f"T={T} threads={threads}"
