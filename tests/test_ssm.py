"""Stacked selective-SSM blocks (config 3).

CPU: the oracle restatement (tgo_ssm_forward) against `tgc batch` of the reference
over the same program (tests/golden/nano_ssm: int8 and int4 `tgc quantize`d), bit
for bit. GPU: the engine (tg_cuda_ssm_*) against the oracle on seeded inputs, chunk
boundaries and a partial last chunk included; |gpu - oracle| <= 1e-4 + 1e-3 |oracle|."""
import os

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import ssm

RTOL, ATOL = 1e-3, 1e-4
NANO = dict(blocks=2, d_model=16, d_inner=32, d_state=4, dt_rank=4)


@pytest.mark.parametrize("tag", ["q8", "q4"])
def test_oracle_matches_tgc_batch(golden, tag):
    d = os.path.join(golden, "nano_ssm")
    m = ssm.Model.from_tgir(os.path.join(d, f"{tag}.tgir"), NANO)
    assert m.bits == (8 if tag == "q8" else 4)
    desc, keep = m.desc()
    u = np.loadtxt(os.path.join(d, "u.csv"), delimiter=",", dtype=np.float64).astype(np.float32).reshape(-1, 10, 16)
    want = np.loadtxt(os.path.join(d, f"{tag}_out.csv"), delimiter=",", dtype=np.float64).astype(np.float32)
    got = tgo.ssm_forward(desc, u).reshape(want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


MICRO = dict(blocks=2, d_model=64, d_inner=128, d_state=4, dt_rank=4)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,bits,S,T,chunk", [
    (MICRO, 8, 5, 70, 32),
    (MICRO, 4, 3, 33, 64),
    (dict(ssm.CONFIG3, blocks=1), 8, 4, 40, 16),
    (ssm.CONFIG3, 8, 2, 24, 24),
])
def test_engine_vs_oracle(cuda, cfg, bits, S, T, chunk):
    w = ssm.random_weights(cfg, seed=3)
    m = ssm.quantize_rtn_device(w, cfg, bits)
    u = np.random.default_rng(4).standard_normal((S, T, cfg["d_model"])).astype(np.float32)
    eng = ssm.Engine(m, max_seqs=4, chunk=chunk)
    got = eng.forward(u)
    desc, keep = m.desc()
    want = tgo.ssm_forward(desc, u)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    again = eng.forward(u)  # state and conv carries start from zero on every call
    assert np.array_equal(again, got)


@pytest.mark.gpu
def test_host_and_device_paths_agree(cuda):
    """The host path (chunks copied in and out on their own streams while the next chunk
    computes) with pageable and with pinned buffers, and the device path, give the same
    bits; three waves of sequences and a partial last chunk."""
    import torch

    from technograd_b200 import _lib
    m = ssm.quantize_rtn_device(ssm.random_weights(MICRO, seed=5), MICRO, 8)
    S, T = 7, 100
    u = np.random.default_rng(6).standard_normal((S, T, MICRO["d_model"])).astype(np.float32)
    eng = ssm.Engine(m, max_seqs=3, chunk=16)
    pageable = eng.forward(u)
    hu = torch.from_numpy(u).pin_memory()
    ho = torch.full_like(hu, float("nan")).pin_memory()
    _lib.check(_lib.lib().tg_cuda_ssm_forward(eng.handle, hu.data_ptr(), S, T, ho.data_ptr()))
    du = hu.cuda()
    dout = torch.empty_like(du)
    eng.forward_device(du.data_ptr(), S, T, dout.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(ho.numpy(), pageable)
    assert np.array_equal(dout.cpu().numpy(), pageable)
    desc, keep = m.desc()
    np.testing.assert_allclose(pageable, tgo.ssm_forward(desc, u), rtol=RTOL, atol=ATOL)


@pytest.mark.gpu
def test_engine_rejects_bad_shapes(cuda):
    from technograd_b200 import _lib
    cfg = dict(MICRO, d_state=8)
    m = ssm.quantize_rtn_device(ssm.random_weights(cfg, seed=1), cfg, 8)
    with pytest.raises(_lib.TgCudaError) as e:
        ssm.Engine(m, max_seqs=2)
    assert e.value.status == _lib.EUNSUPPORTED
