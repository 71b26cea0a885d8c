"""The micro-batcher (tg_cuda_batcher_*, the device side of `tgc serve`): rows submitted
one at a time from many threads come back with the reference's `tgc batch` outputs (values
within 1e-3 relative + 1e-4 absolute, think steps equal except rows whose halting quantity
came within 1e-6 of its threshold), with exactly the outputs and steps a single batch of
the same rows gives (the same kernel), and gathered into far fewer GPU batches than rows."""
import ctypes as C
import os
import threading

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import _lib, tgir
from technograd_b200.batch import Batch, Batcher, load_samples

RTOL, ATOL = 1e-3, 1e-4


def _serve(bt, rows, threads):
    """rows submitted one at a time, round-robin over `threads` threads"""
    out = [None] * rows.shape[0]
    errors = []

    def worker(t):
        try:
            for i in range(t, rows.shape[0], threads):
                out[i] = bt.run(rows[i])
        except Exception as e:  # surfaced below
            errors.append(e)

    th = [threading.Thread(target=worker, args=(t,)) for t in range(threads)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert not errors, errors[0]
    return np.stack([o[0] for o in out]), np.stack([o[1] for o in out])


def test_batcher_rejects_bad_arguments():
    L = _lib.lib()
    h = C.c_void_p()
    assert L.tg_cuda_batcher_new(None, 16, 100, C.byref(h)) == _lib.EINVAL


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["latent_reasoner", "halt", "scan"])
def test_concurrent_rows_match_the_reference(cuda, golden, name):
    """The reference's recorded `tgc batch` output of each program's fixture rows."""
    if name == "latent_reasoner":
        path, rows_p, out_p = (os.path.join(golden, f) for f in ("latent_reasoner.q8.tgir", "lr_rows.csv", "lr_q8_out.csv"))
    else:
        path, rows_p, out_p = (os.path.join(golden, "programs", f"{name}{x}") for x in (".tgir", "_rows.csv", "_out.csv"))
    m = tgir.load(path)
    rows = load_samples(rows_p, m.per)
    ref = np.loadtxt(out_p, delimiter=",", dtype=np.float64, ndmin=2)
    bt = Batcher(Batch(m), max_rows=256, max_wait_us=2000)
    got, steps = _serve(bt, rows, threads=16)
    np.testing.assert_allclose(got, ref[:, :m.nout].astype(np.float32), rtol=RTOL, atol=ATOL)
    if m.nthink:
        bad = steps != ref[:, m.nout:].astype(np.int32)
        if bad.any():
            _, _, margin = tgo.program_run(tgir.CProgram(m), rows, margins=True)
            assert (margin[bad] < 1e-6).all(), f"{int(bad.any(axis=1).sum())} rows differ in think steps"
    bt.close()


@pytest.mark.gpu
def test_concurrent_rows_match_one_batch(cuda, golden):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    b = Batch(m)
    rng = np.random.default_rng(21)
    threads, per_thread = 32, 150
    rows = rng.uniform(-2, 2, size=(threads * per_thread, m.per)).astype(np.float32)
    want, want_steps = b.run(rows)
    bt = Batcher(b, max_rows=1024, max_wait_us=2000)
    got = np.zeros_like(want)
    got_steps = np.zeros_like(want_steps)
    errors = []

    def worker(t):
        try:
            for i in range(t * per_thread, (t + 1) * per_thread):
                got[i], got_steps[i] = bt.run(rows[i])
        except Exception as e:  # surfaced below
            errors.append(e)

    th = [threading.Thread(target=worker, args=(t,)) for t in range(threads)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert not errors, errors[0]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(got_steps, want_steps)
    nrows, nbatches = bt.stats()
    assert nrows == rows.shape[0]
    assert nbatches < nrows // 4, (nrows, nbatches)  # rows of different threads share batches
    bt.close()


@pytest.mark.gpu
def test_batcher_reports_a_failed_batch(cuda, golden, monkeypatch):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    bt = Batcher(Batch(m), max_rows=64, max_wait_us=100)
    monkeypatch.setenv("TG_CUDA_FAULT", "h2d")
    with pytest.raises(_lib.TgCudaError) as e:
        bt.run(np.zeros(m.per, np.float32))
    assert e.value.status == _lib.EFAULT
    monkeypatch.delenv("TG_CUDA_FAULT")
    out, _ = bt.run(np.zeros(m.per, np.float32))  # the batcher keeps serving
    assert np.isfinite(out).all()
    bt.close()
