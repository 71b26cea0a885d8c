"""The micro-batcher (tg_cuda_batcher_*, the device side of `tgc serve`): rows submitted
one at a time from many threads come back with exactly the outputs and think steps a
single batch of the same rows gives (the same kernel), and they are gathered into far
fewer GPU batches than rows."""
import ctypes as C
import os
import threading

import numpy as np
import pytest

from technograd_b200 import _lib, tgir
from technograd_b200.batch import Batch, Batcher


def test_batcher_rejects_bad_arguments():
    L = _lib.lib()
    h = C.c_void_p()
    assert L.tg_cuda_batcher_new(None, 16, 100, C.byref(h)) == _lib.EINVAL


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
