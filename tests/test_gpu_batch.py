"""tg_cuda_batch (the `tgc batch --device cuda` path) against the reference's
own batch output and the oracle VM (GPU).

Values: |gpu - ref| <= 1e-4 + 1e-3 |ref|. Think steps: equal, except rows
whose halting delta came within 1e-6 of the threshold in some iteration
(north_star); the oracle reports that margin per row."""
import os

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import _lib, tgir
from technograd_b200.batch import Batch, load_samples, write_rows

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-3, 1e-4


def check_rows(out, steps, want, want_steps, margin):
    np.testing.assert_allclose(out, want, rtol=RTOL, atol=ATOL)
    bad = steps != want_steps
    if bad.any():
        assert (margin[bad] < 1e-6).all(), f"{int(bad.sum())} rows differ in think steps away from the threshold"


@pytest.mark.parametrize("tag", ["f32", "q8"])
def test_latent_reasoner_vs_tgc_batch(cuda, golden, tag):
    m = tgir.load(os.path.join(golden, f"latent_reasoner.{tag}.tgir"))
    rows = load_samples(os.path.join(golden, "lr_rows.csv"), m.per)
    ref = np.loadtxt(os.path.join(golden, f"lr_{tag}_out.csv"), delimiter=",", dtype=np.float64)
    out, steps = Batch(m).run(rows)
    _, _, margin = tgo.program_run(tgir.CProgram(m), rows, margins=True)
    check_rows(out, steps, ref[:, :4].astype(np.float32), ref[:, 4:].astype(np.int32), margin)


def test_latent_reasoner_large_vs_oracle(cuda, golden):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    rng = np.random.default_rng(1)
    rows = np.concatenate([rng.integers(0, 2, size=(30000, 8)), rng.uniform(-2, 2, size=(30001, 8))]).astype(np.float32)
    out, steps = Batch(m).run(rows)
    want, want_steps, margin = tgo.program_run(tgir.CProgram(m), rows, margins=True)
    check_rows(out, steps, want, want_steps, margin)
    # The arithmetic follows the reference order; CUDA's tanhf/expf differ from glibc by
    # an ulp now and then, so only some rows end bit-identical (about 15% measured).
    exact = (out == want).all(axis=1).mean()
    print(f"bit-identical rows: {exact:.3f}")


def test_ops_program(cuda, golden):
    m = tgir.load(os.path.join(golden, "ops.tgir"))
    want = np.array(open(os.path.join(golden, "ops_expected.txt")).read().split(), np.float64).astype(np.float32)
    out, _ = Batch(m).run(np.array([[1, -2, 3, 0.5]] * 3, np.float32))  # tests/run.sh:32
    for r in range(3):
        np.testing.assert_allclose(out[r], want, rtol=RTOL, atol=ATOL)


def test_text_output_format(cuda, golden, tmp_path):
    m = tgir.load(os.path.join(golden, "latent_reasoner.f32.tgir"))
    out, steps = Batch(m).run(np.array([[1, 0, 0, 1, 0, 1, 1, 0]], np.float32))
    p = tmp_path / "o.csv"
    write_rows(str(p), out, steps)
    vals = p.read_text().strip().split(",")
    assert vals[-1] == "9"  # README.md:48-51 of the reference: steps 0 9
    np.testing.assert_allclose(np.array(vals[:4], np.float32), [0.225605994, 0.24476327, 0.162138939, 0.367491812],
                               rtol=RTOL, atol=ATOL)


def test_stateful_model_rejected(cuda, golden):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    m.nupd = 1
    with pytest.raises(_lib.TgCudaError) as e:
        Batch(m)
    assert e.value.status == _lib.EUNSUPPORTED


@pytest.mark.parametrize("step", ["alloc", "h2d", "launch", "gather"])
def test_injected_failures_are_reported(cuda, golden, step, monkeypatch):
    """TG_CUDA_FAULT makes one host step report an error status: no GPU fault is produced."""
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    b = Batch(m)
    monkeypatch.setenv("TG_CUDA_FAULT", step)
    with pytest.raises(_lib.TgCudaError) as e:
        b.run(np.zeros((100, 8), np.float32))
    assert e.value.status == _lib.EFAULT
    monkeypatch.delenv("TG_CUDA_FAULT")
    out, _ = b.run(np.zeros((10, 8), np.float32))  # the context stays usable
    assert np.isfinite(out).all()


def test_empty_and_single_rows(cuda, golden):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    b = Batch(m)
    out, steps = b.run(np.zeros((0, 8), np.float32))
    assert out.shape == (0, 4)
    for n in (1, 127, 128, 129, 1025):
        rows = np.random.default_rng(n).integers(0, 2, size=(n, 8)).astype(np.float32)
        out, steps = b.run(rows)
        want, want_steps, margin = tgo.program_run(tgir.CProgram(m), rows, margins=True)
        check_rows(out, steps, want, want_steps, margin)


def test_registered_host_buffers_match_staged(cuda, golden):
    """Caller buffers page-locked with tg_cuda_host_register are copied straight to and
    from the GPU: the same bits as through the staging buffers. 300,001 rows are four full
    2 MB input chunks and a partial one, so each of the three slots is reused; a buffer only
    partly registered goes through staging; an overlapping registration and an unknown
    pointer are refused."""
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    b = Batch(m)
    rows = np.random.default_rng(7).uniform(-2, 2, size=(300001, 8)).astype(np.float32)
    want, want_steps = b.run(rows)
    L = _lib.lib()

    def call(o, s):
        _lib.check(L.tg_cuda_batch(b.handle, rows.ctypes.data, rows.shape[0], 8, o.ctypes.data, 4, s.ctypes.data, 1))

    out = np.full((rows.shape[0], 4), np.nan, np.float32)
    steps = np.full((rows.shape[0], 1), -1, np.int32)
    with _lib.HostRegistered(rows, out, steps):
        call(out, steps)
        with pytest.raises(_lib.TgCudaError) as e:
            _lib.check(L.tg_cuda_host_register(rows.ctypes.data + 4096, 64))
        assert e.value.status == _lib.EINVAL
    assert np.array_equal(out, want) and np.array_equal(steps, want_steps)
    out2 = np.full_like(out, np.nan)
    steps2 = np.full_like(steps, -1)
    with _lib.HostRegistered(rows[:150000], out2, steps2):
        call(out2, steps2)
    assert np.array_equal(out2, want) and np.array_equal(steps2, want_steps)
    with pytest.raises(_lib.TgCudaError) as e:
        _lib.check(L.tg_cuda_host_unregister(rows.ctypes.data))
    assert e.value.status == _lib.EINVAL
