"""The C host binding compiled and run: the reference's tgc driver with `tgc batch ...
--device cuda` (technograd_b200/host: the src/cuda.c adapter and the batch branch a
maintainer adds; built by oracle/Makefile against the reference's sources into
oracle/_ref/tgc_cuda, linked to libtgcuda.so).

CPU: every other command is the reference's own; the adapter's flattening of a loaded,
planned Module gives the library the same program as the Python reader's (the generated
CUDA source is byte-identical) and that kernel compiles for sm_100a without a GPU; a bad
row, a bad --device and a missing GPU end the run before the output file exists.

GPU: `--device cuda` against the reference's `tgc batch -j auto` on the same rows, and on
every stateless program fixture against the reference's recorded output: values within
1e-3 relative + 1e-4 absolute, think steps equal except rows whose halting quantity came
within 1e-6 of its threshold."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFDIR = os.path.join(ROOT, "oracle", "_ref")
TGC_CUDA, TGC = os.path.join(REFDIR, "tgc_cuda"), os.path.join(REFDIR, "tgc")
PROGRAMS = os.path.join(ROOT, "tests", "golden", "programs")
LR = os.path.join(ROOT, "tests", "golden", "latent_reasoner.q8.tgir")
RTOL, ATOL = 1e-3, 1e-4
# the reference's stateless test and example programs with their `tgc batch` fixtures
STATELESS = ["scan", "halt", "nested_grad", "window", "topk", "topk_pad", "memscan", "sufmatch", "mlp_f32", "mlp_q8",
             "mlp_q4", "memscan_grad", "memscan4", "broadcast", "xor", "newton", "use_import", "bcast", "file_param",
             "multi_input", "nested", "cycle", "diamond", "take_along", "native_matmul"]

pytestmark = pytest.mark.skipif(not (os.path.exists(TGC_CUDA) and os.path.exists(TGC)),
                                reason="oracle/_ref/tgc_cuda is built only where the reference sources are present")


def run(exe, *args, cwd):
    return subprocess.run([exe, *args], capture_output=True, text=True, timeout=600, cwd=cwd)


def test_other_commands_are_the_reference(tmp_path):
    for args in (["check", LR], ["plan", LR], ["ir", os.path.join(PROGRAMS, "halt.tgir")]):
        a, b = run(TGC_CUDA, *args, cwd=tmp_path), run(TGC, *args, cwd=tmp_path)
        assert (a.returncode, a.stdout, a.stderr) == (b.returncode, b.stdout, b.stderr)
    rows = os.path.join(ROOT, "tests", "golden", "lr_rows.csv")
    a = run(TGC_CUDA, "batch", LR, rows, "-j", "2", "-o", "a.csv", cwd=tmp_path)
    b = run(TGC, "batch", LR, rows, "-j", "2", "-o", "b.csv", cwd=tmp_path)
    assert a.returncode == b.returncode == 0
    assert (tmp_path / "a.csv").read_bytes() == (tmp_path / "b.csv").read_bytes()


@pytest.mark.parametrize("name", ["latent_reasoner"] + STATELESS)
def test_adapter_flattening_matches_the_reader(tmp_path, name):
    """cuda.c flattens the reference's own loaded, planned Module; tgir.py reads the same
    TGIR in Python. Both hand tg_cuda_program_kernel a program: the sources must be equal,
    and the adapter's must compile for sm_100a (or both go to the interpreter)."""
    from technograd_b200 import _lib, tgir
    path = LR if name == "latent_reasoner" else os.path.join(PROGRAMS, f"{name}.tgir")
    r = run(TGC_CUDA, "cuda-kernel", path, "-o", "k.cu", cwd=tmp_path)
    assert r.returncode == 0, r.stderr
    prog = tgir.CProgram(tgir.load(path))
    n = C.c_long(0)
    L = _lib.lib()
    rc = L.tg_cuda_program_kernel(C.byref(prog.c), None, 0, C.byref(n), 0)
    if r.stdout.startswith("interpreter:"):
        assert rc == _lib.EUNSUPPORTED
        assert r.stdout.strip() == "interpreter: " + L.tg_cuda_error().decode()
        return
    assert rc == 0 and "compiled for sm_100a" in r.stderr
    buf = C.create_string_buffer(n.value + 1)
    assert L.tg_cuda_program_kernel(C.byref(prog.c), buf, n.value + 1, C.byref(n), 0) == 0
    assert (tmp_path / "k.cu").read_bytes() == buf.value


def test_bad_row_fails_before_the_output_exists(tmp_path):
    (tmp_path / "bad.csv").write_text("1,0,1,0,1,0,1,0\n1,2,x\n")
    a = run(TGC_CUDA, "batch", LR, "bad.csv", "-o", "out.csv", "--device", "cuda", cwd=tmp_path)
    b = run(TGC, "batch", LR, "bad.csv", "-o", "ref.csv", cwd=tmp_path)
    assert a.returncode == b.returncode == 1 and a.stderr == b.stderr
    assert not (tmp_path / "out.csv").exists() and not (tmp_path / "ref.csv").exists()
    (tmp_path / "short.csv").write_text("1,0,1\n")
    a = run(TGC_CUDA, "batch", LR, "short.csv", "-o", "out.csv", "--device", "cuda", cwd=tmp_path)
    assert a.returncode == 1 and "row has 3 values, model latent_reasoner needs 8" in a.stderr
    assert not (tmp_path / "out.csv").exists()
    a = run(TGC_CUDA, "batch", LR, "short.csv", "-o", "out.csv", "--device", "tpu", cwd=tmp_path)
    assert a.returncode == 1 and "only 'cuda'" in a.stderr and not (tmp_path / "out.csv").exists()


def _gpu_visible() -> bool:
    import torch
    return torch.cuda.is_available()


def test_no_gpu_fails_before_the_output_exists(tmp_path):
    if _gpu_visible():
        pytest.skip("a GPU is visible")
    rows = os.path.join(ROOT, "tests", "golden", "lr_rows.csv")
    a = run(TGC_CUDA, "batch", LR, rows, "-o", "out.csv", "--device", "cuda", cwd=tmp_path)
    assert a.returncode == 1 and "--device cuda:" in a.stderr
    assert not (tmp_path / "out.csv").exists()


def _check(m_path, rows, got, want, nout, nthink):
    """values within tolerance; think steps equal except near-threshold rows (oracle margins)"""
    from oracle import tgo
    from technograd_b200 import tgir
    np.testing.assert_allclose(got[:, :nout], want[:, :nout], rtol=RTOL, atol=ATOL)
    if nthink:
        bad = got[:, nout:] != want[:, nout:]
        if bad.any():
            _, _, margin = tgo.program_run(tgir.CProgram(tgir.load(m_path)), rows, margins=True)
            assert (margin[bad] < 1e-6).all(), f"{int(bad.any(axis=1).sum())} rows differ in think steps"


@pytest.mark.gpu
def test_device_cuda_matches_reference_batch(tmp_path):
    """100,003 rows of config 1 as binary files through `--device cuda`, against the
    reference's `tgc batch -j auto` run here on the same rows; the text format (which
    carries the think steps) on the first 3000."""
    from technograd_b200 import tgir
    rows = np.random.default_rng(11).integers(0, 2, size=(100003, 8)).astype("<f4")
    rows.tofile(tmp_path / "rows.bin")
    a = run(TGC_CUDA, "batch", LR, "rows.bin", "-o", "gpu.bin", "--device", "cuda", "-v", cwd=tmp_path)
    assert a.returncode == 0, a.stderr
    assert "--device cuda" in a.stderr
    b = run(TGC, "batch", LR, "rows.bin", "-o", "cpu.bin", "-j", "auto", cwd=tmp_path)
    assert b.returncode == 0, b.stderr
    got = np.fromfile(tmp_path / "gpu.bin", "<f4").reshape(-1, 4)
    want = np.fromfile(tmp_path / "cpu.bin", "<f4").reshape(-1, 4)
    assert got.shape == want.shape == (100003, 4)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    np.savetxt(tmp_path / "rows.csv", rows[:3000], fmt="%g", delimiter=",")
    a = run(TGC_CUDA, "batch", LR, "rows.csv", "-o", "gpu.csv", "--device", "cuda", cwd=tmp_path)
    b = run(TGC, "batch", LR, "rows.csv", "-o", "cpu.csv", "-j", "auto", cwd=tmp_path)
    assert a.returncode == b.returncode == 0
    got = np.loadtxt(tmp_path / "gpu.csv", delimiter=",", ndmin=2)
    want = np.loadtxt(tmp_path / "cpu.csv", delimiter=",", ndmin=2)
    _check(LR, rows[:3000], got, want, 4, tgir.load(LR).nthink)


@pytest.mark.gpu
@pytest.mark.parametrize("name", STATELESS)
def test_device_cuda_programs_match_fixtures(tmp_path, name):
    from technograd_b200 import tgir
    path = os.path.join(PROGRAMS, f"{name}.tgir")
    m = tgir.load(path)
    a = run(TGC_CUDA, "batch", path, os.path.join(PROGRAMS, f"{name}_rows.csv"), "-o", "gpu.csv", "--device", "cuda",
            cwd=tmp_path)
    assert a.returncode == 0, a.stderr
    got = np.loadtxt(tmp_path / "gpu.csv", delimiter=",", dtype=np.float64, ndmin=2)
    want = np.loadtxt(os.path.join(PROGRAMS, f"{name}_out.csv"), delimiter=",", dtype=np.float64, ndmin=2)
    assert got.shape == want.shape
    from technograd_b200.batch import load_samples
    rows = load_samples(os.path.join(PROGRAMS, f"{name}_rows.csv"), m.per)
    _check(path, rows, got, want, m.nout, m.nthink)


@pytest.mark.gpu
def test_stream_device_cuda_matches_reference_stream(tmp_path):
    """`tgc stream --device cuda` (rows through the micro-batcher) against the reference's
    `tgc stream` on the same lines: the same error lines for malformed rows, values within
    tolerance and think steps under the 1e-6 rule for the rest."""
    from technograd_b200 import tgir
    rows = np.random.default_rng(13).integers(0, 2, size=(300, 8)).astype(np.float32)
    lines = [",".join(f"{v:g}" for v in r) for r in rows]
    lines[7], lines[100] = "1,2,x", "1,2,3"  # a bad number and a short row
    lines[200] += "\r"  # a CRLF line ending
    (tmp_path / "in.csv").write_text("\n".join(lines) + "\n")
    a = run(TGC_CUDA, "stream", LR, "in.csv", "-o", "gpu.txt", "--device", "cuda", cwd=tmp_path)
    b = run(TGC, "stream", LR, "in.csv", "-o", "cpu.txt", cwd=tmp_path)
    assert a.returncode == b.returncode == 0, a.stderr
    got, want = (tmp_path / "gpu.txt").read_text().splitlines(), (tmp_path / "cpu.txt").read_text().splitlines()
    assert len(got) == len(want) == 300
    good = [i for i in range(300) if not want[i].startswith("error:")]
    for i in set(range(300)) - set(good):
        assert got[i] == want[i]
    g = np.array([[float(x) for x in got[i].split(",")] for i in good])
    w = np.array([[float(x) for x in want[i].split(",")] for i in good])
    _check(LR, rows[good], g, w, 4, tgir.load(LR).nthink)
