"""The row executor's generated kernels: every golden program is turned into CUDA
source and compiled for sm_100a (no GPU needed), and on the GPU the generated
kernel gives the same bits as the tape interpreter kernel (both run the same
element functions in the same order) and matches the oracle / reference output."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import _lib, tgir
from technograd_b200.batch import Batch, load_samples

RTOL, ATOL = 1e-3, 1e-4
# program -> True when it is within the generator's limits
PROGRAMS = {
    "latent_reasoner.q8.tgir": True,
    "latent_reasoner.f32.tgir": True,
    "ops.tgir": True,
    "programs/halt.tgir": True,
    "programs/scan.tgir": False,  # scans index the arena at run time: interpreter
    "programs/nested_grad.tgir": False,
    "programs/window.tgir": False,  # 400 floats per row: interpreter
    "programs/topk.tgir": True,
    "programs/topk_pad.tgir": True,
    "programs/memscan.tgir": False,  # the memory is indexed at run time: interpreter
    "programs/sufmatch.tgir": False,
    # spmm from a param table is generated; whether the compiled kernel needs a few bytes
    # of local memory (then jit_build refuses it and the interpreter runs) is the compiler's
    "programs/mlp_f32.tgir": None,
    "programs/mlp_q8.tgir": None,
    "programs/mlp_q4.tgir": None,
    "programs/memscan_grad.tgir": False,  # arenas past the register budget
    "programs/memscan4.tgir": False,
    "programs/broadcast.tgir": False,
}

# sum_to over the broadcast patterns of src/util.c:172-212: rows, columns, rank 3, scalars
SUM_TO_CASES = [((3, 4), (1, 4)), ((3, 4), (3, 1)), ((2, 3, 4), (3, 1)), ((2, 3, 4), (4,)), ((2, 3, 4), (2, 1, 4)),
                ((2, 3, 4), (1,)), ((2, 3, 4), (2, 3, 1))]


def sum_to_src(xs, ts):
    sh = lambda s: " ".join(map(str, s))
    return (f"(tgir 1 (model st) (input x (f32 {sh(xs)})) (input y (f32 {sh(ts)}))"
            f" (block (%2 (f32 {sh(ts)}) (sum_to x y))) (output %2))")

# take from a param table by rounded index (runtime/tg_rt.h:316-322), with indices out of range
TAKE_SRC = """(tgir 1
  (model take)
  (param emb (f32 5 3)
    (data 1 2 3 4 5 6 7 8 9 10 11 12 13 14 15))
  (input x (f32 2))
  (block
    (%2 (f32 2 3) (take emb x))
    (%3 (f32 2 3) (tanh %2)))
  (output %3))
"""


def kernel_source(m, compile_: bool):
    L = _lib.lib()
    cp = tgir.CProgram(m)
    n = C.c_long()
    rc = L.tg_cuda_program_kernel(cp.ptr(), None, 0, C.byref(n), 0)
    if rc:
        return rc, ""
    buf = C.create_string_buffer(n.value + 1)
    rc = L.tg_cuda_program_kernel(cp.ptr(), buf, n.value + 1, C.byref(n), 1 if compile_ else 0)
    return rc, buf.value.decode()


# The reference's other stateless programs: whether the generator takes them (NVRTC compiles
# them here, without a GPU)
SMALL_PROGRAMS = {
    "programs/xor.tgir": True,
    "programs/newton.tgir": True,
    "programs/use_import.tgir": True,
    "programs/bcast.tgir": True,
    "programs/file_param.tgir": True,
    "programs/multi_input.tgir": True,
    "programs/nested.tgir": True,
    "programs/cycle.tgir": True,
    "programs/diamond.tgir": True,
    "programs/take_along.tgir": False,  # the gather indexes the arena at run time: interpreter
    "programs/native_matmul.tgir": False,  # more than 192 floats per row: interpreter
}


@pytest.mark.parametrize("name", sorted(SMALL_PROGRAMS))
def test_generated_kernel_compiles_small(golden, name):
    m = tgir.load(os.path.join(golden, name))
    rc, src = kernel_source(m, True)
    if SMALL_PROGRAMS[name]:
        assert rc == 0, _lib.lib().tg_cuda_error().decode()
        assert 'extern "C" __global__' in src and "tg_rowvm" in src
    else:
        assert rc == _lib.EUNSUPPORTED


@pytest.mark.parametrize("name", sorted(PROGRAMS))
def test_generated_kernel_compiles(golden, name):
    m = tgir.load(os.path.join(golden, name))
    rc, src = kernel_source(m, True)
    if PROGRAMS[name] is not False:
        assert rc == 0, _lib.lib().tg_cuda_error().decode()
        assert 'extern "C" __global__' in src and "tg_rowvm" in src
    else:
        assert rc == _lib.EUNSUPPORTED


def test_think_loop_is_a_warp_uniform_jump(golden):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    rc, src = kernel_source(m, False)
    assert rc == 0
    # the think loop of src/vm.c:383-411: halted lanes masked, the warp repeats while any lane runs
    assert "__any_sync(0xffffffffu, done == 0u)) goto L" in src
    assert "it0 >= 32" in src  # maxit of the program
    # quantized matmuls multiply exact codes and scale after the sum
    assert "acc = __fmul_rn(CP(" in src


def _both(m, rows, monkeypatch):
    jit = Batch(m)
    monkeypatch.setenv("TG_CUDA_ROWVM", "interp")
    interp = Batch(m)
    monkeypatch.delenv("TG_CUDA_ROWVM")
    assert interp.specialized == (False, "TG_CUDA_ROWVM=interp")
    return jit, jit.run(rows), interp.run(rows)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(PROGRAMS))
def test_generated_kernel_equals_interpreter(cuda, golden, name, monkeypatch):
    m = tgir.load(os.path.join(golden, name))
    rng = np.random.default_rng(7)
    rows = rng.uniform(-2, 2, size=(1000, m.per)).astype(np.float32)
    jit, (o1, s1), (o2, s2) = _both(m, rows, monkeypatch)
    if PROGRAMS[name] is not None:
        assert jit.specialized[0] == PROGRAMS[name], jit.specialized[1]
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
    assert np.array_equal(s1, s2)


@pytest.mark.gpu
@pytest.mark.parametrize("rows_n", [1, 127, 129, 70001])
def test_latent_reasoner_generated_vs_oracle(cuda, golden, rows_n, monkeypatch):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    rng = np.random.default_rng(rows_n)
    rows = np.where(rng.uniform(size=(rows_n, 8)) < 0.5, rng.integers(0, 2, size=(rows_n, 8)),
                    rng.uniform(-2, 2, size=(rows_n, 8))).astype(np.float32)
    jit, (out, steps), (o2, s2) = _both(m, rows, monkeypatch)
    assert jit.specialized == (True, "")
    assert np.array_equal(out.view(np.uint32), o2.view(np.uint32)) and np.array_equal(steps, s2)
    want, want_steps, margin = tgo.program_run(tgir.CProgram(m), rows, margins=True)
    np.testing.assert_allclose(out, want, rtol=RTOL, atol=ATOL)
    bad = steps != want_steps
    if bad.any():
        assert (margin[bad] < 1e-6).all()


@pytest.mark.gpu
def test_reference_rows_on_generated_kernel(cuda, golden):
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    rows = load_samples(os.path.join(golden, "lr_rows.csv"), m.per)
    ref = np.loadtxt(os.path.join(golden, "lr_q8_out.csv"), delimiter=",", dtype=np.float64)
    b = Batch(m)
    assert b.specialized == (True, "")
    out, steps = b.run(rows)
    np.testing.assert_allclose(out, ref[:, :4].astype(np.float32), rtol=RTOL, atol=ATOL)
    _, _, margin = tgo.program_run(tgir.CProgram(m), rows, margins=True)
    bad = steps != ref[:, 4:].astype(np.int32)
    if bad.any():
        assert (margin[bad] < 1e-6).all()


def test_take_program_generates(golden):
    rc, src = kernel_source(tgir.read(TAKE_SRC), True)
    assert rc == 0, _lib.lib().tg_cuda_error().decode()
    assert "__ldg(GP + " in src


@pytest.mark.gpu
def test_take_on_generated_kernel(cuda, monkeypatch):
    m = tgir.read(TAKE_SRC)
    rows = np.array([[0, 4], [1.49, 1.5], [-0.6, -0.4], [5, 4.49], [2.5, 3.5]] * 50, np.float32)
    jit, (o1, s1), (o2, s2) = _both(m, rows, monkeypatch)
    assert jit.specialized == (True, "")
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
    want, _ = tgo.program_run(tgir.CProgram(m), rows)
    np.testing.assert_allclose(o1, want, rtol=RTOL, atol=ATOL)


@pytest.mark.gpu
def test_host_pipeline_many_chunks(cuda, golden):
    """tg_cuda_batch moves rows through pinned staging in ~4 MB chunks on two streams; a
    ragged multi-chunk batch must give exactly the rows the device-pointer entry gives."""
    import torch
    m = tgir.load(os.path.join(golden, "latent_reasoner.q8.tgir"))
    rng = np.random.default_rng(11)
    rows = rng.uniform(-2, 2, size=(333_333, 8)).astype(np.float32)
    b = Batch(m)
    out, steps = b.run(rows)
    d_in = torch.from_numpy(rows).cuda()
    d_out = torch.empty((rows.shape[0], 4), device="cuda")
    d_steps = torch.zeros((rows.shape[0], 1), dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream()
    _lib.check(cuda.tg_cuda_batch_device(b.handle, d_in.data_ptr(), rows.shape[0], d_out.data_ptr(), d_steps.data_ptr(),
                                         C.c_void_p(s.cuda_stream)))
    torch.cuda.synchronize()
    assert np.array_equal(out.view(np.uint32), d_out.cpu().numpy().view(np.uint32))
    assert np.array_equal(steps, d_steps.cpu().numpy())
    # a second call reuses the staging buffers
    out2, steps2 = b.run(rows[:1000])
    assert np.array_equal(out2, out[:1000]) and np.array_equal(steps2, steps[:1000])


@pytest.mark.parametrize("xs,ts", SUM_TO_CASES)
def test_sum_to_generates(xs, ts):
    rc, src = kernel_source(tgir.read(sum_to_src(xs, ts)), True)
    assert rc == 0, _lib.lib().tg_cuda_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("xs,ts", SUM_TO_CASES)
def test_sum_to_on_generated_kernel(cuda, xs, ts, monkeypatch):
    m = tgir.read(sum_to_src(xs, ts))
    rows = np.random.default_rng(3).normal(size=(300, m.per)).astype(np.float32)
    jit, (o1, _), (o2, _) = _both(m, rows, monkeypatch)
    assert jit.specialized == (True, "")
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
    want, _ = tgo.program_run(tgir.CProgram(m), rows)
    np.testing.assert_allclose(o1, want, rtol=RTOL, atol=ATOL)
