"""The reference's control-flow test programs (tests/scan/scan.tg, tests/think/halt.tg,
tests/scan/nested_grad.tg, tests/attn/window.tg) and the programs of its sparse and
memory tests (tests/memory/topk.tg, topk_pad.tg, scan.tg, sufmatch.tg; tests/quant/mlp.tg
as f32 and quantized to int8 / int4, an spmm table) on the oracle VM and on the device
row executor, against `tgc batch` output of the reference (tests/golden/programs), and the
reference's remaining stateless programs the same way.

The oracle follows the reference's arithmetic order with the same libm, so it must
agree bit for bit. The device path: values within 1e-4 + 1e-3 |ref|; think steps
equal except rows whose halting quantity came within 1e-6 of its threshold."""
import os

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import tgir
from technograd_b200.batch import Batch, load_samples

RTOL, ATOL = 1e-3, 1e-4
NAMES = ["scan", "halt", "nested_grad", "window",
         # the sparse and memory models' ops: spmm (f32 and quantized tables), topk, memscan, sufmatch
         "topk", "topk_pad", "memscan", "sufmatch", "mlp_f32", "mlp_q8", "mlp_q4",
         # gradients inside forward programs: memscan_t and take_t (tests/memory/scan_grad.tg,
         # scan4.tg), sum_to with batched matmuls and rank-3 transposes (tests/native/broadcast.tg)
         "memscan_grad", "memscan4", "broadcast"]


def fixture(golden, name):
    d = os.path.join(golden, "programs")
    m = tgir.load(os.path.join(d, f"{name}.tgir"))
    rows = load_samples(os.path.join(d, f"{name}_rows.csv"), m.per)
    ref = np.loadtxt(os.path.join(d, f"{name}_out.csv"), delimiter=",", dtype=np.float64, ndmin=2)
    return m, rows, ref[:, :m.nout].astype(np.float32), ref[:, m.nout:].astype(np.int32)


@pytest.mark.parametrize("name", NAMES)
def test_oracle_vm_matches_tgc_batch(golden, name):
    m, rows, want, want_steps = fixture(golden, name)
    out, steps = tgo.program_run(tgir.CProgram(m), rows)
    assert steps.shape == want_steps.shape
    assert np.array_equal(steps, want_steps)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_known_answers_of_the_reference_suite(golden):
    """tests/run.sh:33-36 expect_run rows: topk, topk with k past the row, suffix match."""
    for name, want in [("topk", [1, 3, 2, 5, 0, 1, 2, 3, 0, 1, 2, 3]), ("topk_pad", [1, 0, 2, -1, -1]),
                       ("sufmatch", [-1, 0, -1, 0, -1, 0, -1, 0, -1, 0, 6, 1, 2, 1, 5, 2, 3, 2, 6, 3, 1, 3, 5, 4, 2, 4,
                                     -1, 0, 3, 5, 6, 1, 1, 6, 5, 2, -1, 0, -1, 0, 2, 1, 5, 1, 3, 2, 6, 2])]:
        m, rows, ref, _ = fixture(golden, name)
        out, _ = tgo.program_run(tgir.CProgram(m), rows[:1])
        assert out[0].tolist() == want == ref[0].tolist()


# Every other stateless program of the reference's tests and examples (tests/golden/make_golden.py
# SMALL): plain ops, imports (diamond and cycle), file() params, several inputs, broadcasts,
# take_along, a think loop (newton) and the native matmul forms.
SMALL_NAMES = ["xor", "newton", "use_import", "bcast", "file_param", "multi_input", "nested", "cycle", "diamond",
               "take_along", "native_matmul"]


@pytest.mark.parametrize("name", SMALL_NAMES)
def test_oracle_vm_matches_tgc_batch_small(golden, name):
    m, rows, want, want_steps = fixture(golden, name)
    out, steps = tgo.program_run(tgir.CProgram(m), rows)
    assert np.array_equal(steps, want_steps)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_known_answers_of_the_small_programs(golden):
    """tests/run.sh:26-35,427-428: xor's truth table, newton's square roots and 5 steps,
    take_along, and the import diamond and cycle."""
    cases = [("xor", 4, [[0], [1], [1], [0]], None), ("newton", 1, [[1.41421354, 3, 4]], [[5]]),
             ("take_along", 1, [[4, 1, 0, 6, 0, 11]], None), ("diamond", 1, [[23, 43]], None),
             ("cycle", 1, [[11, 21]], None)]
    for name, k, want, want_steps in cases:
        m, rows, ref, ref_steps = fixture(golden, name)
        out, steps = tgo.program_run(tgir.CProgram(m), rows[:k])
        np.testing.assert_array_equal(out, np.array(want, np.float32))
        np.testing.assert_array_equal(ref[:k], np.array(want, np.float32))
        if want_steps is not None:
            assert steps.tolist() == want_steps == ref_steps[:k].tolist()


def test_halt_step_counts(golden):
    """tests/run.sh:374: `tgc run tests/think/halt.tg 1,1` stops after 5 steps, 0,0 after 19."""
    m, rows, _, want_steps = fixture(golden, "halt")
    _, steps = tgo.program_run(tgir.CProgram(m), rows[:2])
    assert steps[:, 0].tolist() == [5, 19] == want_steps[:2, 0].tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES + SMALL_NAMES)
def test_device_executor_matches_tgc_batch(cuda, golden, name):
    m, rows, want, want_steps = fixture(golden, name)
    out, steps = Batch(m).run(rows)
    np.testing.assert_allclose(out, want, rtol=RTOL, atol=ATOL)
    bad = steps != want_steps
    if bad.any():
        _, _, margin = tgo.program_run(tgir.CProgram(m), rows, margins=True)
        assert (margin[bad] < 1e-6).all(), f"{int(bad.any(axis=1).sum())} rows differ in think steps away from the threshold"
