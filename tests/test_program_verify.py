"""tg_cuda_load checks the program it is handed before anything reaches a GPU: operand and
body indices in range, every instruction in one block, and every declared shape equal to the
one its operands give by the reference's rules (op_infer, src/ops.c:96-295; the think, scan,
topk and reshape checks of src/ir.c:258-447). A malformed program is TG_CUDA_EINVAL, never a
kernel that indexes past a value. CPU only: tg_cuda_program_kernel runs the same checks
without a device. Where the reference's `tgc` is built, it rejects the same TGIR files."""
import ctypes as C
import glob
import os
import subprocess

import pytest

from technograd_b200 import _lib, tgir

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TGC = os.path.join(ROOT, "oracle", "_ref", "tgc")
BASE = "(tgir 1 (model m) {params} (input x (f32 2)) (block {block}) (output {out}))"
P2 = "(param p (f32 2) (data 1 2))"


def check(cp):
    n = C.c_long()
    rc = _lib.lib().tg_cuda_program_kernel(cp.ptr(), None, 0, C.byref(n), 0)
    return rc, _lib.lib().tg_cuda_error().decode()


BAD_TGIR = {
    "declared shape": BASE.format(params=P2, block="(%2 (f32 3) (add x p))", out="%2"),
    "operand count": BASE.format(params=P2, block="(%2 (f32 2) (add x))", out="%2"),
    "matmul": BASE.format(params="(param w (f32 3 5) (data " + " ".join(["1"] * 15) + "))",
                          block="(%2 (f32 3) (matmul w x))", out="%2"),
    "broadcast": BASE.format(params="(param p (f32 3) (data 1 2 3))", block="(%2 (f32 3) (add x p))", out="%2"),
    "outer": BASE.format(params="(param w (f32 2 2) (data 1 2 3 4))", block="(%2 (f32 2 2) (outer w x))", out="%2"),
    "topk k": BASE.format(params="", block="(%2 (f32 300) (topk x))", out="%2"),
    "reshape count": BASE.format(params="", block="(%2 (f32 3) (reshape x))", out="%2"),
    "transpose": BASE.format(params="", block="(%2 (f32 2) (transpose x))", out="%2"),
    "think yield": BASE.format(params=P2, block="(%2 (f32 2) (think x 5 none (%3 (f32) (sum %2)) (yield %3)))",
                               out="%2"),
}


@pytest.mark.parametrize("name", sorted(BAD_TGIR))
def test_malformed_programs_are_rejected_at_load(name, tmp_path):
    src = BAD_TGIR[name]
    try:
        m = tgir.read(src)
    except tgir.TgirError:
        pytest.skip("the TGIR reader already rejects it")
    rc, msg = check(tgir.CProgram(m))
    assert rc == _lib.EINVAL, msg
    assert ": instruction " in msg, msg
    if os.path.exists(TGC):  # the reference rejects the same file
        mp = tmp_path / "m.tgir"
        mp.write_text(src)
        (tmp_path / "r.csv").write_text("0,0\n")
        r = subprocess.run([TGC, "batch", str(mp), str(tmp_path / "r.csv")], capture_output=True, text=True, timeout=60)
        assert r.returncode != 0


def test_every_golden_program_passes():
    """No valid program is rejected: every TGIR fixture the reference produced."""
    paths = sorted(glob.glob(os.path.join(ROOT, "tests", "golden", "**", "*.tgir"), recursive=True))
    assert len(paths) >= 20
    for p in paths:
        rc, msg = check(tgir.CProgram(tgir.load(p)))
        assert rc in (_lib.OK, _lib.EUNSUPPORTED) and ": instruction " not in msg, (p, msg)


def scan_program():
    return tgir.CProgram(tgir.load(os.path.join(ROOT, "tests", "golden", "programs", "scan.tgir")))


def think_program():
    return tgir.CProgram(tgir.load(os.path.join(ROOT, "tests", "golden", "programs", "halt.tgir")))


def first(cp, op):
    return next(i for i in range(cp.c.nins) if cp.c.ins[i].op == _lib.OP[op])


@pytest.mark.parametrize("mutate,why", [
    (lambda cp: setattr(cp.c.ins[first(cp, "scan")], "scan", 7), "scan out of range"),
    (lambda cp: setattr(cp.c.ins[first(cp, "scan")], "nbody", 10 ** 6), "block out of range"),
    (lambda cp: setattr(cp.c.ins[first(cp, "scan")], "body", 0), "belongs to two blocks"),
    (lambda cp: setattr(cp.c.scans[0], "T", cp.c.scans[0].T + 1), "T steps"),
    (lambda cp: setattr(cp.c.scans[0], "nc", 0), "malformed scan"),
])
def test_corrupt_scans_are_rejected(mutate, why):
    cp = scan_program()
    assert check(cp)[0] in (_lib.OK, _lib.EUNSUPPORTED)
    mutate(cp)
    rc, msg = check(cp)
    assert rc == _lib.EINVAL and why in msg, msg


@pytest.mark.parametrize("mutate,why", [
    (lambda cp: setattr(cp.c.ins[first(cp, "think")], "tid", 5), "malformed think"),
    (lambda cp: setattr(cp.c.ins[first(cp, "think")], "maxit", 0), "malformed think"),
    (lambda cp: setattr(cp.c.ins[first(cp, "think")], "yield_", cp.c.nval), "malformed think"),
    (lambda cp: setattr(cp.c, "ntop", cp.c.nins), "belongs to two blocks"),
])
def test_corrupt_thinks_are_rejected(mutate, why):
    cp = think_program()
    assert check(cp)[0] == _lib.OK
    mutate(cp)
    rc, msg = check(cp)
    assert rc == _lib.EINVAL and why in msg, msg


def test_bad_values_and_inputs_are_rejected():
    cp = think_program()
    cp.c.val[0].dim[0] = 0
    assert check(cp)[0] == _lib.EINVAL
    cp = think_program()
    cp.c.inputs[0] = 0  # a param, not an input
    rc, msg = check(cp)
    assert rc == _lib.EINVAL and "not an input" in msg
