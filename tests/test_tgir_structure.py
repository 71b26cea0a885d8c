"""Which TGIR files load: our reader plus tg_cuda_load's checks against the reference's own
`tgc` (src/ir.c: the order of top-level forms, names defined once, quant forms, shapes and
operand counts). A file the reference rejects is rejected here too, by the reader
(TgirError) or at load (TG_CUDA_EINVAL). CPU only."""
import ctypes as C
import os
import subprocess

import pytest

from technograd_b200 import _lib, tgir

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TGC = os.path.join(ROOT, "oracle", "_ref", "tgc")
BASE = "(tgir 1 (model m) {params} (input x (f32 2)) (block {block}) (output {out}))"
P = "(param p (f32 2) (data 1 2))"
ADD = "(%2 (f32 2) (add x p))"
CASES = {
    "valid": (True, BASE.format(params=P, block=ADD, out="%2")),
    "comment inside data": (True, BASE.format(params="(param p (f32 2) (data 1 ; c\n 2))", block=ADD, out="%2")),
    "int4 code -8": (False, BASE.format(params="(param W (f32 1 2) (quant 4 0 (scale 1) (codes -8 2)))",
                                       block="(%2 (f32 2) (tanh x))", out="%2")),
    "value count": (False, BASE.format(params="(param p (f32 2) (data 1 2 3))", block=ADD, out="%2")),
    "declared shape": (False, BASE.format(params=P, block="(%2 (f32 3) (add x p))", out="%2")),
    "unknown op": (False, BASE.format(params=P, block="(%2 (f32 2) (frob x p))", out="%2")),
    "undefined name": (False, BASE.format(params=P, block="(%2 (f32 2) (add x q))", out="%2")),
    "undefined output": (False, BASE.format(params=P, block=ADD, out="%9")),
    "redefinition": (False, BASE.format(params=P + " " + P, block=ADD, out="%2")),
    "operand count": (False, BASE.format(params=P, block="(%2 (f32 2) (add x))", out="%2")),
    "version": (False, "(tgir 2 (model m) (input x (f32 2)) (block (%2 (f32 2) (tanh x))) (output %2))"),
    "no model": (False, "(tgir 1 (input x (f32 2)) (block (%2 (f32 2) (tanh x))) (output %2))"),
    "two models": (False, "(tgir 1 (model m) (model n) (input x (f32 2)) (block (%2 (f32 2) (tanh x))) (output %2))"),
    "zero dimension": (False, BASE.format(params="(param p (f32 0) (data))", block="(%2 (f32 2) (tanh x))", out="%2")),
    "param after block": (False, "(tgir 1 (model m) (input x (f32 2)) (block (%2 (f32 2) (tanh x)))"
                                 " (param p (f32 2) (data 1 2)) (output %2))"),
    "two blocks": (False, "(tgir 1 (model m) (input x (f32 2)) (block (%2 (f32 2) (tanh x)))"
                          " (block (%3 (f32 2) (tanh x))) (output %2))"),
    "output before block": (False, "(tgir 1 (model m) (input x (f32 2)) (output x) (block (%2 (f32 2) (tanh x))))"),
    "two outputs": (False, BASE.format(params=P, block=ADD, out="%2) (output %2")),
    "no output": (False, "(tgir 1 (model m) (input x (f32 2)) (block (%2 (f32 2) (tanh x))))"),
    "trailing form": (False, BASE.format(params="", block="(%2 (f32 2) (tanh x))", out="%2") + " (extra)"),
    "rank 5": (False, BASE.format(params="(param p (f32 1 1 1 1 2) (data 1 2))", block="(%2 (f32 2) (tanh x))",
                                  out="%2")),
    "quant bits": (False, BASE.format(params="(param W (f32 1 2) (quant 5 0 (scale 1) (codes 1 2)))",
                                      block="(%2 (f32 2) (tanh x))", out="%2")),
    "quant axis": (False, BASE.format(params="(param W (f32 1 2) (quant 8 2 (scale 1) (codes 1 2)))",
                                      block="(%2 (f32 2) (tanh x))", out="%2")),
    "int4 code 8": (False, BASE.format(params="(param W (f32 1 2) (quant 4 0 (scale 1) (codes 8 2)))",
                                       block="(%2 (f32 2) (tanh x))", out="%2")),
    "string in data": (False, BASE.format(params='(param p (f32 2) (data 1 "2"))', block=ADD, out="%2")),
    "unterminated": (False, "(tgir 1 (model m) (input x (f32 2)) (block (%2 (f32 2) (tanh x))) (output %2)"),
    "extra close": (False, BASE.format(params="", block="(%2 (f32 2) (tanh x))", out="%2") + ")"),
}


def ours_accepts(src: str) -> bool:
    try:
        m = tgir.read(src)
    except tgir.TgirError:
        return False
    n = C.c_long()
    return _lib.lib().tg_cuda_program_kernel(tgir.CProgram(m).ptr(), None, 0, C.byref(n), 0) != _lib.EINVAL


@pytest.mark.parametrize("name", sorted(CASES))
def test_loads_exactly_what_the_reference_loads(name, tmp_path):
    valid, src = CASES[name]
    assert ours_accepts(src) == valid
    if os.path.exists(TGC):
        mp = tmp_path / "m.tgir"
        mp.write_text(src)
        (tmp_path / "r.csv").write_text("0,0\n")
        r = subprocess.run([TGC, "batch", str(mp), str(tmp_path / "r.csv")], capture_output=True, text=True, timeout=60)
        assert (r.returncode == 0) == valid, r.stderr
