"""Numbers in TGIR params as the reference's reader takes them (src/sexp.c:112-121,
src/ir.c:484-521): an atom is a number when strtod consumes all of it and it starts with a
digit, or with a sign or '.' and is longer than one character. Checked against the
reference's own `tgc` on CPU, through both of our readers (the fast array path and the
atom-by-atom one)."""
import os
import subprocess

import numpy as np
import pytest

from technograd_b200 import tgir

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TGC = os.path.join(ROOT, "oracle", "_ref", "tgc")
pytestmark = pytest.mark.skipif(not os.path.exists(TGC), reason="oracle/_ref/tgc is built only where the reference sources are")


def model(values: list[str]) -> str:
    n = len(values)
    return (f"(tgir 1 (model nums) (param p (f32 {n}) (data {' '.join(values)})) (input x (f32 {n}))"
            f" (block (%2 (f32 {n}) (add x p))) (output %2))")


def quant_model(codes: list[str], bits: int = 8) -> str:
    n = len(codes)
    return (f"(tgir 1 (model q) (param W (f32 1 {n}) (quant {bits} 0 (scale 0.5) (codes {' '.join(codes)})))"
            f" (input x (f32 1 {n})) (block (%2 (f32 1 {n}) (add x W))) (output %2))")


def tgc_values(tmp_path, src: str, n: int):
    """The param as `tgc batch` computes x + p on a zero row, or None when tgc rejects the file."""
    mp, dp, op = tmp_path / "m.tgir", tmp_path / "zero.csv", tmp_path / "o.bin"
    mp.write_text(src)
    dp.write_text(",".join(["0"] * n) + "\n")
    r = subprocess.run([TGC, "batch", str(mp), str(dp), "-o", str(op)], capture_output=True, text=True, timeout=60)
    return np.fromfile(op, dtype="<f4") if r.returncode == 0 else None


GOOD = ["0x10", "+inf", "-inf", "-nan", "+nan", "1e5", ".5", "+.5", "-.5", "5.", "1.e2", "0x1.8p1", "1E-3",
        "3.4028235677973366e38", "1e-46", "1e400", "-0", "00012", "0.1"]
BAD = ["inf", "nan", "1_0", "0x", "1e", "+", ".", "1.2.3", "--1", "infinity"]


@pytest.mark.parametrize("fast", [True, False])
def test_accepted_numbers_read_as_the_reference_reads_them(tmp_path, fast):
    src = model(GOOD)
    want = tgc_values(tmp_path, src, len(GOOD))
    assert want is not None
    p = tgir.read(src, fast=fast).vals[0].data.astype(np.float32)
    got = np.zeros(len(GOOD), np.float32) + p
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (got, want)


@pytest.mark.parametrize("fast", [True, False])
@pytest.mark.parametrize("tok", BAD)
def test_rejected_numbers_are_rejected(tmp_path, fast, tok):
    src = model(["1", tok, "2"])
    assert tgc_values(tmp_path, src, 3) is None
    with pytest.raises(tgir.TgirError):
        tgir.read(src, fast=fast)


@pytest.mark.parametrize("fast", [True, False])
def test_codes_as_the_reference_reads_them(tmp_path, fast):
    codes = ["+5", "5.", "1e1", "-0x7f", "0", "-127"]
    src = quant_model(codes)
    want = tgc_values(tmp_path, src, len(codes))
    assert want is not None
    w = tgir.read(src, fast=fast).vals[0]
    assert np.array_equal(np.zeros(len(codes), np.float32) + w.dense().astype(np.float32), want)
    for bad in (["+", "1", "2"], ["1.5", "1", "2"], ["128", "1", "2"], ["nan", "1", "2"]):
        src = quant_model(bad)
        assert tgc_values(tmp_path, src, 3) is None
        with pytest.raises(tgir.TgirError):
            tgir.read(src, fast=fast)
