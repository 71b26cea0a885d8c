"""The `tgc batch` driver's input and output handling (technograd_b200/batch.py) against the
reference's own `tgc` (oracle/_ref/tgc, built from its sources), on the CPU: text rows are read
as glibc's strtof reads them (src/io.c:25-41) -- hex floats, inf/nan forms, signs, numbers on
an f32 rounding midpoint -- and rejected where the reference rejects them, binary streams must
hold whole f32 values, and text output is printf's "%.9g" (src/io.c:79-92)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from technograd_b200 import batch, tgir

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TGC = os.path.join(ROOT, "oracle", "_ref", "tgc")
needs_tgc = pytest.mark.skipif(not os.path.exists(TGC), reason="oracle/_ref/tgc is built only where the reference sources are")

# y = x + 0: the program hands its input back, so `tgc batch` to a .bin file shows the exact
# f32 values it parsed (x86 addition keeps a NaN's sign and payload)
IDENT = """(tgir 1
  (model ident)
  (param z (f32 2)
    (data 0 0))
  (input x (f32 2))
  (block
    (%2 (f32 2) (add x z)))
  (output %2))
"""

ROWS_OK = [
    "1.5, -2",
    "  0x1.8p3\t+.25 ",
    "inf,-INFINITY",
    "nan, -nan",
    "NaN(12) 1e-50",
    "1e40 -1e-46",
    "1.00000005960464477539062500000000001 16777217",  # just above an f32 midpoint; 2^24 + 1
    "0.1 2 # a comment, 3",
    "",
    "   # only a comment",
    "3.4028235677973366e38 1.40129846432481707e-45",
    "7.,0x10",
]
ROWS_BAD = ["1_000 2", "1.5abc 2", "0x 1", "1e 2", "nan( 2", "- 1", "infin 2", "1;2"]


def run_tgc(tmp_path, model_src: str, data: str, out_name: str):
    mp = tmp_path / "m.tgir"
    mp.write_text(model_src)
    dp = tmp_path / "rows.csv"
    dp.write_text(data)
    op = tmp_path / out_name
    r = subprocess.run([TGC, "batch", str(mp), str(dp), "-j", "1", "-o", str(op)], capture_output=True, text=True,
                       timeout=60)
    return r, op


@needs_tgc
def test_text_rows_parse_as_the_reference_parses_them(tmp_path):
    data = "\n".join(ROWS_OK) + "\n"
    r, op = run_tgc(tmp_path, IDENT, data, "out.bin")
    assert r.returncode == 0, r.stderr
    want = np.fromfile(op, dtype="<f4").reshape(-1, 2)
    got = batch.load_samples(str(tmp_path / "rows.csv"), 2, "ident")
    got = got + np.zeros(2, np.float32)  # the program's own addition
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (got, want)


@needs_tgc
@pytest.mark.parametrize("row", ROWS_BAD)
def test_bad_numbers_are_rejected_like_the_reference(tmp_path, row):
    r, _ = run_tgc(tmp_path, IDENT, "1 2\n" + row + "\n", "out.bin")
    assert r.returncode != 0 and "bad number" in r.stderr
    with pytest.raises(ValueError, match=r"rows.csv:2: bad number near"):
        batch.load_samples(str(tmp_path / "rows.csv"), 2, "ident")


@needs_tgc
def test_row_width_errors_name_the_model(tmp_path):
    r, _ = run_tgc(tmp_path, IDENT, "1 2\n1 2 3\n", "out.bin")
    assert r.returncode != 0 and "row has 3 values, model ident needs 2 per sample" in r.stderr
    with pytest.raises(ValueError, match="rows.csv:2: row has 3 values, model ident needs 2 per sample"):
        batch.load_samples(str(tmp_path / "rows.csv"), 2, "ident")


@needs_tgc
def test_text_output_is_printf_g9(tmp_path):
    vals = ["1.5 -0", "0.1 1e-45", "inf -inf", "nan -nan", "123456789 3.14159265"]
    r, op = run_tgc(tmp_path, IDENT, "\n".join(vals) + "\n", "out.csv")
    assert r.returncode == 0, r.stderr
    rows = batch.load_samples(str(tmp_path / "rows.csv"), 2, "ident") + np.zeros(2, np.float32)
    mine = tmp_path / "mine.csv"
    batch.write_rows(str(mine), rows, np.zeros((rows.shape[0], 0), np.int32))
    assert mine.read_text() == op.read_text()


def test_binary_streams_hold_whole_values(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(np.arange(6, dtype="<f4").tobytes() + b"\x00")
    with pytest.raises(ValueError, match="7 bytes|25 bytes"):
        batch.load_samples(str(p), 2)
    p.write_bytes(np.arange(6, dtype="<f4").tobytes())
    assert batch.load_samples(str(p), 2).tolist() == [[0, 1], [2, 3], [4, 5]]
    with pytest.raises(ValueError, match="6 values is not a multiple of the 4 per sample"):
        batch.load_samples(str(p), 4)


def test_binary_extension_is_the_last_dot():
    assert batch.is_binary("a.bin") and batch.is_binary("dir.x/a.f32") and not batch.is_binary("a.bin.csv")
    assert not batch.is_binary("dir.bin/rows")


def test_every_golden_rows_file_reads_as_before(golden):
    """The fixtures' rows (plain decimals) read the same as a plain float conversion gives."""
    import glob
    for p in sorted(glob.glob(os.path.join(golden, "programs", "*_rows.csv"))):
        per = tgir.load(p.replace("_rows.csv", ".tgir")).per
        plain = np.loadtxt(p, delimiter=",", dtype=np.float64, ndmin=2).astype(np.float32)
        got = batch.load_samples(p, per)
        assert np.array_equal(got.view(np.uint32), plain.view(np.uint32)) or np.array_equal(got, plain, equal_nan=True)


@pytest.mark.parametrize("rows,msg", [("1 2\n1 x\n", "bad number near 'x'"),
                                      ("1 2\n1 2 3\n", "row has 3 values, model ident needs 2 per sample")])
def test_bad_input_fails_before_the_output_exists(tmp_path, rows, msg):
    """src/main.c:414-419: the whole input is validated before any compute and before the
    output file is created, so a failed run leaves no partial output."""
    mp, dp, op = tmp_path / "m.tgir", tmp_path / "rows.csv", tmp_path / "out.csv"
    mp.write_text(IDENT)
    dp.write_text(rows)
    r = subprocess.run([sys.executable, "-m", "technograd_b200.batch", str(mp), str(dp), "-o", str(op)],
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 1 and msg in r.stderr and r.stderr.startswith("error: ")
    assert not op.exists()
    if os.path.exists(TGC):
        r = subprocess.run([TGC, "batch", str(mp), str(dp), "-o", str(op)], capture_output=True, text=True, timeout=60)
        assert r.returncode != 0 and msg in r.stderr and not op.exists()


def test_bad_model_fails_before_the_output_exists(tmp_path):
    mp, dp, op = tmp_path / "m.tgir", tmp_path / "rows.csv", tmp_path / "out.csv"
    mp.write_text(IDENT.replace("(data 0 0)", "(data 0 0 0)"))
    dp.write_text("1 2\n")
    r = subprocess.run([sys.executable, "-m", "technograd_b200.batch", str(mp), str(dp), "-o", str(op)],
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 1 and "needs 2 values, has 3" in r.stderr
    assert not op.exists()


def test_rows_from_standard_input_and_missing_files(tmp_path):
    """src/util.c:100-103: DATA "-" is standard input; a missing file is "cannot open"."""
    mp = tmp_path / "m.tgir"
    mp.write_text(IDENT)
    r = subprocess.run([sys.executable, "-m", "technograd_b200.batch", str(mp), "-"], input="1 2\n1 y\n",
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 1 and "-:2: bad number near 'y'" in r.stderr
    r = subprocess.run([sys.executable, "-m", "technograd_b200.batch", str(mp), str(tmp_path / "none.csv")],
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 1 and r.stderr.startswith("error: cannot open '")
    r = subprocess.run([sys.executable, "-m", "technograd_b200.batch", str(tmp_path / "none.tgir"), "-"], input="1 2\n",
                       capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 1 and r.stderr.startswith("error: cannot open '")
    import io
    old = sys.stdin
    try:
        sys.stdin = io.TextIOWrapper(io.BytesIO(b"0x1p1, 3 # rows from stdin\n"))
        assert batch.load_samples("-", 2).tolist() == [[2.0, 3.0]]
    finally:
        sys.stdin = old


def test_unwritable_output_fails_before_compute(tmp_path):
    """src/main.c:64-68: an output path that cannot be written ends the run before any
    compute (here: before a GPU is touched), with the reference's wording."""
    mp, dp = tmp_path / "m.tgir", tmp_path / "rows.csv"
    mp.write_text(IDENT)
    dp.write_text("1 2\n")
    for bad in (tmp_path / "no_such_dir" / "out.csv", tmp_path):
        r = subprocess.run([sys.executable, "-m", "technograd_b200.batch", str(mp), str(dp), "-o", str(bad)],
                           capture_output=True, text=True, timeout=120, cwd=ROOT)
        assert r.returncode == 1 and r.stderr.startswith("error: cannot write '"), r.stderr


@pytest.mark.parametrize("suffix", [".csv", ".bin"])
def test_main_writes_what_write_rows_writes(tmp_path, monkeypatch, suffix):
    """The output the CLI opens before compute (src/main.c:414-419) holds exactly what
    write_rows writes for the same rows, as text or as binary f32; the device is stubbed."""
    mp, dp = tmp_path / "m.tgir", tmp_path / "rows.csv"
    mp.write_text(IDENT)
    dp.write_text("1 2\n3 4\n")
    out = np.array([[0.5, -1.25], [3.0, 1e-9]], np.float32)
    steps = np.zeros((2, 0), np.int32)

    class Stub:
        def __init__(self, module, gpus=0):
            pass

        def run(self, rows):
            assert rows.shape[0] == 2
            return out, steps

    monkeypatch.setattr(batch, "Batch", Stub)
    got, want = tmp_path / ("got" + suffix), tmp_path / ("want" + suffix)
    assert batch.main([str(mp), str(dp), "-o", str(got)]) == 0
    batch.write_rows(str(want), out, steps)
    assert got.read_bytes() == want.read_bytes()
