"""The TGIR loader's fast path for params' number lists (the streaming loader of a
quantized model): `(data ...)`, `(scale ...)` and `(codes ...)` are parsed straight into
arrays from a memory map, with no Python object per number. It must give exactly what
the generic reader (an atom per number, as the reference's Sx nodes) gives, and read a
large quantized matrix in memory proportional to its arrays. CPU only."""
import glob
import os
import time
import tracemalloc

import numpy as np
import pytest

from technograd_b200 import tgir


def _same(a: tgir.Module, b: tgir.Module):
    assert len(a.vals) == len(b.vals) and len(a.top) == len(b.top)
    for va, vb in zip(a.vals, b.vals):
        assert (va.kind, tuple(va.shape)) == (vb.kind, tuple(vb.shape))
        for k in ("data", "q", "qs"):
            x, y = getattr(va, k, None), getattr(vb, k, None)
            assert (x is None) == (y is None)
            if x is not None:
                assert np.array_equal(np.asarray(x).view(np.uint8), np.asarray(y).view(np.uint8))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "**", "*.tgir"),
                                               recursive=True)))
def test_fast_reader_matches_generic(path):
    with open(path) as f:
        src = f.read()
    _same(tgir.load(path), tgir.read(src, fast=False))


def _big_quant_src(rows: int, cols: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    codes = rng.integers(-7, 8, size=rows * cols)
    scale = (np.abs(rng.normal(0, 0.02, size=rows)) / 7).astype(np.float32)
    src = "\n".join([
        "(tgir 1",
        "  (model big)",
        f"  (param W (f32 {rows} {cols})",
        "    (quant 4 0",
        "      (scale " + " ".join("%.9g" % v for v in scale) + ")",
        "      (codes " + " ".join(map(str, codes.tolist())) + ")))",
        f"  (input x (f32 {cols}))",
        "  (block",
        f"    (%2 (f32 {rows}) (matmul W x)))",
        "  (output %2))",
        "",
    ])
    return src, codes, scale


def test_large_quantized_param_reads_in_bounded_memory(tmp_path):
    rows, cols = 1024, 4096  # 4.2 M int4 codes, ~11 MB of text
    src, codes, scale = _big_quant_src(rows, cols)
    path = tmp_path / "big.tgir"
    path.write_text(src)
    del src
    tracemalloc.start()
    t0 = time.perf_counter()
    m = tgir.load(str(path))
    dt = time.perf_counter() - t0
    _, peak = tracemalloc.get_traced_memory()
    tracemalloc.stop()
    w = m.vals[0]
    assert w.qbits == 4 and w.qaxis == 0 and tuple(w.shape) == (rows, cols)
    assert np.array_equal(w.q, tgir.pack_codes(codes, 4))
    assert np.array_equal(w.qs, scale)
    want = (codes.reshape(rows, cols).astype(np.float32) * scale[:, None]).ravel()
    assert w.data is None and np.array_equal(w.dense(), want)  # dequantized on demand
    # arrays of the param: codes parsed as int32 (16.8 MB), data f32 (16.8 MB) and its
    # f32 codes (16.8 MB), packed codes (2.1 MB); one atom per number would need > 200 MB
    assert peak < 80 << 20, f"peak {peak >> 20} MB"
    assert dt < 10.0
    tgir.CProgram(m)  # flattens for tg_cuda_load


@pytest.mark.parametrize("payload,msg", [
    ("(data 1 2 x 4)", "bad number"),
    ("(data 1 2", "unterminated"),
])
def test_bad_number_lists_are_rejected(payload, msg):
    src = f"(tgir 1 (model m) (param p (f32 4) {payload}) (input x (f32 4)) (block (%2 (f32 4) (add p x))) (output %2))"
    with pytest.raises(tgir.TgirError, match=msg):
        tgir.read(src)


def test_non_integer_codes_are_rejected():
    src = ("(tgir 1 (model m) (param W (f32 2 2) (quant 8 0 (scale 0.5 0.5) (codes 1 2.5 3 4)))"
           " (input x (f32 2)) (block (%2 (f32 2) (matmul W x))) (output %2))")
    with pytest.raises(tgir.TgirError, match="integers"):
        tgir.read(src)


@pytest.mark.parametrize("chunk", [5, 64])
def test_chunked_number_lists_match_generic(monkeypatch, chunk):
    """Number lists parsed a few bytes at a time (split at whitespace) read exactly as the
    generic reader reads them."""
    monkeypatch.setattr(tgir, "_CHUNK", chunk)
    for path in sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "programs", "*.tgir")))[:12]:
        with open(path) as f:
            src = f.read()
        _same(tgir.load(path), tgir.read(src, fast=False))
    src, codes, scale = _big_quant_src(16, 64)
    m = tgir.read(src)
    assert np.array_equal(m.vals[0].q, tgir.pack_codes(codes, 4)) and np.array_equal(m.vals[0].qs, scale)


@pytest.mark.parametrize("chunk", [3, 1 << 20])
@pytest.mark.parametrize("codes,bits", [("1 2 3 -128", 8), ("1 2 3 300", 8), ("1 -8 3 4", 4), ("1 8 3 4", 4)])
def test_out_of_range_codes_are_rejected(monkeypatch, chunk, codes, bits):
    monkeypatch.setattr(tgir, "_CHUNK", chunk)
    src = (f"(tgir 1 (model m) (param W (f32 2 2) (quant {bits} 0 (scale 0.5 0.5) (codes {codes})))"
           " (input x (f32 2)) (block (%2 (f32 2) (matmul W x))) (output %2))")
    with pytest.raises(tgir.TgirError, match="out of range"):
        tgir.read(src)


@pytest.mark.parametrize("chunk", [2, 1 << 20])
def test_a_bare_sign_at_a_chunk_end_goes_atom_by_atom(monkeypatch, chunk):
    """'1 -' ends a chunk with a sign: not a plain decimal list, so the generic reader
    decides (a bare sign is a symbol, src/sexp.c:112-121, and a symbol among numbers an
    error)."""
    monkeypatch.setattr(tgir, "_CHUNK", chunk)
    src = "(tgir 1 (model m) (param p (f32 3) (data 1 - 2)) (input x (f32 3)) (block (%2 (f32 3) (add p x))) (output %2))"
    with pytest.raises(tgir.TgirError, match="bad number"):
        tgir.read(src)
