"""The Qwen3 TGIR writer the full-size loader test uses (oracle/qwen3_tgir.py), pinned
against a TGIR the reference wrote (tests/golden/nano/q4.tgir.gz: examples/qwen3/import.py
run through `tgc quantize`): the block is the reference's line for line, the params come
in its order with its shapes, its rotary tables and mask are the reference's values bit
for bit, and a file written from the fixture's own params reads back to the same module
(and to the same Model, whose oracle logits match the reference's recorded ones). CPU."""
import gzip
import io
import os
import re

import numpy as np
import pytest

from oracle import qwen3_tgir
from technograd_b200 import _lib, lm, tgir


def _cfg(golden):
    kv = dict(x.split("=") for x in open(os.path.join(golden, "nano", "config.txt")).read().split())
    return {k: (float(v) if k == "theta" else int(v)) for k, v in kv.items()}


def _fixture(golden, tag="q4"):
    with gzip.open(os.path.join(golden, "nano", f"{tag}.tgir.gz"), "rb") as f:
        return f.read().decode()


def test_block_is_the_references(golden):
    cfg = _cfg(golden)
    src = _fixture(golden)
    want = src[src.index("  (block\n"):].splitlines()
    names = qwen3_tgir.param_names(cfg)
    ins = qwen3_tgir.block(cfg, cfg["T"], len(names) + 1)
    got = ["  (block"]
    for v, shape, name, args in ins:
        inner = f"({name} {args[0]})" if name == "const" else f"({name} {' '.join(args)})"
        got.append(f"    ({v} {qwen3_tgir._shape(shape)} {inner})")
    got += ["  )", f"  (output %{len(names) + len(ins)}))"]
    assert got == want


def test_params_order_shapes_and_tables(golden):
    cfg = _cfg(golden)
    T = cfg["T"]
    m = tgir.read(_fixture(golden))
    params = [v for v in m.vals if v.kind == _lib.PARAM]
    assert [v.name for v in params] == qwen3_tgir.param_names(cfg)
    assert [tuple(v.shape) for v in params] == [qwen3_tgir.param_shape(cfg, v.name, T) for v in params]
    assert re.findall(r"\(param (\S+) \(f32[^)]*\)\n    \(quant", _fixture(golden)) == \
        [v.name for v in params if lm.is_linear(v.name)]
    tab = qwen3_tgir.tables(T, cfg["head_dim"], cfg["theta"])
    for v in params:
        if v.name in tab:
            assert np.array_equal(v.data.view(np.uint32), tab[v.name].ravel().view(np.uint32)), v.name


@pytest.mark.parametrize("tag", ["q4", "q8", "q4gptq"])
def test_written_file_reads_back_to_the_fixture(golden, tmp_path, tag):
    cfg = _cfg(golden)
    ref = tgir.read(_fixture(golden, tag))
    f32, quant = {}, {}
    for v in ref.vals:
        if v.kind != _lib.PARAM:
            continue
        if v.qbits:
            quant[v.name] = (tgir.unpack_codes(v.q, v.qbits, v.numel), v.qs, v.qbits)
        else:
            f32[v.name] = v.data
    path = str(tmp_path / "w.tgir")
    qwen3_tgir.write(path, cfg, cfg["T"], f32, quant)
    got = tgir.load(path)
    assert (got.name, len(got.vals), got.output, got.inputs) == (ref.name, len(ref.vals), ref.output, ref.inputs)
    for a, b in zip(got.vals, ref.vals):
        assert (a.kind, a.shape, a.name, a.qbits, a.qaxis) == (b.kind, b.shape, b.name, b.qbits, b.qaxis)
        for k in ("data", "q", "qs"):
            x, y = getattr(a, k), getattr(b, k)
            assert (x is None) == (y is None), (a.name, k)
            if x is not None:
                assert np.array_equal(np.asarray(x).view(np.uint8), np.asarray(y).view(np.uint8)), (a.name, k)
    assert [(i.op, i.out, i.a, i.k) for i in got.top] == [(i.op, i.out, i.a, i.k) for i in ref.top]
    # the same Model (the loader path of the full-size test) as from the reference's file
    ma, mb = lm.Model.from_tgir(path, cfg), lm.Model.from_tgir(os.path.join(golden, "nano", f"{tag}.tgir.gz"), cfg)
    assert ma.bits == mb.bits and ma.f32.keys() == mb.f32.keys() and ma.q.keys() == mb.q.keys()
    for k in ma.q:
        assert np.array_equal(ma.q[k].q, mb.q[k].q) and np.array_equal(ma.q[k].s, mb.q[k].s)


def _numbers(a, **kw) -> list:
    f = io.BytesIO()
    qwen3_tgir._write_numbers(f, a, **kw)
    return f.getvalue().split()


def test_number_formatting():
    """integers as integers, the rest as %.9g of the f32 value (src/ir.c's printing): one by
    one, through the token table in chunks, and as indexed values"""
    c = np.array([-7, 0, 7, 3, -1], np.int8)
    assert _numbers(c, chunk=2) == [b"-7", b"0", b"7", b"3", b"-1"]
    assert _numbers(np.array([0, 70000], np.int64)) == [b"0", b"70000"]
    x = np.random.default_rng(0).standard_normal(500).astype(np.float32)
    toks = _numbers(x)
    assert toks == [("%.9g" % float(v)).encode() for v in x]
    assert np.array_equal(np.array([float(t) for t in toks], np.float32), x)
    vals = np.array([0.5, -0.0625, 1e-9], np.float32)
    idx = np.array([2, 0, 0, 1, 2], np.int8)
    assert _numbers((idx, vals), chunk=3) == [("%.9g" % float(vals[i])).encode() for i in idx]
