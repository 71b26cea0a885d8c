"""The streaming loader at full size (GPU): a `tgc quantize`-form TGIR of the whole
Qwen3-0.6B architecture (28 layers, vocab 151,936; 596 M int4 codes, a 155 M-value
embedding, ~2.7 GB of text) read by tgir.load through a memory map into packed codes,
turned into the engine's model (lm.Model.from_tgir), loaded on the GPU and run.

- every param reads back exactly: codes, scales (printed %.9g, so the f32 round-trips)
  and f32 data, against the arrays the file was written from;
- the loader's peak Python-heap allocation stays under 5 GB (the text is never held as
  a string, and quantized params are never expanded to f32);
- the logits of the last position of two 128-token prompts are within 1e-3 relative +
  1e-4 absolute of the oracle's (tgo_lm_forward_mt) over all 151,936 entries, and a
  greedy token of the engine equals the oracle's argmax (or the oracle's top two are
  within that tolerance).

The file is written by oracle/qwen3_tgir.py (pinned against a TGIR the reference wrote,
tests/test_qwen3_tgir.py) from seeded random codes: uniform int4 codes in [-7, 7],
per-channel scales 0.02 * U(0.5, 1.5) / 7, the embedding k / 16 for uniform k in
[-8, 8], norm weights 1 + 0.05 N(0, 1) rounded to 1/64."""
import ctypes as C
import os
import time
import tracemalloc

import numpy as np
import pytest

from oracle import qwen3_tgir, tgo
from technograd_b200 import lm

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-3, 1e-4
CFG = lm.QWEN3_0_6B
T_PROGRAM = 1024


def synthetic(cfg: dict, seed: int):
    rng = np.random.default_rng(seed)
    D, HD, FF, V = cfg["hidden"], cfg["head_dim"], cfg["ffn"], cfg["vocab"]
    f32, quant = {}, {}
    emb = (np.arange(-8, 9) / 16).astype(np.float32)
    f32["E"] = (rng.integers(0, 17, size=V * D, dtype=np.int8), emb)

    def norm(n):
        return (np.round((1 + 0.05 * rng.standard_normal(n)) * 64) / 64).astype(np.float32)

    for name in qwen3_tgir.param_names(cfg):
        shape = qwen3_tgir.param_shape(cfg, name, T_PROGRAM)
        if lm.is_linear(name):
            codes = rng.integers(-7, 8, size=shape[0] * shape[1], dtype=np.int8)
            scales = (0.02 * rng.uniform(0.5, 1.5, size=shape[1]) / 7).astype(np.float32)
            quant[name] = (codes, scales, 4)
        elif name.split("_")[0] in ("lnf", "ln1", "ln2", "qn", "kn"):
            f32[name] = norm(shape[0])
    return f32, quant


@pytest.fixture(scope="module")
def full(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("tgir") / "qwen3_0_6b_q4.tgir")
    f32, quant = synthetic(CFG, seed=17)
    t0 = time.time()
    qwen3_tgir.write(path, CFG, T_PROGRAM, f32, quant)
    t1 = time.time()
    tracemalloc.start()
    model = lm.Model.from_tgir(path, CFG)
    peak = tracemalloc.get_traced_memory()[1]
    tracemalloc.stop()
    t2 = time.time()
    print(f"\nwrote {os.path.getsize(path) / 1e9:.2f} GB in {t1 - t0:.0f} s; loaded in {t2 - t1:.0f} s, "
          f"peak Python-heap {peak / 1e9:.2f} GB")
    os.unlink(path)
    return model, f32, quant, peak


def test_params_read_back_exactly(full):
    model, f32, quant, peak = full
    assert model.bits == 4 and set(model.q) == set(quant)
    for name, (codes, scales, _) in quant.items():
        p = model.q[name]
        assert np.array_equal(p.codes().ravel(), codes), name
        assert np.array_equal(p.s.view(np.uint32), scales.view(np.uint32)), name
    idx, emb = f32["E"]
    assert np.array_equal(model.f32["E"].ravel(), emb[idx])
    for name, v in f32.items():
        if name != "E":
            assert np.array_equal(model.f32[name].ravel(), v), name
    assert peak < 5e9, f"loader peak {peak / 1e9:.2f} GB"


def test_engine_runs_the_loaded_model(cuda, full):
    model = full[0]
    eng = lm.Engine(model, max_seqs=2, max_len=160)
    rng = np.random.default_rng(3)
    ids = rng.integers(0, CFG["vocab"], size=(2, 128)).astype(np.float32)
    got = eng.forward(ids)
    toks = eng.generate(ids, 1)
    desc, keep = model.desc()
    for s in range(2):
        want = np.zeros(CFG["vocab"], np.float32)
        x = np.ascontiguousarray(ids[s])
        assert tgo.tgo().tgo_lm_forward_mt(C.addressof(desc), tgo.f32p(x), x.size, tgo.f32p(want), 0) == 0
        np.testing.assert_allclose(got[s], want, rtol=RTOL, atol=ATOL)
        t = int(toks[s, 0])
        top2 = np.sort(want)[-2:]
        assert t == int(want.argmax()) or (top2[1] - top2[0] <= ATOL + RTOL * abs(top2[1]) and want[t] >= top2[0])
    del keep
