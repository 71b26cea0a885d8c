"""The CPU oracle against the reference: golden vectors the reference produced
(tests/golden, made by tests/golden/make_golden.py) and, where oracle/_ref was
built from the reference sources, live calls on fresh seeded inputs."""
import gzip
import os

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import tgir


def test_kernels_match_golden(golden):
    z = np.load(os.path.join(golden, "kernels.npz"))
    L = tgo.tgo()
    i = 0
    while f"mq{i}_meta" in z:
        axis, bits, m, k, n = (int(v) for v in z[f"mq{i}_meta"])
        o = tgo.matmul_q(L, "tgo_", axis, z[f"mq{i}_act"], z[f"mq{i}_q"], bits, z[f"mq{i}_s"], m, k, n)
        assert np.array_equal(o.view(np.uint32), z[f"mq{i}_o"].view(np.uint32)), f"case {i}"
        # the reference packing: code -8 survives, every code decodes back
        codes = tgir.unpack_codes(z[f"mq{i}_q"], bits, z[f"mq{i}_codes"].size)
        assert np.array_equal(codes, z[f"mq{i}_codes"].astype(np.int32))
        i += 1
    assert i >= 8
    o = np.zeros((7, 5), np.float32)
    L.tgo_matmul(tgo.f32p(o), tgo.f32p(z["mm_a"]), tgo.f32p(z["mm_b"]), 7, 13, 5)
    assert np.array_equal(o, z["mm_o"])
    x = z["row_x"]
    rn, sm = np.zeros_like(x), np.zeros_like(x)
    L.tgo_rmsnorm(tgo.f32p(rn), tgo.f32p(x), 6, 37)
    L.tgo_softmax(tgo.f32p(sm), tgo.f32p(x), 6, 37)
    assert np.array_equal(rn, z["rms_o"]) and np.array_equal(sm, z["softmax_o"])


def test_quantizer_matches_golden(golden):
    z = np.load(os.path.join(golden, "quant.npz"))
    for name in ("r8a0", "r8a1", "r4a0", "r4a1", "g4a1", "g8a0", "zero"):
        bits, axis, r, c, gptq = (int(v) for v in z[name + "_meta"])
        H = None
        if gptq:
            K = (r, c)[1 - axis]
            H = np.zeros((K, K))
            tgo.tgo().tgo_hessian_add(H.ctypes.data_as(tgo.DP), tgo.f32p(z[name + "_x"]), z[name + "_x"].shape[0], K)
        q, s = tgo.quantize(tgo.tgo(), "tgo_", z[name + "_w"], axis, bits, H)
        assert np.array_equal(q, z[name + "_q"]), name
        assert np.array_equal(s.view(np.uint32), z[name + "_s"].view(np.uint32)), name


def test_rand_matches_reference_program(golden):
    """rand(seed, scale) of src/lower.c regenerates the f32 params of latent_reasoner."""
    m = tgir.load(os.path.join(golden, "latent_reasoner.f32.tgir"))
    L = tgo.tgo()
    for name, seed, scale in (("w_emb", 11, 0.35), ("w_core", 23, 0.12), ("w_inj", 37, 0.10), ("w_out", 41, 0.5)):
        v = next(x for x in m.vals if x.name == name)
        out = np.zeros(v.numel, np.float32)
        L.tgo_rand(seed, scale, tgo.f32p(out), v.numel)
        assert np.array_equal(out, v.data), name


def _batch_golden(path):
    rows = np.loadtxt(path, delimiter=",", dtype=np.float64)
    return rows[:, :-1].astype(np.float32), rows[:, -1].astype(np.int32)


@pytest.mark.parametrize("tag", ["f32", "q8"])
def test_program_vm_matches_tgc_batch(golden, tag):
    m = tgir.load(os.path.join(golden, f"latent_reasoner.{tag}.tgir"))
    prog = tgir.CProgram(m)
    rows = np.loadtxt(os.path.join(golden, "lr_rows.csv"), delimiter=",", dtype=np.float32)
    out, steps = tgo.program_run(prog, rows)
    want, want_steps = _batch_golden(os.path.join(golden, f"lr_{tag}_out.csv"))
    # text output holds %.9g, which round-trips f32 exactly
    assert np.array_equal(out, want)
    assert np.array_equal(steps[:, 0], want_steps)


def test_readme_golden_and_ops(golden):
    m = tgir.load(os.path.join(golden, "latent_reasoner.f32.tgir"))
    out, steps = tgo.program_run(tgir.CProgram(m), np.array([1, 0, 0, 1, 0, 1, 1, 0], np.float32))
    # README.md:48-51 of the reference
    assert [f"{v:.9g}" for v in out[0]] == ["0.225605994", "0.24476327", "0.162138939", "0.367491812"]
    assert steps[0, 0] == 9
    ops = tgir.load(os.path.join(golden, "ops.tgir"))
    want = np.array(open(os.path.join(golden, "ops_expected.txt")).read().split(), np.float64).astype(np.float32)
    out, _ = tgo.program_run(tgir.CProgram(ops), np.array([1, -2, 3, 0.5], np.float32))  # tests/run.sh:32
    assert np.array_equal(out[0], want)


def test_live_reference_kernels():
    R = tgo.ref()
    if R is None:
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    rng = np.random.default_rng(123)
    for axis, bits, m, k, n in ((0, 4, 9, 23, 3), (1, 4, 4, 19, 21), (1, 8, 6, 40, 9), (0, 8, 3, 64, 5)):
        codes = rng.integers(-8 if bits == 4 else -127, 8 if bits == 4 else 128, size=m * k if axis == 0 else k * n)
        q = tgir.pack_codes(codes, bits)
        s = rng.random(m if axis == 0 else n).astype(np.float32)
        act = rng.normal(size=k * n if axis == 0 else m * k).astype(np.float32)
        a = tgo.matmul_q(tgo.tgo(), "tgo_", axis, act, q, bits, s, m, k, n)
        b = tgo.matmul_q(R, "ref_", axis, act, q, bits, s, m, k, n)
        assert np.array_equal(a, b)
    for bits, axis in ((8, 0), (4, 1), (4, 0)):
        w = rng.normal(0, 0.05, size=(20, 36)).astype(np.float32)
        K = w.shape[1 - axis]
        x = rng.normal(size=(50, K)).astype(np.float32)
        H = np.zeros((K, K))
        tgo.tgo().tgo_hessian_add(H.ctypes.data_as(tgo.DP), tgo.f32p(x), 50, K)
        for h in (None, H):
            qa, sa = tgo.quantize(tgo.tgo(), "tgo_", w, axis, bits, h)
            qb, sb = tgo.quantize(R, "ref_", w, axis, bits, h)
            assert np.array_equal(qa, qb) and np.array_equal(sa, sb)


def _nano_cfg(golden):
    kv = dict(x.split("=") for x in open(os.path.join(golden, "nano", "config.txt")).read().split())
    return {k: (float(v) if k == "theta" else int(v)) for k, v in kv.items()}


@pytest.mark.parametrize("tag", ["q8", "q4", "q4gptq"])
def test_lm_oracle_matches_tgc_on_the_qwen3_program(golden, tag):
    """tgo_lm_forward restates the program examples/qwen3/import.py emits; the reference
    ran that program (quantized by `tgc quantize`) through `tgc batch`."""
    import ctypes as C

    from technograd_b200 import lm
    cfg = _nano_cfg(golden)
    model = lm.Model.from_tgir(os.path.join(golden, "nano", f"{tag}.tgir.gz"), cfg)
    d, keep = model.desc()
    ids = np.loadtxt(os.path.join(golden, "nano", "ids.csv"), delimiter=",", dtype=np.float32)
    want = np.loadtxt(os.path.join(golden, "nano", f"{tag}_logits.csv"), delimiter=",", dtype=np.float64).astype(np.float32)
    L = tgo.tgo()
    for r in range(ids.shape[0]):
        out = np.zeros(cfg["vocab"], np.float32)
        L.tgo_lm_forward(C.addressof(d), tgo.f32p(np.ascontiguousarray(ids[r])), ids.shape[1], tgo.f32p(out))
        np.testing.assert_allclose(out, want[r], rtol=1e-5, atol=1e-6)
        assert out.argmax() == want[r].argmax()
