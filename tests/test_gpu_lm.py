"""The decoder engine (tg_cuda_lm_*) against the oracle restatement of the Qwen3
program (tgo_lm_forward, pinned to the reference's `tgc batch` output in
test_oracle.py). GPU.

Logits: |gpu - oracle| <= 1e-4 + 1e-3 |oracle| (north_star tolerance). Greedy
decode: every generated token is checked by re-running the oracle's prefill on
the GPU's own prefix (teacher forcing) and comparing argmax tokens; positions
whose top-2 logit gap is below the logit tolerance are excused, and at least
99.9% must match overall."""
import ctypes as C

import numpy as np
import pytest

from oracle import tgo
from technograd_b200 import lm

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-3, 1e-4
MICRO = dict(layers=2, hidden=256, nq=4, nkv=2, head_dim=128, ffn=512, vocab=1000, theta=1e6)


def oracle_logits(model, ids):
    d, keep = model.desc()
    out = np.zeros((ids.shape[0], model.cfg["vocab"]), np.float32)
    for r in range(ids.shape[0]):
        row = np.ascontiguousarray(ids[r], np.float32)
        tgo.tgo().tgo_lm_forward(C.addressof(d), tgo.f32p(row), ids.shape[1], out[r].ctypes.data_as(tgo.FP))
    return out


@pytest.fixture(scope="module", params=[8, 4])
def micro(request, cuda):
    w = lm.random_weights(MICRO, seed=11, norm_jitter=0.1)
    w["E"] = np.random.default_rng(12).standard_normal(w["E"].shape).astype(np.float32)  # unit embeddings
    return lm.quantize_rtn_device(w, MICRO, request.param)


def test_prefill_logits_vs_oracle(micro):
    rng = np.random.default_rng(3)
    # query tiles of 128 and key tiles of 64: T = 77 is one partial query tile, 300 three
    # query tiles (the last partial) over five key tiles
    for T in (1, 5, 64, 77, 128, 300):
        ids = rng.integers(0, MICRO["vocab"], size=(3, T)).astype(np.float32)
        eng = lm.Engine(micro, max_seqs=4, max_len=320)
        got = eng.forward(ids)
        want = oracle_logits(micro, ids)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL, err_msg=f"T={T}")


def test_out_of_range_ids_embed_zero(micro):
    ids = np.array([[-3, 5, 1e9, 7.4, 999.5]], np.float32)  # take(): rounded, out of range -> zero row
    got = lm.Engine(micro, max_seqs=2, max_len=16).forward(ids)
    np.testing.assert_allclose(got, oracle_logits(micro, ids), rtol=RTOL, atol=ATOL)


def test_generate_teacher_forced(micro):
    rng = np.random.default_rng(5)
    S, T, nnew = 6, 20, 12
    ids = rng.integers(0, MICRO["vocab"], size=(S, T)).astype(np.float32)
    eng = lm.Engine(micro, max_seqs=4, max_len=T + nnew)  # two waves of sequences
    tok = eng.generate(ids, nnew)
    assert tok.shape == (S, nnew) and (tok >= 0).all() and (tok < MICRO["vocab"]).all()
    match = total = 0
    for step in range(nnew):
        prefix = np.concatenate([ids, tok[:, :step].astype(np.float32)], axis=1)
        want = oracle_logits(micro, prefix)
        for s in range(S):
            total += 1
            top2 = np.sort(want[s])[-2:]
            if tok[s, step] == want[s].argmax():
                match += 1
            else:
                assert top2[1] - top2[0] <= ATOL + RTOL * abs(top2[1]), f"seq {s} step {step}"
                match += 0
    assert match / total >= 0.999 or total - match <= 1


def test_code_weights_match_bf16_weights(micro, monkeypatch):
    """With TG_CUDA_CODES_ROWS=128 the tensor-core GEMMs of at most 128 rows read the weights
    as packed codes, expanded inside the GEMM (o_proj: the hi/lo of code * per-head scale, as
    the load-time copy holds them); the bf16 copies give the same bits. Prefill of 3 x 40 =
    120 rows (every GEMM on codes), of 3 x 60 (180 rows: the layers on bf16, the 3-row head on
    codes), and greedy decode of 3 rows (the GEMVs off in both engines)."""
    rng = np.random.default_rng(9)
    short = rng.integers(0, MICRO["vocab"], size=(3, 40)).astype(np.float32)
    long_ = rng.integers(0, MICRO["vocab"], size=(3, 60)).astype(np.float32)
    monkeypatch.setenv("TG_CUDA_GEMV_ROWS", "0")
    res = {}
    for rows in ("128", "0"):
        monkeypatch.setenv("TG_CUDA_CODES_ROWS", rows)
        eng = lm.Engine(micro, max_seqs=4, max_len=72)
        eng.profile(True)
        a = eng.forward(short)
        wb = eng.stats()["gemm_weight_bytes"]
        b = eng.forward(long_)
        t = eng.generate(short, 8)
        res[rows] = (a, b, t, wb)
    for i in range(2):
        assert np.array_equal(res["128"][i].view(np.uint32), res["0"][i].view(np.uint32))
    assert np.array_equal(res["128"][2], res["0"][2])
    # codes: a quarter (int4) or half (int8) of the bf16 bytes, o_proj's two planes included
    assert 0 < res["128"][3] < (0.3 if micro.bits == 4 else 0.55) * res["0"][3]


@pytest.mark.parametrize("S,T", [(1, 1), (5, 1), (1, 8), (2, 4), (8, 1)])
def test_gemv_batches_vs_oracle(micro, S, T):
    """Batches of at most 8 rows (S x T) run every layer product as a dequant GEMV over the
    packed codes (1, 5 and 8 rows: the 1-, 8- and 8-column kernels, padding included); logits
    against the oracle."""
    ids = np.random.default_rng(100 + S * T).integers(0, MICRO["vocab"], size=(S, T)).astype(np.float32)
    eng = lm.Engine(micro, max_seqs=8, max_len=16)
    eng.profile(True)
    got = eng.forward(ids)
    st = eng.stats()
    np.testing.assert_allclose(got, oracle_logits(micro, ids), rtol=RTOL, atol=ATOL)
    # the layers' weight bytes are the codes' (+ scales); the head reads its bf16 copy
    D, FF, V, HQ = MICRO["hidden"], MICRO["ffn"], MICRO["vocab"], MICRO["nq"] * MICRO["head_dim"]
    HQKV = (MICRO["nq"] + 2 * MICRO["nkv"]) * MICRO["head_dim"]
    want = MICRO["layers"] * (HQKV * D + D * HQ + 2 * FF * D + D * FF) * micro.bits / 8 + V * D * 2
    assert want <= st["gemm_weight_bytes"] < 1.1 * want


@pytest.mark.parametrize("T", [500, 20])
def test_decode_split_keys_teacher_forced(micro, T):
    """Waves that fill few SMs split each decode step's attention over key ranges of 64k keys
    (here 3 sequences x 2 KV heads: 8 ranges at max_len 600) and combine the ranges' maxima,
    sums and partial outputs. T = 500: every range used, the last one partly; T = 20: one range
    holds every key and seven are empty. Greedy tokens teacher-forced against the oracle."""
    rng = np.random.default_rng(21)
    S, nnew = 3, 5
    ids = rng.integers(0, MICRO["vocab"], size=(S, T)).astype(np.float32)
    tok = lm.Engine(micro, max_seqs=S, max_len=600).generate(ids, nnew)
    for step in range(nnew):
        want = oracle_logits(micro, np.concatenate([ids, tok[:, :step].astype(np.float32)], axis=1))
        for s in range(S):
            if tok[s, step] != want[s].argmax():
                top2 = np.sort(want[s])[-2:]
                assert top2[1] - top2[0] <= ATOL + RTOL * abs(top2[1]), f"seq {s} step {step}"


def test_generate_consistent_with_prefill(micro):
    """The decode path (KV cache, one token per step) agrees with a fresh prefill of the same
    prefix: every token is the prefill's argmax, or (both paths being within the logit
    tolerance of the oracle, so within twice it of each other) one of the prefill's top two
    whose logits lie within twice the tolerance."""
    rng = np.random.default_rng(8)
    ids = rng.integers(0, MICRO["vocab"], size=(4, 9)).astype(np.float32)
    eng = lm.Engine(micro, max_seqs=4, max_len=32)
    tok = eng.generate(ids, 6)
    for step in range(6):
        prefix = np.concatenate([ids, tok[:, :step].astype(np.float32)], axis=1)
        lg = eng.forward(prefix)
        for s in range(ids.shape[0]):
            t = int(tok[s, step])
            if t == int(lg[s].argmax()):
                continue
            top2 = np.sort(lg[s])[-2:]
            assert lg[s][t] >= top2[0] and top2[1] - top2[0] <= 2 * (ATOL + RTOL * abs(top2[1])), f"seq {s} step {step}"


def test_lm_rejects_bad_shapes(cuda):
    from technograd_b200 import _lib
    bad = dict(MICRO, head_dim=64)
    w = lm.random_weights(dict(bad, layers=1), seed=1)
    m = lm.Model(dict(bad, layers=1), 8, {k: v for k, v in w.items() if not lm.is_linear(k)}, {})
    with pytest.raises(Exception):
        lm.Engine(m, 2, 8)
    h = C.c_void_p()
    assert _lib.lib().tg_cuda_lm_load(None, 1, 1, C.byref(h)) == _lib.EINVAL
