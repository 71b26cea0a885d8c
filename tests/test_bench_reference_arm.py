"""`bench.py --impl reference` on the host cores (CPU only): the reference's own `tgc batch`
(built from its sources into oracle/_ref by the build step) times config 1 and prints one
JSON line carrying the keys the benchmark contract names for the reference arm."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "tgc")),
                    reason="oracle/_ref/tgc is built only where the reference sources are present")
def test_reference_arm_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "lr",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "latent_reasoner int8 batch rows/s (config 1)" and d["unit"] == "rows/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    base = d["cpu_baseline"]
    assert base["kind"] == "reference" and base["value"] == d["value"] and base["cores"] >= 1 and base["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("config1")


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libtgref.so")),
                    reason="oracle/_ref is built only where the reference sources are present")
def test_reference_arm_runs_the_reference_vm_without_the_product():
    """Config 3 through the reference's own VM (load_module, quantize_param, vm_run_into):
    the line is the reference's, and nothing of technograd_b200 was imported on the way."""
    code = ("import runpy, sys, json; sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'ssm', '--steps', '1',"
            " '--warmup', '3']; runpy.run_path('bench.py', run_name='__main__');"
            " bad = sorted(m for m in sys.modules if m.startswith('technograd_b200'));"
            " print('PRODUCT_MODULES', json.dumps(bad))")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "PRODUCT_MODULES []" in r.stdout
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][0])
    assert d["impl"] == "reference" and d["metric"] == "int8 stacked selective-SSM tokens/s (config 3)"
    assert d["cpu_baseline"]["kind"] == "reference" and d["value"] > 0
    assert d["config"]["workload"].startswith("config3")


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libtgref.so")),
                    reason="oracle/_ref is built only where the reference sources are present")
@pytest.mark.parametrize("piece", ["attn", "gate", "down", "head"])
def test_qwen3_pieces_run_on_the_reference_vm(tmp_path, piece):
    """Each piece of the Qwen3 forward the reference arm times parses, plans, quantizes (int4
    GPTQ, as config 5) and runs in the reference's VM; a small architecture keeps it quick."""
    import ctypes as C

    sys.path.insert(0, ROOT)
    from oracle import refvm
    small = dict(refvm.QWEN3, hidden=256, nq=4, nkv=2, ffn=512, vocab=3000)
    path = refvm.emit_piece(piece, 24, str(tmp_path), seed=1, cfg=small)
    R = refvm.lib()
    mod = R.ref_vm_load(path.encode(), 4, 1 if piece != "head" else 0, 128 * 128 + 1, 256)
    assert mod
    sec = (C.c_double * 2)()
    assert R.ref_vm_run(mod, 3, 2, sec) >= 1
    assert sec[0] > 0 and sec[1] > 0


def test_every_workload_has_a_metric_and_config():
    """Both arms name each workload's metric and config from the same static tables; reduced
    shapes (profiling overrides) say so in the config."""
    import argparse
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_static", os.path.join(ROOT, "bench.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    args = argparse.Namespace(seqs=0, prompt=0, new=0, layers=0, bits=4)
    for wl in ("decode", "decode_small", "prefill", "ssm", "lr"):
        metric, unit = b.METRICS[wl]
        assert metric and unit in ("tokens/s", "rows/s")
        cfg = b.workload_config(wl, args)
        assert cfg["workload"].startswith("config"), (wl, cfg)
    assert b.workload_config("decode_small", args)["seqs_per_gpu"] == b.SMALL_SEQS
    assert b.workload_config("gemm", args, 16)["M"] == 16
    small = argparse.Namespace(seqs=2, prompt=64, new=3, layers=2, bits=4)
    for wl in ("decode", "decode_small", "prefill", "ssm"):
        assert b.workload_config(wl, small)["workload"].startswith("REDUCED"), wl
