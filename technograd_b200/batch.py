"""`tgc batch MODEL DATA [-o OUT] --device cuda`: the batch branch of the
reference driver (src/main.c:400-444) over libtgcuda.

Same contract as the reference: the whole input is read and validated before
any compute and before the output file is created (src/main.c:414-419), rows
keep input order, text output is `%.9g` values joined by commas followed by
`,steps` per think loop (src/io.c:79-92), binary output (.bin/.f32) is raw
little-endian f32 without steps. A failure of the device path is an error:
there is no CPU fallback.

    python -m technograd_b200.batch MODEL.tgir DATA [-o OUT] [--gpus N]
"""
from __future__ import annotations

import argparse
import ctypes as C
import sys
import time

import numpy as np

from . import _lib, tgir


def is_binary(path: str) -> bool:
    return path.endswith(".bin") or path.endswith(".f32")


def load_samples(path: str, per: int) -> np.ndarray:
    """src/main.c:175-214 load_samples: raw f32 streams or text rows of exactly `per` numbers."""
    if is_binary(path):
        raw = np.fromfile(path, dtype="<f4")
        if raw.size % per:
            raise ValueError(f"'{path}': {raw.size} values is not a multiple of the {per} per sample")
        return raw.reshape(-1, per).astype(np.float32)
    rows = []
    with open(path, encoding="utf-8") as f:
        for lineno, line in enumerate(f, 1):
            line = line.split("#", 1)[0]
            toks = [t for t in line.replace(",", " ").split()]
            if not toks:
                continue
            try:
                vals = [float(t) for t in toks]
            except ValueError as e:
                raise ValueError(f"{path}:{lineno}: bad number") from e
            if len(vals) != per:
                raise ValueError(f"{path}:{lineno}: row has {len(vals)} values, the model needs {per} per sample")
            rows.append(vals)
    return np.array(rows, dtype=np.float64).astype(np.float32).reshape(-1, per)


class Batch:
    """A loaded model on the selected GPUs."""

    def __init__(self, module: tgir.Module, gpus: int = 0):
        self.module = module
        self.prog = tgir.CProgram(module)
        _lib.init(gpus)
        h = C.c_void_p()
        _lib.check(_lib.lib().tg_cuda_load(self.prog.ptr(), C.byref(h)))
        self.handle = h

    @property
    def specialized(self) -> tuple[bool, str]:
        """(True, "") when rows run on the kernel generated for this program, else
        (False, reason): they run on the tape interpreter kernel."""
        why = C.create_string_buffer(512)
        r = _lib.lib().tg_cuda_model_jit(self.handle, why, 512)
        if r < 0:
            _lib.check(r)
        return r == 1, why.value.decode()

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            _lib.lib().tg_cuda_free(h)
            self.handle = None

    def run(self, rows: np.ndarray):
        m = self.module
        rows = np.ascontiguousarray(rows, np.float32).reshape(-1, m.per)
        n, nt = m.nout, max(m.nthink, 1)
        out = np.empty((rows.shape[0], n), np.float32)
        steps = np.zeros((rows.shape[0], nt), np.int32)
        _lib.check(_lib.lib().tg_cuda_batch(self.handle, rows.ctypes.data, rows.shape[0], m.per, out.ctypes.data, n,
                                            steps.ctypes.data, nt))
        return out, steps[:, :m.nthink]


class Batcher:
    """Micro-batching of single-row requests from many threads (tg_cuda_batcher_*), the
    device side of `tgc serve`: each run() blocks until its row has gone through the GPU
    in a batch with whatever other rows were waiting."""

    def __init__(self, batch: Batch, max_rows: int = 8192, max_wait_us: int = 1000):
        self.batch = batch  # keeps the model alive as long as the batcher
        h = C.c_void_p()
        _lib.check(_lib.lib().tg_cuda_batcher_new(batch.handle, max_rows, max_wait_us, C.byref(h)))
        self.handle = h

    def run(self, row) -> tuple[np.ndarray, np.ndarray]:
        m = self.batch.module
        row = np.ascontiguousarray(row, np.float32).reshape(m.per)
        out = np.empty(m.nout, np.float32)
        steps = np.zeros(max(m.nthink, 1), np.int32)
        _lib.check(_lib.lib().tg_cuda_batcher_run(self.handle, row.ctypes.data, out.ctypes.data, steps.ctypes.data))
        return out, steps[:m.nthink]

    def stats(self) -> tuple[int, int]:
        rows, batches = C.c_long(), C.c_long()
        _lib.check(_lib.lib().tg_cuda_batcher_stats(self.handle, C.byref(rows), C.byref(batches)))
        return rows.value, batches.value

    def close(self):
        if getattr(self, "handle", None):
            _lib.lib().tg_cuda_batcher_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


def write_rows(path: str | None, out: np.ndarray, steps: np.ndarray) -> None:
    if path and is_binary(path):
        out.astype("<f4").tofile(path)
        return
    lines = []
    for r in range(out.shape[0]):
        vals = ",".join(f"{float(v):.9g}" for v in out[r])
        extra = "".join(f",{int(s)}" for s in steps[r])
        lines.append(vals + extra)
    text = "\n".join(lines) + ("\n" if lines else "")
    if path:
        with open(path, "w", encoding="utf-8") as f:
            f.write(text)
    else:
        sys.stdout.write(text)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="tgc batch --device cuda")
    ap.add_argument("model")
    ap.add_argument("data")
    ap.add_argument("-o", dest="out")
    ap.add_argument("--gpus", type=int, default=0)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args(argv)
    t0 = time.perf_counter()
    m = tgir.load(a.model)
    rows = load_samples(a.data, m.per)  # everything validated before compute or output
    b = Batch(m, a.gpus)
    out, steps = b.run(rows)
    write_rows(a.out, out, steps)
    if a.v:
        ms = (time.perf_counter() - t0) * 1e3
        sys.stderr.write(f"[batch] {rows.shape[0]} row(s) in {ms:.2f} ms on {_lib.lib().tg_cuda_ngpus()} GPU(s)\n")
    return 0


if __name__ == "__main__":
    try:
        sys.exit(main())
    except (ValueError, _lib.TgCudaError, tgir.TgirError) as e:
        sys.stderr.write(f"error: {e}\n")
        sys.exit(1)
