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
import re
import sys
import time

import numpy as np

from . import _lib, cnum, tgir


def is_binary(path: str) -> bool:
    """src/io.c:17-21: the extension after the last dot is .bin or .f32."""
    dot = path.rfind(".")
    return dot >= 0 and path[dot:] in (".bin", ".f32")


# One field as strtof reads it: its own leading white space, then a number in the C library's
# grammar; the match ends where strtof stops.
_NUMBER = re.compile(r"[ \t\n\v\f\r]*(?P<num>" + cnum.PATTERN + ")", re.X)
_SEPARATORS = " \t,\r\n"


def parse_row(line: str) -> tuple[list, list] | int:
    """io_parse_row (src/io.c:25-41): the numbers of one line up to its end or a '#', as
    (doubles, tokens); or the offset of the first bad number. A number must end at a
    separator (space, tab, comma, CR, LF), a '#' or the end of the line."""
    vals, toks, i, n = [], [], 0, len(line)
    while True:
        while i < n and line[i] in _SEPARATORS:
            i += 1
        if i >= n or line[i] == "#":
            return vals, toks
        m = _NUMBER.match(line, i)
        if m is None or (m.end() < n and line[m.end()] not in _SEPARATORS + "#"):
            return i
        tok = m.group("num")
        vals.append(cnum.strtod(tok))
        toks.append(tok)
        i = m.end()


def _narrow(vals: list, toks: list) -> np.ndarray:
    """Doubles of correctly rounded tokens -> the f32 values strtof gives. Rounding the double
    to f32 gives strtof's result unless the double sits exactly on a midpoint between two f32
    values (the decimal may lie on either side of it), overflowed, or is a NaN (whose sign and
    payload strtof sets); those few tokens are read by strtof itself."""
    d = np.array(vals, np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        f = d.astype(np.float32)
        other = np.nextafter(f, np.where(f.astype(np.float64) > d, np.float32(-np.inf), np.float32(np.inf)))
        mid = (f.astype(np.float64) + other.astype(np.float64)) / 2
    redo = np.isnan(d) | (np.isinf(f) & ~np.isinf(d)) | ((f.astype(np.float64) != d) & (mid == d))
    for i in np.flatnonzero(redo):
        f[i] = cnum.strtof(toks[i])
    return f


def load_samples(path: str, per: int, model: str = "model") -> np.ndarray:
    """src/main.c:175-214 load_samples: raw little-endian f32 streams, or text rows of exactly
    `per` numbers (blank and comment-only lines skipped). Everything is validated before
    anything is returned; errors carry the reference's wording."""
    if path == "-":  # src/util.c:100-103: "-" is standard input
        raw = sys.stdin.buffer.read()
    else:
        try:
            with open(path, "rb") as fh:
                raw = fh.read()
        except OSError as e:
            raise ValueError(f"cannot open '{path}'") from e
    if is_binary(path):
        if len(raw) % 4:  # src/io.c:49
            raise ValueError(f"'{path}': {len(raw)} bytes is not a whole number of f32 values")
        v = np.frombuffer(raw, dtype="<f4")
        if v.size % per:
            raise ValueError(f"'{path}': {v.size} values is not a multiple of the {per} per sample")
        return v.astype(np.float32).reshape(-1, per)
    text = raw.split(b"\0", 1)[0].decode("latin-1")  # the C loop stops at a NUL byte
    vals, toks = [], []
    for lineno, line in enumerate(text.split("\n"), 1):
        r = parse_row(line)
        if isinstance(r, int):
            raise ValueError(f"{path}:{lineno}: bad number near '{line[r:r + 20]}'")
        if r[0] and len(r[0]) != per:
            raise ValueError(f"{path}:{lineno}: row has {len(r[0])} values, model {model} needs {per} per sample")
        vals += r[0]
        toks += r[1]
    return _narrow(vals, toks).reshape(-1, per)


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


def _g9(v) -> str:
    """printf("%.9g", (double)v) as glibc writes it: NaN with its sign ("-nan")."""
    v = float(v)
    if v != v:
        return "-nan" if np.signbit(v) else "nan"
    return f"{v:.9g}"


def _text_rows(out: np.ndarray, steps: np.ndarray) -> str:
    lines = []
    for r in range(out.shape[0]):
        vals = ",".join(_g9(v) for v in out[r])
        extra = "".join(f",{int(s)}" for s in steps[r])
        lines.append(vals + extra)
    return "\n".join(lines) + ("\n" if lines else "")


def write_rows(path: str | None, out: np.ndarray, steps: np.ndarray) -> None:
    if path and is_binary(path):
        out.astype("<f4").tofile(path)
        return
    text = _text_rows(out, steps)
    if path:
        with open(path, "w", encoding="utf-8") as f:
            f.write(text)
    else:
        sys.stdout.write(text)


def _open_out(path: str):
    """src/main.c:64-68 open_out: the output file, created (or truncated) once the samples
    have validated and before any compute (src/main.c:414-419); 'cannot write' otherwise."""
    try:
        return open(path, "wb") if is_binary(path) else open(path, "w", encoding="utf-8")
    except OSError as e:
        raise ValueError(f"cannot write '{path}'") from e


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="tgc batch --device cuda")
    ap.add_argument("model")
    ap.add_argument("data")
    ap.add_argument("-o", dest="out")
    ap.add_argument("--gpus", type=int, default=0)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args(argv)
    t0 = time.perf_counter()
    try:
        m = tgir.load(a.model)
    except OSError as e:
        raise ValueError(f"cannot open '{a.model}'") from e
    rows = load_samples(a.data, m.per, m.name)  # everything validated before compute or output
    f = _open_out(a.out) if a.out else None
    try:
        b = Batch(m, a.gpus)
        out, steps = b.run(rows)
        try:
            if f is None:
                sys.stdout.write(_text_rows(out, steps))
            else:
                f.write(out.astype("<f4").tobytes() if is_binary(a.out) else _text_rows(out, steps))
                f.close()  # src/main.c:71-74 close_out: an error here is 'write failed'
        except OSError as e:
            raise ValueError(f"write failed '{a.out}'") from e
    finally:
        if f is not None and not f.closed:
            f.close()
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
