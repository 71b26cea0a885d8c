"""TGIR reader and the flattening of a module into the C ABI's tg_cuda_program.

Reads the canonical S-expression form written by `tgc ir` / `tgc quantize`
(the grammar of IlumCI/Technograd src/ir.c:1-22, reader src/ir.c:458-554,
tokens src/sexp.c:70-126): params with `(data ...)` or `(quant BITS AXIS
(scale ...) (codes ...))`, inputs, the SSA block with think and scan forms,
the output and any updates. Codes are stored in the reference packing (int8
one per byte; int4 two per byte, low nibble first) and every quantized param
keeps `data = code * scale`, as src/ir.c:495-507 does.
"""
from __future__ import annotations

import ctypes as C
import mmap
import re
import warnings
from dataclasses import dataclass, field

import numpy as np

from . import _lib, cnum

_TOKEN = re.compile(rb'\s+|;[^\n]*|(\()|(\))|"([^"\n]*)"|([^\s();"]+)')
# the number lists of params: read straight into arrays (no object per number)
_PAYLOAD = re.compile(rb'\(\s*(data|codes|scale)(?=[\s)])')


class TgirError(ValueError):
    pass


def _atom(tok: str):
    # src/sexp.c:112-121: a number when strtod consumes it all and it starts like one
    v = cnum.atom_number(tok)
    return Sym(tok) if v is None else v


class Sym(str):
    pass


_DECIMAL_BYTES = b"0123456789eE+-. \t\n\r\v\f"
_SPACE = re.compile(rb"\s")
_CHUNK = 1 << 25  # bytes of text parsed at a time


def _plain_decimals(span) -> bool:
    """Whether a number list holds only decimal forms numpy parses as strtod does. Lists with
    anything else (hex floats, inf/nan, symbols, a nested list or comment) or a bare sign go
    atom by atom."""
    if span.translate(None, _DECIMAL_BYTES):
        return False
    b = np.frombuffer(span, np.uint8)
    sign = (b == 43) | (b == 45)  # '+' or '-'
    if not sign.any():
        return True
    if sign[-1]:
        return False
    nx = b[1:]
    number = (nx - np.uint8(48) <= 9) | (nx == 46)  # a digit (uint8 wrap) or '.' follows
    return not (sign[:-1] & ~number).any()


def _parse_chunk(span: bytes, head: str) -> np.ndarray:
    with warnings.catch_warnings():
        warnings.simplefilter("error", DeprecationWarning)  # a partial parse is an error
        try:
            if head == "codes":
                try:
                    c = np.fromstring(span, dtype=np.int32, sep=" ")
                    return c.astype(np.int8) if c.size and -128 <= c.min() and c.max() <= 127 else c
                except (ValueError, DeprecationWarning):
                    pass  # not plain integers: let the generic check below decide
            return np.fromstring(span, dtype=np.float64, sep=" ")
        except (ValueError, DeprecationWarning) as e:
            raise TgirError(f"bad number in ({head} ...)") from e


def _payload(buf, start: int, end: int, head: str) -> np.ndarray | None:
    """The numbers of the (data ...), (codes ...) or (scale ...) list whose text is
    buf[start:end], parsed in C a few tens of MB at a time (split at whitespace), or None
    when the list holds anything but plain decimals. Codes are integers (src/ir.c:478-509;
    int8 when they fit); data and scales are read as doubles, as the reference's strtod
    does (src/sexp.c:112-121), and rounded to f32 chunk by chunk as its (float) does, so a
    list of hundreds of millions of numbers never exists as doubles or as one string."""
    parts = []
    s = start
    while s < end:
        e = min(end, s + _CHUNK)
        if e < end:  # end the chunk at whitespace so that no number is split
            m = _SPACE.search(buf, e, end)
            e = m.start() if m else end
        span = buf[s:e]
        if not _plain_decimals(span):
            return None
        if span and not span.isspace():
            x = _parse_chunk(span, head)
            if x.dtype == np.float64 and head != "codes":
                with np.errstate(over="ignore"):  # (float) of a double past the f32 range is inf, as in C
                    x = x.astype(np.float32)
            parts.append(x)
        s = e
    if not parts:
        return np.zeros(0, np.int32 if head == "codes" else np.float32)
    return parts[0] if len(parts) == 1 else np.concatenate(parts)


def read_sexp(src, fast: bool = True) -> list:
    """S-expressions of `src` (str, bytes or a read-only mmap). With `fast`, the number
    lists of params become [Sym(head), ndarray] without a Python object per number, so a
    quantized model of hundreds of millions of codes reads in bounded memory; without it,
    every number is an atom, as the reference's reader builds its Sx nodes."""
    buf = src.encode("utf-8") if isinstance(src, str) else src
    stack: list[list] = [[]]
    pos = 0
    n = len(buf)
    while pos < n:
        m = _TOKEN.match(buf, pos)
        if not m:
            raise TgirError(f"bad character at offset {pos}")
        if m.group(1) and fast:
            pm = _PAYLOAD.match(buf, pos)
            if pm:
                end = buf.find(b")", pm.end())
                if end < 0:
                    raise TgirError("unterminated list")
                head = pm.group(1).decode()
                arr = _payload(buf, pm.end(), end, head)
                if arr is not None:
                    stack[-1].append([Sym(head), arr])
                    pos = end + 1
                    continue
        pos = m.end()
        if m.group(1):
            stack.append([])
        elif m.group(2):
            if len(stack) == 1:
                raise TgirError("unexpected ')'")
            done = stack.pop()
            stack[-1].append(done)
        elif m.group(3) is not None:
            stack[-1].append(m.group(3).decode("utf-8"))
        elif m.group(4):
            stack[-1].append(_atom(m.group(4).decode("utf-8")))
    if len(stack) != 1:
        raise TgirError("unterminated list")
    return stack[0]


def _numbers(node) -> np.ndarray:
    """The values of a number list, parsed fast (an array) or as atoms."""
    if len(node) == 2 and isinstance(node[1], np.ndarray):
        return node[1]
    if any(isinstance(x, (str, list)) for x in node[1:]):  # a symbol, string or list among the numbers
        raise TgirError(f"bad number in ({node[0]} ...)")
    return np.array(node[1:], dtype=np.float64)


@dataclass
class PValue:
    kind: int
    shape: tuple
    name: str | None = None
    data: np.ndarray | None = None
    qbits: int = 0
    qaxis: int = 0
    q: np.ndarray | None = None
    qs: np.ndarray | None = None
    index: int = 0

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def dense(self) -> np.ndarray | None:
        """The param's f32 values: its data, or for a quantized param code * scale of the
        element's channel (src/ir.c:495-507, one f32 rounding), made on demand so that a
        large quantized model is held as its codes only."""
        if self.data is not None or not self.qbits:
            return self.data
        c2 = unpack_codes(self.q, self.qbits, self.numel).reshape(self.shape[0], -1).astype(np.float32)
        return (c2 * (self.qs[:, None] if self.qaxis == 0 else self.qs[None, :])).astype(np.float32).ravel()


@dataclass
class PScan:
    T: int
    reverse: int
    tid: int
    c: list = field(default_factory=list)
    init: list = field(default_factory=list)
    next: list = field(default_factory=list)
    x: list = field(default_factory=list)
    xt: list = field(default_factory=list)
    y: list = field(default_factory=list)
    ys: list = field(default_factory=list)


@dataclass
class PIns:
    op: int
    out: int
    a: list = field(default_factory=list)
    k: float = 0.0
    init: int = -1
    maxit: int = 0
    eps: float = -1.0
    yield_: int = -1
    tid: int = -1
    halt: int = -1
    hthr: float = 0.0
    body: list = field(default_factory=list)
    scan: PScan | None = None


@dataclass
class Module:
    name: str
    vals: list = field(default_factory=list)
    top: list = field(default_factory=list)
    inputs: list = field(default_factory=list)
    output: int = -1
    nthink: int = 0
    nupd: int = 0

    def value(self, kind, shape, name=None) -> int:
        self.vals.append(PValue(kind, tuple(int(d) for d in shape), name))
        return len(self.vals) - 1

    @property
    def per(self) -> int:
        return sum(self.vals[v].numel for v in self.inputs)

    @property
    def nout(self) -> int:
        return self.vals[self.output].numel


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Reference packing (runtime/tg_rt.h:124-129): int8 as is; int4 element i in
    byte i/2, low nibble first."""
    codes = np.asarray(codes).ravel()
    if codes.dtype.kind not in "iu":
        codes = codes.astype(np.int64)
    if bits == 8:
        return codes.astype(np.int8)
    u = codes.astype(np.uint8)  # the low nibble survives the wrap
    if u.size % 2:
        u = np.concatenate([u, np.zeros(1, np.uint8)])
    pair = u.reshape(-1, 2)
    return ((pair[:, 0] & 0x0F) | (pair[:, 1] << 4)).view(np.int8)


def unpack_codes(q: np.ndarray, bits: int, n: int) -> np.ndarray:
    q = np.asarray(q).view(np.int8).ravel()
    if bits == 8:
        return q[:n].astype(np.int32)
    b = q.astype(np.int32)
    lo = ((b & 0x0F) ^ 0x08) - 0x08  # low nibble, sign-extended
    hi = b >> 4                      # arithmetic shift of the signed byte
    out = np.empty(2 * b.size, dtype=np.int32)
    out[0::2] = lo
    out[1::2] = hi
    return out[:n]


def _shape(x) -> tuple:
    if not isinstance(x, list) or not x or x[0] != "f32" or len(x) - 1 > 4:
        raise TgirError("expected type (f32 d...)")
    dims = []
    for d in x[1:]:
        if not isinstance(d, float) or d < 1 or d != int(d):
            raise TgirError("bad dimension")
        dims.append(int(d))
    return tuple(dims)


class _Reader:
    def __init__(self, m: Module):
        self.m = m
        self.scope: list[tuple[str, int]] = []

    def get(self, name) -> int:
        if not isinstance(name, Sym):
            raise TgirError("expected value name")
        for n, v in reversed(self.scope):
            if n == name:
                return v
        raise TgirError(f"undefined value '{name}'")

    def define(self, name, v: int) -> None:
        # src/ir.c:223-227: a name, defined once in the scope
        if not isinstance(name, Sym):
            raise TgirError("expected value name")
        if any(n == name for n, _ in self.scope):
            raise TgirError(f"redefinition of '{name}'")
        self.scope.append((str(name), v))

    def block(self, forms) -> list:
        out = []
        for x in forms:
            if isinstance(x, list) and x and x[0] == "scan":
                out.append(self.scan(x))
                continue
            if not (isinstance(x, list) and len(x) == 3 and isinstance(x[2], list) and x[2]):
                raise TgirError("malformed instruction")
            shape = _shape(x[1])
            e = x[2]
            head = e[0]
            m = self.m
            if head == "const":
                v = m.value(_lib.TMP, shape)
                ins = PIns(_lib.OP["const"], v, k=float(np.float32(e[1])))
                self.define(x[0], v)
            elif head == "think":
                init = self.get(e[1])
                maxit = int(e[2])
                eps = -1.0 if e[3] == "none" else float(np.float32(e[3]))
                v = m.value(_lib.TMP, shape)
                has_halt = isinstance(e[-1], list) and e[-1] and e[-1][0] == "halt"
                y = e[-1 - has_halt]
                if not (isinstance(y, list) and len(y) == 2 and y[0] == "yield"):
                    raise TgirError("think (missing yield)")
                tid = m.nthink
                m.nthink += 1
                mark = len(self.scope)
                self.define(x[0], v)
                body = self.block(e[4:len(e) - 1 - has_halt])
                ins = PIns(_lib.OP["think"], v, init=init, maxit=maxit, eps=eps, tid=tid, body=body)
                ins.yield_ = self.get(y[1])
                if has_halt:
                    ins.halt = self.get(e[-1][1])
                    ins.hthr = float(np.float32(e[-1][2]))
                del self.scope[mark:]
                self.define(x[0], v)
            else:
                if head not in _lib.OP:
                    raise TgirError(f"unknown op '{head}'")
                args = [self.get(a) for a in e[1:]]
                v = m.value(_lib.TMP, shape)
                ins = PIns(_lib.OP[head], v, a=args)
                self.define(x[0], v)
            out.append(ins)
        return out

    def scan(self, x) -> PIns:
        m = self.m
        T = int(x[1])
        rev = 1 if x[2] == "reverse" else 0
        i = 3
        tid = -1
        if i < len(x) and x[i] == "steps":
            tid = m.nthink
            m.nthink += 1
            i += 1
        s = PScan(T, rev, tid)
        cnames, xnames = [], []
        while i < len(x) and isinstance(x[i], list) and len(x[i]) == 4 and x[i][0] == "carry":
            c = x[i]
            s.init.append(self.get(c[3]))
            s.c.append(m.value(_lib.TMP, _shape(c[2])))
            cnames.append(c[1])
            i += 1
        while i < len(x) and isinstance(x[i], list) and len(x[i]) == 4 and x[i][0] == "in":
            c = x[i]
            s.x.append(self.get(c[3]))
            s.xt.append(m.value(_lib.TMP, _shape(c[2])))
            xnames.append(c[1])
            i += 1
        mark = len(self.scope)
        for n, v in zip(cnames, s.c):
            self.define(n, v)
        for n, v in zip(xnames, s.xt):
            self.define(n, v)
        if not (isinstance(x[i], list) and x[i] and x[i][0] == "body"):
            raise TgirError("scan (body)")
        body = self.block(x[i][1:])
        i += 1
        for _ in s.c:
            s.next.append(self.get(x[i][2]))
            i += 1
        ynames = []
        while i < len(x):
            c = x[i]
            s.y.append(self.get(c[3]))
            ynames.append((c[1], _shape(c[2])))
            i += 1
        del self.scope[mark:]
        for n, v in zip(cnames, s.c):
            self.define(n, v)
        for n, sh in ynames:
            ys = m.value(_lib.TMP, sh)
            s.ys.append(ys)
            self.define(n, ys)
        return PIns(_lib.OP["scan"], s.c[0], body=body, scan=s, tid=tid)


def read(src, fast: bool = True) -> Module:
    forms = read_sexp(src, fast)
    if len(forms) != 1 or not isinstance(forms[0], list) or forms[0][:2] != ["tgir", 1.0]:
        raise TgirError("expected (tgir 1 ...)")
    m = None
    rd = None
    seen_block = seen_out = False  # the order of src/ir.c:462-548
    for f in forms[0][2:]:
        if not (isinstance(f, list) and f and isinstance(f[0], Sym)):
            raise TgirError("malformed top-level form")
        h = f[0]
        if h == "model":
            if m is not None or len(f) != 2 or not isinstance(f[1], Sym):
                raise TgirError("malformed model")
            m = Module(str(f[1]))
            rd = _Reader(m)
            continue
        if m is None:
            raise TgirError("(model ...) must come first")
        if h in ("param", "state", "input") and seen_block:
            raise TgirError(f"malformed {h} (after the block)")
        if h in ("param", "state") and len(f) == 4 and isinstance(f[3], list) and f[3] and f[3][0] == "quant":
            shape = _shape(f[2])
            if len(f[3]) != 5 or f[3][1] not in (8.0, 4.0):
                raise TgirError("malformed quant bits (8 or 4)")
            if len(shape) != 2 or f[3][2] not in (0.0, 1.0):
                raise TgirError("malformed quant axis (0 or 1, rank-2 param)")
            bits, axis = int(f[3][1]), int(f[3][2])
            with np.errstate(over="ignore"):  # (float) of a double past the f32 range is inf, as in C
                sc = _numbers(f[3][3]).astype(np.float32, copy=False)
            codes = _numbers(f[3][4])
            if codes.dtype.kind == "f":
                if not np.array_equal(codes, np.round(codes)):
                    raise TgirError(f"param '{f[1]}': codes must be integers")
                codes = codes.astype(np.int32)
            n = int(np.prod(shape))
            if codes.size != n or sc.size != shape[axis]:
                raise TgirError(f"param '{f[1]}': quant sizes")
            lim = 127 if bits == 8 else 7
            if codes.size and (codes.min() < -lim or codes.max() > lim):
                raise TgirError(f"param '{f[1]}': code out of range")
            v = m.value(_lib.PARAM, shape, str(f[1]))
            pv = m.vals[v]
            pv.qbits, pv.qaxis = bits, axis
            pv.q = pack_codes(codes, bits)
            pv.qs = sc  # data (code * scale, src/ir.c:495-507) is made on demand: PValue.dense()
            del codes
            rd.define(f[1], v)
        elif h in ("param", "state"):
            shape = _shape(f[2])
            with np.errstate(over="ignore"):
                data = _numbers(f[3]).astype(np.float32, copy=False)
            if data.size != int(np.prod(shape)):
                raise TgirError(f"param '{f[1]}' needs {int(np.prod(shape))} values, has {data.size}")
            v = m.value(_lib.PARAM if h == "param" else _lib.STATE, shape, str(f[1]))
            m.vals[v].data = data
            rd.define(f[1], v)
        elif h == "input":
            v = m.value(_lib.INPUT, _shape(f[2]), str(f[1]))
            m.vals[v].index = len(m.inputs)
            m.inputs.append(v)
            rd.define(f[1], v)
        elif h == "block":
            if seen_block:
                raise TgirError("malformed block (duplicate)")
            seen_block = True
            m.top = rd.block(f[1:])
        elif h == "output":
            if not seen_block or seen_out or len(f) != 2:
                raise TgirError("malformed output")
            seen_out = True
            m.output = rd.get(f[1])
        elif h == "update":
            if not seen_block:
                raise TgirError("malformed update (before the block)")
            m.nupd += 1
        else:
            raise TgirError(f"unknown top-level form '{h}'")
    if m is None or not m.inputs or m.output < 0:
        raise TgirError("incomplete module")
    return m


def load(path: str, fast: bool = True) -> Module:
    """Reads a TGIR file through a read-only memory map: the text is never held as a
    Python string, and the params' number lists are parsed straight into arrays."""
    with open(path, "rb") as f:
        try:
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError:  # an empty file cannot be mapped
            return read(b"", fast)
        with mm:
            return read(mm, fast)


class CProgram:
    """A Module flattened into tg_cuda_program, owning every buffer it points to."""

    def __init__(self, m: Module):
        self.module = m
        self._keep: list = []
        vals = (_lib.Value * len(m.vals))()
        for i, pv in enumerate(m.vals):
            cv = vals[i]
            cv.kind = pv.kind
            cv.rank = len(pv.shape)
            for d, n in enumerate(pv.shape):
                cv.dim[d] = n
            cv.index = pv.index
            dense = pv.dense()
            if dense is not None:
                arr = np.ascontiguousarray(dense, dtype=np.float32)
                self._keep.append(arr)
                cv.data = arr.ctypes.data_as(_lib.FP)
            if pv.qbits:
                q = np.ascontiguousarray(pv.q, dtype=np.int8)
                qs = np.ascontiguousarray(pv.qs, dtype=np.float32)
                self._keep += [q, qs]
                cv.qbits, cv.qaxis = pv.qbits, pv.qaxis
                cv.q = q.ctypes.data_as(C.POINTER(C.c_byte))
                cv.qs = qs.ctypes.data_as(_lib.FP)
        flat: list[PIns] = []
        scans: list[PScan] = []
        ranges: dict[int, tuple[int, int]] = {}

        def lay(block: list) -> tuple[int, int]:
            start = len(flat)
            flat.extend(block)
            for ins in block:
                if ins.op in (_lib.OP["think"], _lib.OP["scan"]):
                    ranges[id(ins)] = lay(ins.body)
            return start, len(block)

        _, ntop = lay(m.top)
        ins_arr = (_lib.Ins * max(len(flat), 1))()
        for i, pi in enumerate(flat):
            ci = ins_arr[i]
            ci.op, ci.out, ci.na, ci.k = pi.op, pi.out, len(pi.a), pi.k
            for j, a in enumerate(pi.a):
                ci.a[j] = a
            for j in range(len(pi.a), 3):
                ci.a[j] = -1
            ci.init, ci.maxit, ci.eps, ci.yield_ = pi.init, pi.maxit, pi.eps, pi.yield_
            ci.tid, ci.halt, ci.hthr, ci.scan = pi.tid, pi.halt, pi.hthr, -1
            if id(pi) in ranges:
                ci.body, ci.nbody = ranges[id(pi)]
            if pi.scan is not None:
                ci.scan = len(scans)
                scans.append(pi.scan)
        scan_arr = (_lib.Scan * max(len(scans), 1))()
        for i, s in enumerate(scans):
            cs = scan_arr[i]
            cs.T, cs.reverse, cs.tid = s.T, s.reverse, s.tid

            def ia(lst):
                a = (C.c_int * max(len(lst), 1))(*lst)
                self._keep.append(a)
                return a

            cs.nc, cs.c, cs.init, cs.next = len(s.c), ia(s.c), ia(s.init), ia(s.next)
            cs.nx, cs.x, cs.xt = len(s.x), ia(s.x), ia(s.xt)
            cs.ny, cs.y, cs.ys = len(s.y), ia(s.y), ia(s.ys)
        inputs = (C.c_int * len(m.inputs))(*m.inputs)
        self._keep += [vals, ins_arr, scan_arr, inputs]
        p = _lib.Program()
        p.nval, p.val = len(m.vals), vals
        p.nins, p.ins, p.ntop = len(flat), ins_arr, ntop
        p.nscan, p.scans = len(scans), scan_arr
        p.ninputs, p.inputs = len(m.inputs), inputs
        p.output, p.nthink, p.nupd = m.output, m.nthink, m.nupd
        self.c = p

    def ptr(self):
        return C.byref(self.c)
