"""Numbers as the reference reads them: glibc's strtod / strtof in the C locale.

The reference's TGIR reader turns an atom into a number when strtod consumes all of it
and it starts with a digit, or with a sign or '.' and is longer than one character
(src/sexp.c:112-121); its row reader calls strtof on each field (src/io.c:25-41). Both
accept what the C library accepts -- hex floats, inf/infinity, nan and nan(chars), in any
case -- and nothing else (no digit separators, no partial numbers). Values are correctly
rounded, as Python's float() and float.fromhex() are, so those give the value wherever
they apply; the C function itself reads the few forms Python does not (nan(chars), hex
floats past the double range).
"""
from __future__ import annotations

import ctypes as C
import re

import numpy as np

# one number in the C library's grammar, from its first character to where strtod stops
PATTERN = r"""[+-]?(?:
      0[xX](?:[0-9a-fA-F]+(?:\.[0-9a-fA-F]*)?|\.[0-9a-fA-F]+)(?:[pP][+-]?[0-9]+)?
    | (?:[0-9]+(?:\.[0-9]*)?|\.[0-9]+)(?:[eE][+-]?[0-9]+)?
    | [iI][nN][fF](?:[iI][nN][iI][tT][yY])?
    | [nN][aA][nN](?:\([0-9A-Za-z_]*\))?)"""
_FULL = re.compile(PATTERN, re.X)
_libc = {}


def _c(name: str, restype):
    f = _libc.get(name)
    if f is None:
        f = getattr(C.CDLL(None), name)
        f.restype, f.argtypes = restype, [C.c_char_p, C.c_void_p]
        _libc[name] = f
    return f


def strtod(tok: str) -> float:
    """The double strtod gives for a token that matches PATTERN in full."""
    t = tok.lower()
    if "nan" in t:
        return _c("strtod", C.c_double)(tok.encode("ascii"), None)  # sign and payload as glibc sets them
    if "x" in t:
        try:
            return float.fromhex(tok)
        except OverflowError:
            return _c("strtod", C.c_double)(tok.encode("ascii"), None)
    return float(tok)


def strtof(tok: str) -> np.float32:
    """The float strtof gives for a token that matches PATTERN in full."""
    return np.float32(_c("strtof", C.c_float)(tok.encode("ascii"), None))


def atom_number(tok: str) -> float | None:
    """src/sexp.c:112-121: the token's value when the reference's reader makes it a number,
    else None (the reader makes it a symbol)."""
    if not (tok[0].isdigit() or (tok[0] in "+-." and len(tok) > 1)):
        return None
    if _FULL.fullmatch(tok) is None:
        return None
    return strtod(tok)
