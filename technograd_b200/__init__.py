"""technograd_b200: a B200 (sm_100a) batch backend for Technograd.

The product is libtgcuda.so (technograd_b200/csrc, C ABI in include/tg_cuda.h).
This package is its Python host mirror: a TGIR reader (tgir), the
`tgc batch --device cuda` equivalent (batch) and the decoder-LM driver (lm).
"""
from . import _lib  # noqa: F401
