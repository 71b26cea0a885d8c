"""The decode-step GEMM (gemm_sk: weights in the MMA's 128-row slot, K split over a cluster
and summed in rank order through distributed shared memory) against a float64 reference of
the same bf16 products, and against the tile kernel it replaces for small batches. GPU.

Shapes: the decoder's four per-layer products at waves of 1, 20, 256 and 512 sequences
(q/k/v: store with per-channel scales; o_proj: three hi/lo pairs added into the residual;
gate/up: SwiGLU with its bf16 hi/lo output; down: scaled and added), plus ragged ones (a
partial 256-row batch tile, a partial channel tile, a short K). bf16 x bf16 products are
exact in f32, so only the summation order differs from the reference: |err| <= 1e-5 of the
sum of |products| (plus the bf16 split of SwiGLU's output). Repeated calls are bit-identical."""
import ctypes as C

import pytest
import torch

from technograd_b200 import _lib

pytestmark = pytest.mark.gpu
STORE, ADD, SWIGLU = 0, 1, 2


def run(path, a, b, pairs, epi, scale=None, scale2=None, out=None, hi=None, lo=None):
    L = _lib.lib()
    M, K = a[0].shape
    N = b[0].shape[0]
    ap = (C.c_void_p * 2)(*[t.data_ptr() for t in a] + [0] * (2 - len(a)))
    bp = (C.c_void_p * 2)(*[t.data_ptr() for t in b] + [0] * (2 - len(b)))
    pa = (C.c_int * 4)(*[q[0] for q in pairs])
    pb = (C.c_int * 4)(*[q[1] for q in pairs])
    ldo = N // 2 if epi == SWIGLU else N
    _lib.check(L.tg_cuda_selftest_gemm(path, ap, len(a), bp, len(b), len(pairs), pa, pb, M, N, K, epi,
                                       scale.data_ptr() if scale is not None else None,
                                       scale2.data_ptr() if scale2 is not None else None,
                                       out.data_ptr() if out is not None else None, ldo,
                                       hi.data_ptr() if hi is not None else None, lo.data_ptr() if lo is not None else None,
                                       None))


def reference(a, b, pairs):
    """sum over pairs of a @ b^T in float64, and the sum of |products| for the error bound"""
    s = sum(a[i].double() @ b[j].double().T for i, j in pairs)
    mag = sum(a[i].double().abs() @ b[j].double().abs().T for i, j in pairs)
    return s, mag


def operands(M, N, K, nw, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g)
    xhi = x.bfloat16()
    xlo = (x - xhi.float()).bfloat16()
    w = torch.randint(-8, 8, (N, K), device="cuda", generator=g).float()
    if nw == 1:
        return [xhi, xlo], [w.bfloat16()]
    ws = w * torch.rand(N, 1, device="cuda", generator=g) * 0.01  # pre-scaled weights: hi/lo too
    whi = ws.bfloat16()
    return [xhi, xlo], [whi, (ws - whi.float()).bfloat16()]


X_W = [(0, 0), (1, 0)]
X_W2 = [(0, 0), (0, 1), (1, 0)]
SHAPES = [(M, N, K) for M in (1, 20, 256, 512) for (N, K) in ((4096, 1024), (1024, 2048), (1024, 3072))] + \
         [(300, 1000, 192), (129, 256, 64), (64, 128, 4096)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("epi", [STORE, ADD])
def test_store_and_add(cuda, M, N, K, epi):
    nw = 2 if (N, K) == (1024, 2048) else 1  # o_proj: pre-scaled hi/lo weights, three pairs
    a, b = operands(M, N, K, nw, seed=M * 7 + N + K)
    pairs = X_W2 if nw == 2 else X_W
    scale = None if nw == 2 else torch.rand(N, device="cuda") * 0.02
    want, mag = reference(a, b, pairs)
    if scale is not None:
        want, mag = want * scale.double(), mag * scale.double().abs()
    base = torch.randn(M, N, device="cuda") if epi == ADD else torch.zeros(M, N, device="cuda")
    if epi == ADD:
        want = want + base.double()
    outs = []
    for path in (1, 1, 0):
        out = base.clone()
        run(path, a, b, pairs, epi, scale=scale, out=out)
        outs.append(out)
    assert torch.equal(outs[0], outs[1]), "two calls of the cluster kernel differ"
    bound = 1e-5 * mag + (base.double().abs() * 2 ** -23 if epi == ADD else 0) + 1e-30
    for out, name in ((outs[0], "gemm_sk"), (outs[2], "tile kernel")):
        err = (out.double() - want).abs()
        assert (err <= bound).all(), f"{name}: max err {err.max().item():.3g}, bound {bound.min().item():.3g}"


@pytest.mark.parametrize("M", [1, 20, 256, 512, 300])
def test_swiglu(cuda, M):
    FF, K = 3072, 1024
    a, b = operands(M, 2 * FF, K, 1, seed=M)
    sg, su = torch.rand(FF, device="cuda") * 0.02, torch.rand(FF, device="cuda") * 0.02
    s, mag = reference(a, b, X_W)
    ch = torch.arange(FF, device="cuda")
    gr, ur = ch // 32 * 64 + ch % 32, ch // 32 * 64 + ch % 32 + 32  # channel c: rows (c/32)*64 + c%32 and +32
    g, u = s[:, gr] * sg.double(), s[:, ur] * su.double()
    silu = g / (1 + torch.exp(-g))
    want = silu * u
    res = []
    for path in (1, 1, 0):
        hi = torch.empty(M, FF, dtype=torch.bfloat16, device="cuda")
        lo = torch.empty_like(hi)
        run(path, a, b, X_W, SWIGLU, scale=sg, scale2=su, hi=hi, lo=lo)
        res.append(hi.double() + lo.double())
    assert torch.equal(res[0], res[1])
    # errors of g and u (summation order) through silu(g) * u, and the hi/lo split of the result
    dg, du = 1e-5 * mag[:, gr] * sg.double(), 1e-5 * mag[:, ur] * su.double()
    bound = 1.2 * u.abs() * dg + silu.abs() * du + dg * du + 2 ** -15 * want.abs() + 1e-12
    for y, name in ((res[0], "gemm_sk"), (res[2], "tile kernel")):
        err = (y - want).abs()
        assert (err <= bound).all(), f"{name}: max err {err.max().item():.3g}"
