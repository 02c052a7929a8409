"""slogdet / det under prec="ieee" for float32, 8 <= n <= 256: the tensor-memory LU with IEEE
float32 FMA block updates (one matrix in 128 TMEM lanes up to n = 128, in the SM's whole tensor
memory above). Checked against numpy in float64 and the oracle, with singular members, the
primal-under-gradient identity and the gathered-rows entry, as the reference suite does for
its LU path (tests/test_fermix.py:148-156, :443-481)."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx
import oracle
from oracle.refs64 import log_tol, randn, ref64, relerr
from tests.helpers import cuda, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [8, 10, 16, 33, 64, 100, 128, 129, 200, 256])
def test_ieee_slogdet_fwd_and_grad(n):
    gen = np.random.default_rng(700 + n)
    A = randn((6, n, n), np.float32, gen)
    s, l = host(fx.slogdet(cuda(A), prec="ieee"))
    s64, l64 = np.linalg.slogdet(ref64(A))
    assert np.array_equal(s, s64.astype(np.float32))
    assert np.max(np.abs(l - l64)) < log_tol(np.float32, n)
    so, lo = oracle.slogdet(A)
    assert np.array_equal(s, so)
    assert np.max(np.abs(l - lo)) < log_tol(np.float32, n)
    # the gradient call's primal is the forward's, bit for bit
    s2, l2, g = host(fx.slogdet_parts(cuda(A), prec="ieee"))
    assert np.array_equal(s, s2) and np.array_equal(l, l2)
    # gradients: 1e-3 relative per matrix, or cond(A) * eps32 for the ill-conditioned ones
    g_ref = np.swapaxes(np.linalg.inv(ref64(A)), -1, -2)
    eps = np.finfo(np.float32).eps
    for i in range(len(A)):
        cond = np.linalg.cond(ref64(A[i]))
        assert relerr(g[i], g_ref[i]) <= max(1e-3, cond * eps), (i, relerr(g[i], g_ref[i]), cond)


@pytest.mark.parametrize("n", [128, 256])
def test_ieee_duplicate_rows_are_exactly_singular(n):
    gen = np.random.default_rng(750 + n)
    A = randn((5, n, n), np.float32, gen)
    A[1, 7] = A[1, 3]
    A[2, n - 1] = -A[2, 0]
    A[3] = 0.0
    x = cuda(A, requires_grad=True)
    s, l = fx.slogdet(x, prec="ieee")
    (g,) = torch.autograd.grad(l.sum(), x)
    s, l, g = host(s), host(l), host(g)
    for b in (1, 2, 3):
        assert s[b] == 0 and np.isneginf(l[b]) and np.all(g[b] == 0), b
    assert np.all(np.isfinite(g))
    s64, l64 = np.linalg.slogdet(ref64(A[[0, 4]]))
    assert np.array_equal(s[[0, 4]], s64.astype(np.float32))
    assert np.max(np.abs(l[[0, 4]] - l64)) < log_tol(np.float32, n)
    # det values under ieee (n = 16 keeps |det| within float32)
    T = randn((3, 16, 16), np.float32, gen)
    d = host(fx.det(cuda(T), prec="ieee"))
    assert np.allclose(d, np.linalg.det(ref64(T)), rtol=1e-3, atol=0)


def test_ieee_matches_tf32x3_on_well_conditioned_inputs():
    n = 256
    gen = np.random.default_rng(780)
    A = (randn((16, n, n), np.float32, gen) / np.sqrt(n) + 2 * np.eye(n)).astype(np.float32)
    s1, l1 = host(fx.slogdet(cuda(A), prec="ieee"))
    s2, l2 = host(fx.slogdet(cuda(A), prec="tf32x3"))
    assert np.array_equal(s1, s2)
    assert np.max(np.abs(l1 - l2)) < 1e-4 * max(1.0, np.abs(l1).max())


def test_ieee_gather_matches_materialised():
    gen = np.random.default_rng(790)
    phi = (gen.standard_normal((512, 256)) / 16.0).astype(np.float32)
    occ = np.sort(np.stack([gen.choice(512, 256, replace=False) for _ in range(24)]), axis=1).astype(np.int32)
    P, O = cuda(phi), torch.from_numpy(occ).cuda()
    s1, l1 = host(fx.slogdet_gather(P, O, prec="ieee"))
    s2, l2 = host(fx.slogdet(cuda(phi[occ]), prec="ieee"))
    assert np.array_equal(s1, s2) and np.array_equal(l1, l2)


@pytest.mark.parametrize("n,B", [(128, 1500), (256, 400)])
def test_ieee_several_matrices_per_block(n, B):
    """More matrices than resident blocks (592 at n <= 128, 148 at n = 256): each block walks
    several members in turn. Forward and gradient against float64, per member."""
    g = torch.Generator(device="cuda").manual_seed(800 + n)
    A = torch.randn(B, n, n, device="cuda", generator=g)
    s, l, G = fx.slogdet_parts(A, prec="ieee")
    A64 = A.double()
    s64, l64 = torch.linalg.slogdet(A64)
    assert torch.equal(s.double(), s64)
    err = (l.double() - l64).abs()
    eps = np.finfo(np.float32).eps
    over = torch.nonzero(err > 1e-4 * l64.abs().clamp(min=1)).flatten()
    if over.numel():
        cond = torch.linalg.cond(A64[over])
        assert bool((err[over] <= 2 * cond * eps).all())
    R = torch.linalg.inv(A64[:64]).transpose(-1, -2)
    for i in range(64):
        rel = float((G[i].double() - R[i]).abs().max() / R[i].abs().max())
        cond = float(torch.linalg.cond(A64[i]))
        assert rel <= max(1e-3, cond * eps), (i, rel, cond)
