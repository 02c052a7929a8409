"""slogpf / pf under prec="ieee" for float32, 8 <= n <= 128: the tensor-memory resident
Parlett-Reid with IEEE float32 FMA block updates. Checked against the 64-bit references
of the reference suite (tests/test_fermix.py:95-144) and the oracle, for sizes that fill
one to eight panels (8 pairs each) and leave partial panels, singular members and the
primal-under-gradient identity."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx
import oracle
from oracle.refs64 import log_tol, pf64, pf_ref64, randn, relerr, skew, skew_rank_deficient
from tests.helpers import cuda, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [8, 10, 16, 34, 62, 64, 96, 126, 128])
def test_ieee_slogpf_fwd_and_grad(n):
    gen = np.random.default_rng(900 + n)
    S = skew(randn((6, n, n), np.float32, gen))
    s, l = host(fx.slogpf(cuda(S), prec="ieee", skew_symmetrize=False))
    ref = [pf_ref64(S[i]) for i in range(6)]
    assert np.array_equal(s, np.array([r[0] for r in ref], np.float32))
    assert np.max(np.abs(l - [r[1] for r in ref])) < log_tol(np.float32, n)
    so, lo = oracle.slogpf(S, skew_symmetrize=False)
    assert np.array_equal(s, so)
    assert np.max(np.abs(l - lo)) < log_tol(np.float32, n)
    # the gradient call's primal is the forward's, bit for bit
    s2, l2, g = host(fx.slogpf_parts(cuda(S), prec="ieee", skew_symmetrize=False))
    assert np.array_equal(s, s2) and np.array_equal(l, l2)
    # gradients: 1e-3 relative per matrix, or cond(S) * eps32 for the ill-conditioned ones
    g_ref = 0.5 * np.swapaxes(np.linalg.inv(S.astype(np.float64)), -1, -2)
    eps = np.finfo(np.float32).eps
    for i in range(len(S)):
        cond = np.linalg.cond(S[i].astype(np.float64))
        assert relerr(g[i], g_ref[i]) <= max(1e-3, cond * eps), (i, relerr(g[i], g_ref[i]), cond)


def test_ieee_slogpf_singular_members_and_values():
    n = 128
    gen = np.random.default_rng(950)
    S = skew(randn((4, n, n), np.float32, gen))
    S[1] = skew_rank_deficient((n, n), np.float32, gen)
    S[2] = 0.0
    x = cuda(S, requires_grad=True)
    s, l = fx.slogpf(x, prec="ieee", skew_symmetrize=False)
    (g,) = torch.autograd.grad(l.sum(), x)
    s, l, g = host(s), host(l), host(g)
    assert s[2] == 0 and np.isneginf(l[2]) and np.all(g[2] == 0)
    assert np.all(np.isfinite(g))
    for b in (0, 3):
        sr, lr = pf_ref64(S[b])
        assert s[b] == sr and abs(l[b] - lr) < log_tol(np.float32, n)
    # pf values (n = 16: |pf| stays within float32) against the 64-bit Pfaffian
    T = skew(randn((3, 16, 16), np.float32, gen))
    p = host(fx.pf(cuda(T), prec="ieee"))
    ref = np.array([pf64(T[i].astype(np.float64)) for i in range(3)])
    assert np.allclose(p, ref, rtol=1e-4, atol=0)


def test_ieee_matches_tf32x3_on_well_conditioned_inputs():
    """Both precisions on the same skew inputs (diagonally dominant pairs, so both are
    accurate to float32): the same signs, logabs within the float32 tolerance."""
    n = 128
    gen = np.random.default_rng(960)
    A = randn((64, n, n), np.float32, gen) / np.sqrt(n)
    J = np.kron(np.eye(n // 2), np.array([[0.0, 1.0], [-1.0, 0.0]])).astype(np.float32)
    S = (skew(A) + 4 * J).astype(np.float32)
    s1, l1 = host(fx.slogpf(cuda(S), prec="ieee"))
    s2, l2 = host(fx.slogpf(cuda(S), prec="tf32x3"))
    assert np.array_equal(s1, s2)
    assert np.max(np.abs(l1 - l2)) < 1e-4 * max(1.0, np.abs(l1).max())
