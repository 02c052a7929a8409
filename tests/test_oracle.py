"""Pins the CPU oracle (the numpy restatement of the reference's generic path) against
the float64 / complex128 oracles of the reference's own test suite, case by case as in
ChenAo-Phys/fermix tests/test_fermix.py, and against the committed golden fixtures."""

import os

import numpy as np
import pytest

import oracle
from oracle import fallback as F
from oracle.refs64 import (
    adjT64,
    assert_sign,
    is_complex,
    log_tol,
    pf64,
    pf_gradT64,
    pf_ref64,
    randn,
    rank_deficient,
    ref64,
    rel_tol,
    relerr,
    shifted,
    skew,
    skew_rank_deficient,
    tol,
)

DTYPES = [np.float32, np.float64, np.complex64, np.complex128]
IDS = ["f32", "f64", "c64", "c128"]
dtypes = pytest.mark.parametrize("dtype", DTYPES, ids=IDS)


@pytest.mark.parametrize("n", [3, 8, 40, 96])
@dtypes
def test_oracle_slogdet_matches_numpy(n, dtype):
    A = randn((5, n, n), dtype, np.random.default_rng(100 + n))
    s, l = oracle.slogdet(A)
    s64, l64 = np.linalg.slogdet(ref64(A))
    assert s.dtype == dtype and l.dtype == np.finfo(dtype).dtype
    assert_sign(s, s64, dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - l64)) < log_tol(dtype, n)


@pytest.mark.parametrize("n", [4, 6, 34, 64])
@dtypes
def test_oracle_slogpf_matches_pf_ref64(n, dtype):
    S = skew(randn((5, n, n), dtype, np.random.default_rng(200 + n)))
    s, l = oracle.slogpf(S, skew_symmetrize=False)
    ref = [pf_ref64(S[i]) for i in range(5)]
    assert_sign(s, [r[0] for r in ref], dtype, log_tol(dtype))
    assert np.max(np.abs(l - [r[1] for r in ref])) < log_tol(dtype)


@dtypes
def test_oracle_values_and_odd_n(dtype):
    gen = np.random.default_rng(3)
    rt = rel_tol(dtype)
    A = randn((2, 3, 5, 5), dtype, gen)
    d = oracle.det(A)
    assert d.shape == (2, 3) and d.dtype == dtype
    assert np.allclose(d, np.linalg.det(ref64(A)), rtol=rt, atol=rt / 10)
    S = skew(randn((4, 12, 12), dtype, gen))
    p = oracle.pf(S)
    # pf(a) skew-symmetrises a: (S - S^T) / 2 = S for skew S
    assert np.allclose(p, [pf64(S[i]) for i in range(4)], rtol=rt, atol=rt / 10)
    odd = np.zeros((3, 7, 7), dtype)
    assert np.all(oracle.pf(odd) == 0)
    s, l = oracle.slogpf(odd)
    assert np.all(s == 0) and np.all(np.isneginf(l))


@dtypes
def test_oracle_slogdet_grad(dtype):
    A = shifted((4, 48, 48), dtype, 3, np.random.default_rng(4))
    g = oracle.slogdet_grad(A)
    assert relerr(g, np.swapaxes(np.linalg.inv(ref64(A)), -1, -2)) < rel_tol(dtype)
    A = shifted((4, 3, 3), dtype, 3, np.random.default_rng(4))  # the polynomial rule
    g = oracle.slogdet_grad(A)
    assert relerr(g, np.swapaxes(np.linalg.inv(ref64(A)), -1, -2)) < rel_tol(dtype)


@pytest.mark.parametrize("n", [6, 32, 96])
@dtypes
def test_oracle_slogpf_grad(n, dtype):
    A = randn((4, n, n), dtype, np.random.default_rng(1000 + n))  # seeds with cond(S) < 1e3
    g = oracle.slogpf_grad(A)
    S = 0.5 * skew(ref64(A))
    assert relerr(g, 0.5 * np.swapaxes(np.linalg.inv(S), -1, -2)) < rel_tol(dtype)


@dtypes
def test_oracle_det_pf_grad_regular(dtype):
    gen = np.random.default_rng(6)
    A = shifted((3, 12, 12), dtype, 2, gen)
    ref = np.stack([np.linalg.det(a) * np.linalg.inv(a).T for a in ref64(A)])
    assert relerr(oracle.det_grad(A), ref) < rel_tol(dtype)
    S = skew(randn((3, 12, 12), dtype, gen))
    ref = np.stack([0.5 * pf64(s) * np.linalg.inv(s).T for s in ref64(S)])
    assert relerr(oracle.pf_grad(S, skew_symmetrize=False), ref) < rel_tol(dtype)


@dtypes
def test_oracle_singular_slog_grads_zero(dtype):
    gen = np.random.default_rng(7)
    n = 40
    A = randn((3, n, n), dtype, gen)
    A[0, :, 5] = 0.0
    A[1] = 0.0
    s, l = oracle.slogdet(A)
    assert np.all(s[:2] == 0) and np.all(np.isneginf(l[:2]))
    g = oracle.slogdet_grad(A)
    assert np.all(np.isfinite(g)) and np.all(g[:2] == 0)
    S = skew(randn((3, n, n), dtype, gen))
    S[0, 7, :] = 0.0
    S[0, :, 7] = 0.0
    g = oracle.slogpf_grad(S, skew_symmetrize=False)
    assert np.all(np.isfinite(g)) and np.all(g[0] == 0)


@pytest.mark.parametrize("n", [3, 8, 40])
@dtypes
def test_oracle_det_grad_singular(n, dtype):
    B = 6
    A = shifted((B, n, n), dtype, 2, np.random.default_rng(8))
    A[0, :, 1] = 0.0
    A[1, 2 % n] = 0.0
    A[2] = 0.0
    A[3, :, 0] = 0.0
    A[3, :, 1] = 0.0
    A[4, :, 0] = 0.0
    A[4, 1] = 0.0
    g = oracle.det_grad(A)
    assert np.all(np.isfinite(g))
    ref = np.stack([adjT64(a) for a in ref64(A)])
    scale = max(np.abs(ref).max(), 1e-30)
    assert np.max(np.abs(g - ref)) < rel_tol(dtype) * scale
    assert np.all(g[2] == 0) and np.all(g[3] == 0)
    for k in (0, 1, 4):
        assert np.abs(ref[k]).max() > 0 and relerr(g[k], ref[k]) < rel_tol(dtype)


@pytest.mark.parametrize("n", [8, 24])
@dtypes
def test_oracle_det_grad_near_singular(n, dtype):
    A = rank_deficient((4, n, n), dtype, np.random.default_rng(9))
    g = oracle.det_grad(A)
    ref = np.stack([adjT64(a) for a in ref64(A)])
    for k in range(len(A)):
        assert relerr(g[k], ref[k]) < tol(dtype, 1e-4, 1e-9)


@pytest.mark.parametrize("n", [4, 8, 14])
@dtypes
def test_oracle_pf_grad_singular(n, dtype):
    B = 4
    S = skew(randn((B, n, n), dtype, np.random.default_rng(10)))
    S[0, 3 % n, :] = 0.0
    S[0, :, 3 % n] = 0.0
    S[1] = 0.0
    S[2, 1, :] = 0.0
    S[2, :, 1] = 0.0
    S[2, 3 % n, :] = 0.0
    S[2, :, 3 % n] = 0.0
    g = oracle.pf_grad(S, skew_symmetrize=False)
    assert np.all(np.isfinite(g))
    ref = np.stack([pf_gradT64(s) for s in ref64(S)])
    scale = max(np.abs(ref).max(), 1e-30)
    assert np.max(np.abs(g - ref)) < rel_tol(dtype) * scale
    assert np.all(g[1] == 0) and np.abs(ref[0]).max() > 0


@pytest.mark.parametrize("n", [8, 24])
@dtypes
def test_oracle_pf_grad_near_singular(n, dtype):
    S = skew_rank_deficient((4, n, n), dtype, np.random.default_rng(11))
    g = oracle.pf_grad(S, skew_symmetrize=False)
    ref = np.stack([pf_gradT64(s) for s in ref64(S)])
    for k in range(len(S)):
        assert relerr(g[k], ref[k]) < tol(dtype, 1e-4, 1e-9)


def test_oracle_rejects_bad_input():
    with pytest.raises(TypeError):
        oracle.slogdet(np.eye(4, dtype=np.float16))
    with pytest.raises(TypeError):
        oracle.slogdet(np.eye(4, dtype=np.int32))
    with pytest.raises(ValueError):
        oracle.slogdet(np.zeros((3, 4), np.float32))


GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="golden fixtures not generated")
def test_oracle_matches_golden_fixtures():
    """The committed fixtures (tests/golden/make_golden.py) hold seeded inputs with
    their float64 reference answers from numpy / the reference test suite's oracles;
    the oracle must reproduce them within the reference's tolerances."""
    from tests.golden.make_golden import CASES, check_case

    z = np.load(GOLDEN)
    for name in CASES:
        check_case(name, z, F)


# ---------------------------------------------------------------- rank-k row moves
@pytest.mark.parametrize("dtype", [np.float64, np.complex128])
@pytest.mark.parametrize("n,k", [(1, 1), (6, 2), (20, 5), (40, 16)])
def test_move_oracle_woodbury_matches_refactorisation(dtype, n, k):
    """The Woodbury route of the move oracle (the kernels' algorithm) against refactoring
    the moved matrix with the getrf restatement."""
    from oracle import moves

    rng = np.random.default_rng(n * 31 + k)
    B = 3
    A = rng.standard_normal((B, n, n))
    U = rng.standard_normal((B, k, n))
    if np.dtype(dtype).kind == "c":
        A = A + 1j * rng.standard_normal((B, n, n))
        U = U + 1j * rng.standard_normal((B, k, n))
    A, U = A.astype(dtype), U.astype(dtype)
    idx = np.stack([rng.choice(n, k, replace=False) for _ in range(B)])
    G = np.swapaxes(np.linalg.inv(A), -1, -2)
    s1, l1 = moves.ratio_direct(A, U, idx)
    s2, l2 = moves.ratio_woodbury(G, U, idx)
    assert np.allclose(l1, l2, rtol=0, atol=1e-10)
    assert np.allclose(s1, s2, rtol=0, atol=1e-10)
    G1 = moves.inverse_direct(A, U, idx)
    G2 = moves.update_woodbury(G, U, idx)
    assert np.abs(G1 - G2).max() <= 1e-9 * np.abs(G1).max()


@pytest.mark.parametrize("dtype", [np.float64, np.complex128])
@pytest.mark.parametrize("n", [2, 6, 20])
def test_pf_move_oracle_woodbury_matches_refactorisation(dtype, n):
    """The Pfaffian one-index move: the rank-2 skew Woodbury route against refactoring S'
    with the Parlett-Reid restatement."""
    from oracle import moves

    rng = np.random.default_rng(n)
    B = 3
    A = rng.standard_normal((B, n, n))
    U = rng.standard_normal((B, n))
    if np.dtype(dtype).kind == "c":
        A = A + 1j * rng.standard_normal((B, n, n))
        U = U + 1j * rng.standard_normal((B, n))
    S = (A - np.swapaxes(A, -1, -2)).astype(dtype)
    U = U.astype(dtype)
    idx = rng.integers(0, n, size=B)
    G = 0.5 * np.swapaxes(np.linalg.inv(S), -1, -2)
    s1, l1 = moves.pf_ratio_direct(S, U, idx)
    r = moves.pf_ratio_woodbury(G, U, idx)
    assert np.allclose(np.log(np.abs(r)), l1, rtol=0, atol=1e-9)
    assert np.allclose(r / np.abs(r), s1, rtol=0, atol=1e-9)
    G1 = moves.pf_grad_direct(S, U, idx)
    assert np.abs(moves.pf_update_woodbury(G, U, idx) - G1).max() <= 1e-8 * np.abs(G1).max()


@pytest.mark.parametrize("dtype", [np.float64, np.complex128])
@pytest.mark.parametrize("n,k", [(6, 1), (10, 2), (16, 5), (24, 8)])
def test_pf_move_k_recurrence_matches_refactorisation(dtype, n, k):
    """The G-only k-index Pfaffian move (the CUDA kernels' algorithm) against refactoring
    the moved matrix, and k = 1 against the one-index Woodbury route."""
    from oracle import moves

    rng = np.random.default_rng(n + 100 * k)
    B = 4
    S = rng.standard_normal((B, n, n))
    if np.dtype(dtype).kind == "c":
        S = S + 1j * rng.standard_normal((B, n, n))
    S = S - np.swapaxes(S, -1, -2)
    G = 0.5 * np.swapaxes(np.linalg.inv(S), -1, -2)
    idx = np.stack([rng.choice(n, k, replace=False) for _ in range(B)])
    U = rng.standard_normal((B, k, n)) + (1j * rng.standard_normal((B, k, n)) if np.dtype(dtype).kind == "c" else 0)
    s, l = moves.pf_ratio_direct_k(S, U, idx)
    rho = moves.pf_ratio_woodbury_k(G, U, idx)
    assert np.abs(np.log(np.abs(rho)) - l).max() < 1e-9
    assert np.abs(rho / np.abs(rho) - s).max() < 1e-9
    ref = moves.pf_grad_direct_k(S, U, idx)
    assert np.abs(moves.pf_update_woodbury_k(G, U, idx) - ref).max() / np.abs(ref).max() < 1e-9
    if k == 1:
        one = moves.pf_update_woodbury(G, U[:, 0], idx[:, 0])
        assert np.abs(moves.pf_update_woodbury_k(G, U, idx) - one).max() / np.abs(one).max() < 1e-12
