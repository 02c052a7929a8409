"""Rank-k row moves (slogdet_ratio / slogdet_update, fermix_slogdet_ratio /
fermix_slogdet_update) against the move oracle: the determinant ratio and the new
inverse-transpose of a matrix whose rows idx are replaced, from G = A^-T alone.

Tolerances: the forward ones of the slogdet tests for the ratio's logabs, and relative
1e-3 (32-bit) / 1e-8 (64-bit) of the largest entry for the updated G."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx
from oracle import moves

from tests.helpers import DTYPES, IDS, cuda, host

pytestmark = pytest.mark.gpu


def _is32(dtype):
    return np.dtype(dtype) in (np.dtype(np.float32), np.dtype(np.complex64))


def _case(dtype, B, n, k, seed):
    """A well-conditioned batch A (identity shift), G = A^-T in float64 cast to dtype, new
    rows U and distinct indices."""
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((B, n, n)) / np.sqrt(n) + 2.0 * np.eye(n)
    U = rng.standard_normal((B, k, n)) / np.sqrt(n)
    if np.dtype(dtype).kind == "c":
        A = A + 1j * rng.standard_normal((B, n, n)) / np.sqrt(n)
        U = U + 1j * rng.standard_normal((B, k, n)) / np.sqrt(n)
    idx = np.stack([rng.choice(n, k, replace=False) for _ in range(B)]).astype(np.int32)
    for b in range(B):  # keep A' regular: the new row r is near the old row idx_r
        U[b] += A[b, idx[b]]
    G = np.swapaxes(np.linalg.inv(A), -1, -2)
    return A, G.astype(dtype), U.astype(dtype), idx


def _check_ratio(dtype, sign, logabs, A, U, idx):
    s_ref, l_ref = moves.ratio_direct(A, U, idx)
    tol = 1e-4 if _is32(dtype) else 1e-10
    assert np.abs(logabs - l_ref).max() <= tol * max(1.0, np.abs(l_ref).max())
    if np.dtype(dtype).kind == "c":
        assert np.abs(sign - s_ref).max() <= (1e-4 if _is32(dtype) else 1e-10)
        assert np.allclose(np.abs(sign), 1.0, atol=1e-5)
    else:
        assert np.array_equal(sign, s_ref.astype(sign.dtype))


def _relerr(x, ref):
    return np.abs(x - ref).max() / np.abs(ref).max()


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
@pytest.mark.parametrize("n,k", [(1, 1), (8, 1), (33, 3), (128, 1), (128, 4), (300, 16)])
def test_ratio_and_update_match_refactorisation(dtype, n, k):
    _ratio_and_update(dtype, n, k)


@pytest.mark.parametrize("dtype,n,k", [
    (np.float32, 1024, 16),  # the register row kernel with 16 coefficients (U, H beyond shared memory)
    (np.float32, 128, 3),    # shared-memory row kernel, k not a power of two (padded coefficients)
    (np.float64, 128, 7),    # as above, 16 coefficient slots
], ids=["f32-n1024-k16", "f32-n128-k3", "f64-n128-k7"])
def test_row_kernel_variants_match_refactorisation(dtype, n, k):
    _ratio_and_update(dtype, n, k)


def _ratio_and_update(dtype, n, k):
    B = 6
    A, G, U, idx = _case(dtype, B, n, k, seed=n * 17 + k)
    s, l = fx.slogdet_ratio(cuda(G), cuda(U), cuda(idx))
    _check_ratio(dtype, host(s), host(l), A, U, idx)
    s2, l2, G2 = fx.slogdet_update(cuda(G), cuda(U), cuda(idx))
    # the update's ratio is the ratio call's, bit for bit
    assert np.array_equal(host(s2), host(s)) and np.array_equal(host(l2), host(l))
    tol = 1e-3 if _is32(dtype) else 1e-8
    assert _relerr(host(G2), moves.inverse_direct(A, U, idx)) < tol
    assert _relerr(host(G2), moves.update_woodbury(G, U, idx)) < tol


@pytest.mark.parametrize("dtype", [np.float32, np.complex128], ids=["f32", "c128"])
def test_accept_mask_inplace_and_batch_dims(dtype):
    n, k = 64, 2
    A, G, U, idx = _case(dtype, 6, n, k, seed=5)
    shape = (2, 3)
    acc = np.array([1, 0, 1, 1, 0, 0], dtype=bool)
    g = cuda(G.reshape(shape + (n, n)))
    g0 = host(g).copy()
    s, l, out = fx.slogdet_update(g, cuda(U.reshape(shape + (k, n))), cuda(idx.reshape(shape + (k,))),
                                  accept=cuda(acc.reshape(shape)), inplace=True)
    assert out.data_ptr() == g.data_ptr() and tuple(s.shape) == shape and tuple(l.shape) == shape
    _check_ratio(dtype, host(s).reshape(-1), host(l).reshape(-1), A, U, idx)
    new = host(g).reshape(6, n, n)
    ref = moves.inverse_direct(A, U, idx)
    tol = 1e-3 if _is32(dtype) else 1e-8
    for b in range(6):
        if acc[b]:
            assert _relerr(new[b], ref[b]) < tol
        else:
            assert np.array_equal(new[b], g0.reshape(6, n, n)[b])  # rejected: untouched bits


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
def test_sequence_of_single_row_moves(dtype):
    """A QMC-like walk: 20 accepted one-row moves applied to G in place; the accumulated
    log-ratio and the final G match refactoring the final matrix."""
    n, B = 48, 4
    rng = np.random.default_rng(11)
    A, G, _, _ = _case(dtype, B, n, 1, seed=3)
    g = cuda(G)
    total = np.zeros(B)
    cur = A.astype(np.complex128 if np.dtype(dtype).kind == "c" else np.float64)
    for step in range(20):
        idx = rng.integers(0, n, size=(B, 1)).astype(np.int32)
        U = np.stack([cur[b, idx[b]] for b in range(B)]) + 0.3 * rng.standard_normal((B, 1, n)) / np.sqrt(n)
        U = U.astype(dtype)
        _, l, _ = fx.slogdet_update(g, cuda(U), cuda(idx), inplace=True)
        total += host(l)
        cur = moves.apply_move(cur, U, idx)
    _, l_ref = moves.ratio_direct(A, cur, np.tile(np.arange(n, dtype=np.int32), (B, 1)))
    tol = 1e-3 if _is32(dtype) else 1e-9
    assert np.abs(total - l_ref).max() <= tol * max(1.0, np.abs(l_ref).max())
    ref = np.swapaxes(np.linalg.inv(cur), -1, -2)
    assert _relerr(host(g), ref) < (2e-3 if _is32(dtype) else 1e-8)


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
def test_singular_move_bad_index_and_empty_move(dtype):
    n, k = 16, 2
    A, G, U, idx = _case(dtype, 3, n, k, seed=9)
    U[0] = 0  # member 0: zero rows -> R = 0 exactly -> (0, -inf), G' = 0
    idx[1, 1] = n  # member 1: an index outside [0, n) -> NaN, G kept
    g = cuda(G)
    s, l, out = fx.slogdet_update(g, cuda(U), cuda(idx))
    s, l, out = host(s), host(l), host(out)
    assert s[0] == 0 and l[0] == -np.inf and np.all(out[0] == 0)
    assert np.isnan(l[1]) and np.all(np.isnan(s[1].real)) and np.array_equal(out[1], G[1])
    _check_ratio(dtype, s[2:], l[2:], A[2:], U[2:], idx[2:])
    # k = 0: ratio 1, G unchanged
    s0, l0, g0 = fx.slogdet_update(cuda(G), cuda(U[:, :0]), cuda(idx[:, :0]))
    assert np.all(host(s0) == 1) and np.all(host(l0) == 0) and np.array_equal(host(g0), G)


def test_argument_errors():
    G = torch.zeros((2, 8, 8), device="cuda")
    with pytest.raises(ValueError):
        fx.slogdet_ratio(G, torch.zeros((2, 17, 8), device="cuda"), torch.zeros((2, 17), dtype=torch.int32))
    with pytest.raises(TypeError):
        fx.slogdet_ratio(G, torch.zeros((2, 1, 8), device="cuda", dtype=torch.float64),
                         torch.zeros((2, 1), dtype=torch.int32))
    with pytest.raises(ValueError):
        fx.slogdet_ratio(G, torch.zeros((2, 1, 8), device="cuda"), torch.zeros((2, 2), dtype=torch.int32))


# ---------------------------------------------------------------- Pfaffian one-index moves
def _pf_case(dtype, B, n, seed):
    """A skew S (well conditioned: a block-diagonal [[0, 2], [-2, 0]] shift), G = S^-T / 2 in
    float64 cast to dtype, and a new row near the old row idx."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((B, n, n)) / np.sqrt(n)
    if np.dtype(dtype).kind == "c":
        X = X + 1j * rng.standard_normal((B, n, n)) / np.sqrt(n)
    J = np.zeros((n, n))
    for q in range(0, n - 1, 2):
        J[q, q + 1], J[q + 1, q] = 2.0, -2.0
    S = X - np.swapaxes(X, -1, -2) + J
    idx = rng.integers(0, n, size=B).astype(np.int32)
    U = S[np.arange(B), idx] + 0.3 * (rng.standard_normal((B, n)) / np.sqrt(n))
    G = 0.5 * np.swapaxes(np.linalg.inv(S), -1, -2)
    return S, G.astype(dtype), U.astype(dtype), idx


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
@pytest.mark.parametrize("n", [2, 8, 34, 128, 300])
def test_pf_move_matches_refactorisation(dtype, n):
    S, G, U, idx = _pf_case(dtype, 6, n, seed=n + 7)
    s, l = fx.slogpf_ratio(cuda(G), cuda(U), cuda(idx))
    s_ref, l_ref = moves.pf_ratio_direct(S, U, idx)
    tol = 1e-4 if _is32(dtype) else 1e-10
    assert np.abs(host(l) - l_ref).max() <= tol * max(1.0, np.abs(l_ref).max())
    if np.dtype(dtype).kind == "c":
        assert np.abs(host(s) - s_ref).max() <= (1e-4 if _is32(dtype) else 1e-10)
    else:
        assert np.array_equal(host(s), s_ref.astype(host(s).dtype))
    s2, l2, G2 = fx.slogpf_update(cuda(G), cuda(U), cuda(idx))
    assert np.array_equal(host(s2), host(s)) and np.array_equal(host(l2), host(l))
    gt = 1e-3 if _is32(dtype) else 1e-8
    assert _relerr(host(G2), moves.pf_grad_direct(S, U, idx)) < gt
    assert _relerr(host(G2), moves.pf_update_woodbury(G, U, idx)) < gt


@pytest.mark.parametrize("dtype", [np.float32, np.complex128], ids=["f32", "c128"])
def test_pf_move_walk_accept_singular_bad_index(dtype):
    n, B = 40, 4
    rng = np.random.default_rng(21)
    S, G, _, _ = _pf_case(dtype, B, n, seed=5)
    g = cuda(G)
    cur = S.astype(np.complex128 if np.dtype(dtype).kind == "c" else np.float64)
    total = np.zeros(B)
    for step in range(15):
        idx = rng.integers(0, n, size=B).astype(np.int32)
        U = (cur[np.arange(B), idx] + 0.3 * rng.standard_normal((B, n)) / np.sqrt(n)).astype(dtype)
        acc = rng.random(B) < 0.7
        _, l, _ = fx.slogpf_update(g, cuda(U), cuda(idx), accept=cuda(acc), inplace=True)
        total += np.where(acc, host(l), 0.0)
        nxt = moves.pf_apply_move(cur, U, idx)
        cur = np.where(acc[:, None, None], nxt, cur)
    s0, l0 = moves._slogpf(S.astype(cur.dtype))
    s1, l1 = moves._slogpf(cur)
    tol = 1e-3 if _is32(dtype) else 1e-9
    assert np.abs(total - (l1 - l0)).max() <= tol * max(1.0, np.abs(l1 - l0).max())
    ref = 0.5 * np.swapaxes(np.linalg.inv(cur), -1, -2)
    assert _relerr(host(g), ref) < (2e-3 if _is32(dtype) else 1e-8)
    # a zero row gives ratio 0 -> (0, -inf) and G' = 0; an out-of-range index -> NaN, G kept
    U = np.zeros((B, n), dtype=dtype)
    idx = np.array([0, n, 1, 2], dtype=np.int32)
    U[2:] = (cur[np.arange(2, 4), idx[2:]]).astype(dtype)
    s, l, out = fx.slogpf_update(cuda(G), cuda(U), cuda(idx))
    s, l, out = host(s), host(l), host(out)
    assert s[0] == 0 and l[0] == -np.inf and np.all(out[0] == 0)
    assert np.isnan(l[1]) and np.array_equal(out[1], G[1])
