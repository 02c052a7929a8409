"""k-index Pfaffian moves (fermix_slogpf_ratio_k / fermix_slogpf_update_k) against the move
oracle: refactoring the moved skew matrix (pf_ratio_direct_k / pf_grad_direct_k) and the
G-only recurrence the kernels implement (pf_update_woodbury_k). Tolerances as the one-index
move tests: logabs 1e-4 (32-bit) / 1e-10 (64-bit) of max(1, |ref|), G' relative 1e-3 / 1e-8."""

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
    """A well-conditioned skew S (pair blocks [[0, 3], [-3, 0]] plus noise), G = S^-T / 2 in
    float64, new rows near the replaced ones, distinct indices."""
    rng = np.random.default_rng(seed)
    S = rng.standard_normal((B, n, n)) / np.sqrt(n)
    if np.dtype(dtype).kind == "c":
        S = S + 1j * rng.standard_normal((B, n, n)) / np.sqrt(n)
    S = S - np.swapaxes(S, -1, -2)
    r = np.arange(0, n - 1, 2)
    S[:, r, r + 1] += 3.0
    S[:, r + 1, r] -= 3.0
    idx = np.stack([rng.choice(n, k, replace=False) for _ in range(B)]).astype(np.int32)
    U = np.take_along_axis(S, idx[:, :, None].repeat(n, -1), axis=1)
    U = U + 0.2 * rng.standard_normal(U.shape) / np.sqrt(n)
    G = 0.5 * np.swapaxes(np.linalg.inv(S), -1, -2)
    return S, G.astype(dtype), U.astype(dtype), idx


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
@pytest.mark.parametrize("n,k", [(2, 1), (8, 2), (33 + 1, 3), (128, 1), (128, 4), (200, 8), (64, 16)])
def test_k_moves_match_refactorisation(dtype, n, k):
    B = 5
    S, G, U, idx = _case(dtype, B, n, k, seed=n * 31 + k)
    s, l = host(fx.slogpf_ratio_k(cuda(G), cuda(U), cuda(idx)))
    s_ref, l_ref = moves.pf_ratio_direct_k(S, U, idx)
    tol = 1e-4 if _is32(dtype) else 1e-10
    assert np.abs(l - l_ref).max() <= tol * max(1.0, np.abs(l_ref).max()), (l, l_ref)
    if np.dtype(dtype).kind == "c":
        assert np.abs(s - s_ref).max() <= (1e-4 if _is32(dtype) else 1e-9)
    else:
        assert np.array_equal(s, s_ref.astype(s.dtype))
    s2, l2, G2 = host(fx.slogpf_update_k(cuda(G), cuda(U), cuda(idx)))
    assert np.array_equal(s2, s) and np.array_equal(l2, l)  # the update's ratio is the ratio call's
    gtol = 1e-3 if _is32(dtype) else 1e-8
    ref = moves.pf_grad_direct_k(S, U, idx)
    assert np.abs(G2 - ref).max() / np.abs(ref).max() < gtol
    wood = moves.pf_update_woodbury_k(G, U, idx)
    assert np.abs(G2 - wood).max() / np.abs(wood).max() < gtol


def test_k1_equals_one_index_move():
    S, G, U, idx = _case(np.float64, 6, 50, 1, seed=7)
    s1, l1, G1 = host(fx.slogpf_update_k(cuda(G), cuda(U), cuda(idx)))
    s0, l0, G0 = host(fx.slogpf_update(cuda(G), cuda(U[:, 0]), cuda(idx[:, 0])))
    assert np.array_equal(s1, s0)
    assert np.abs(l1 - l0).max() < 1e-12
    assert np.abs(G1 - G0).max() / np.abs(G0).max() < 1e-12


def test_k_moves_accept_mask_bad_index_and_singular():
    n, k = 40, 3
    S, G, U, idx = _case(np.complex128, 6, n, k, seed=11)
    idx[2, 1] = n + 5              # bad index: NaN ratio, G kept
    U[4] = 0.0                      # replaced rows / columns all zero: S' singular
    acc = np.array([1, 0, 1, 1, 1, 1], dtype=bool)
    g = cuda(G)
    s, l, out = fx.slogpf_update_k(g, cuda(U), cuda(idx), accept=cuda(acc), inplace=True)
    s, l, out = host(s), host(l), host(out)
    assert np.isnan(l[2]) and np.array_equal(out[2], G[2])
    assert np.array_equal(out[1], G[1])          # rejected
    assert s[4] == 0 and np.isneginf(l[4]) and np.all(out[4] == 0)
    ok = [0, 3, 5]
    ref = moves.pf_grad_direct_k(S[ok], U[ok], idx[ok])
    assert np.abs(out[ok] - ref).max() / np.abs(ref).max() < 1e-8


def test_k_move_walk_matches_refactoring_the_final_matrix():
    """Ten 2-index moves in a row on float64, against refactoring the final matrix."""
    n, B = 60, 3
    S, G, _, _ = _case(np.float64, B, n, 2, seed=21)
    rng = np.random.default_rng(22)
    g = cuda(G)
    logsum = np.zeros(B)
    for step in range(10):
        idx = np.stack([rng.choice(n, 2, replace=False) for _ in range(B)]).astype(np.int32)
        U = np.take_along_axis(S, idx[:, :, None].repeat(n, -1), axis=1) + 0.2 * rng.standard_normal((B, 2, n)) / 8
        s, l, g = fx.slogpf_update_k(g, cuda(U), cuda(idx), inplace=True)
        logsum += host(l)
        S = moves.pf_apply_move_k(S, U, idx)
    ref = 0.5 * np.swapaxes(np.linalg.inv(S), -1, -2)
    assert np.abs(host(g) - ref).max() / np.abs(ref).max() < 1e-8
