"""CPU oracle of the rank-k row moves (TEST INFRASTRUCTURE ONLY).

The reference has no entry point for these moves: its gradient path exports the inverse
(``_lu_parts``, ``src/fermix/_inverse.py:502-531``), and a QMC caller replaces rows of the
Slater matrix with it. The oracle is therefore the moves' definition, computed two ways in
float64 / complex128:

* ``ratio_direct`` / ``inverse_direct``: refactor the moved matrix A' from scratch with the
  LAPACK-getrf restatement of the reference's generic path (``oracle.fallback.slogdet``,
  ``src/fermix/_fallback.py:19-59``) and take ``inv(A')^T``;
* ``ratio_woodbury`` / ``update_woodbury``: the same quantities from G = A^-T alone,
  det(A') / det(A) = det(U A^-1 E) and G' = G - (V^T - E) R^-T G[idx, :] with V = U A^-1,
  which is the algorithm the CUDA kernels implement.

The tests pin the second route against the first, then the CUDA path against both.
"""

import numpy as np

from .fallback import slogdet as _slogdet


def _wide(x):
    x = np.asarray(x)
    return x.astype(np.complex128 if np.iscomplexobj(x) else np.float64)


def apply_move(A, rows, idx):
    """A' = A with rows idx[..., r] replaced by rows[..., r, :]."""
    A = np.array(A, copy=True)
    B = A.reshape((-1,) + A.shape[-2:])
    U = np.asarray(rows).reshape((B.shape[0],) + np.asarray(rows).shape[-2:])
    I = np.asarray(idx).reshape(B.shape[0], -1)
    for b in range(B.shape[0]):
        for r in range(I.shape[1]):
            B[b, I[b, r]] = U[b, r]
    return B.reshape(A.shape)


def ratio_direct(A, rows, idx):
    """(sign, logabs) of det(A') / det(A) by refactoring both matrices (float64)."""
    A = _wide(A)
    s0, l0 = _slogdet(A)
    s1, l1 = _slogdet(apply_move(A, _wide(rows), idx))
    return s1 / np.where(s0 == 0, 1, s0), l1 - l0


def inverse_direct(A, rows, idx):
    """inv(A')^T (float64)."""
    return np.swapaxes(np.linalg.inv(apply_move(_wide(A), _wide(rows), idx)), -1, -2)


def ratio_woodbury(G, rows, idx):
    """(sign, logabs) of det(R), R[r][s] = U_r . G[idx_s] (float64)."""
    G, U = _wide(G), _wide(rows)
    I = np.asarray(idx)
    Gi = np.take_along_axis(G, I[..., :, None].repeat(G.shape[-1], -1), axis=-2)
    R = np.einsum("...ri,...si->...rs", U, Gi)
    return np.linalg.slogdet(R)


def update_woodbury(G, rows, idx):
    """G' = G - (V^T - E) R^-T G[idx, :] (float64)."""
    G, U = _wide(G), _wide(rows)
    I = np.asarray(idx)
    n, k = G.shape[-1], I.shape[-1]
    Gi = np.take_along_axis(G, I[..., :, None].repeat(n, -1), axis=-2)
    R = np.einsum("...ri,...si->...rs", U, Gi)
    H = np.linalg.solve(np.swapaxes(R, -1, -2), Gi)          # R^-T G[idx, :]
    V = np.einsum("...ri,...ji->...rj", U, G)                 # V = U A^-1
    E = np.zeros(V.shape, dtype=V.dtype)
    np.put_along_axis(E, I[..., :, None], 1.0, axis=-1)
    return G - np.einsum("...rj,...rc->...jc", V - E, H)
