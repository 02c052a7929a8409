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

The Pfaffian one-index moves (row and column i of a skew S replaced by u and -u) follow the
same pattern: ``pf_ratio_direct`` / ``pf_grad_direct`` refactor S' with the Parlett-Reid
restatement (``oracle.fallback.slogpf``, ``src/fermix/_fallback.py:266-300``) and take
S'^-T / 2; ``pf_ratio_woodbury`` / ``pf_update_woodbury`` use G = S^-T / 2 alone:
pf(S') / pf(S) = 2 G_i . u and G' = G + (y g_i^T - g_i y^T) / rho, y = e_i - 2 G u.

The tests pin the second route against the first, then the CUDA path against both.
"""

import numpy as np

from .fallback import slogdet as _slogdet
from .fallback import slogpf as _slogpf


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


def pf_apply_move(S, row, idx):
    """S' = S with row idx[b] replaced by row[b] and column idx[b] by -row[b] (diagonal 0)."""
    S = np.array(S, copy=True)
    B = S.reshape((-1,) + S.shape[-2:])
    U = np.asarray(row).reshape(B.shape[0], -1)
    I = np.asarray(idx).reshape(-1)
    for b in range(B.shape[0]):
        u = U[b].copy()
        u[I[b]] = 0
        B[b, I[b], :] = u
        B[b, :, I[b]] = -u
    return B.reshape(S.shape)


def pf_ratio_direct(S, row, idx):
    """(sign, logabs) of pf(S') / pf(S) by refactoring both (float64 / complex128)."""
    S = _wide(S)
    s0, l0 = _slogpf(S)
    s1, l1 = _slogpf(pf_apply_move(S, _wide(row), idx))
    return s1 / np.where(s0 == 0, 1, s0), l1 - l0


def pf_grad_direct(S, row, idx):
    """S'^-T / 2 (float64 / complex128)."""
    return 0.5 * np.swapaxes(np.linalg.inv(pf_apply_move(_wide(S), _wide(row), idx)), -1, -2)


def pf_ratio_woodbury(G, row, idx):
    """rho = 2 G_i . u (u_i left out)."""
    G, U = _wide(G), _wide(row).copy()
    I = np.asarray(idx)
    np.put_along_axis(U, I[..., None], 0, axis=-1)
    gi = np.take_along_axis(G, I[..., None, None].repeat(G.shape[-1], -1), axis=-2)[..., 0, :]
    return 2 * np.sum(gi * U, axis=-1)


def pf_update_woodbury(G, row, idx):
    """G' = G + (y g_i^T - g_i y^T) / rho, y = e_i - 2 G u."""
    G, U = _wide(G), _wide(row).copy()
    I = np.asarray(idx)
    n = G.shape[-1]
    np.put_along_axis(U, I[..., None], 0, axis=-1)
    gi = np.take_along_axis(G, I[..., None, None].repeat(n, -1), axis=-2)[..., 0, :]
    rho = 2 * np.sum(gi * U, axis=-1)
    y = -2 * np.einsum("...jc,...c->...j", G, U)
    np.put_along_axis(y, I[..., None], np.take_along_axis(y, I[..., None], -1) + 1, axis=-1)
    upd = np.einsum("...j,...c->...jc", y, gi) - np.einsum("...j,...c->...jc", gi, y)
    return G + upd / rho[..., None, None]


# ---------------------------------------------------------------- k-index Pfaffian moves
# A k-index move replaces rows idx[r] of the skew S by rows[r] and columns idx[r] by
# -rows[r], applied in order r = 0 .. k-1 (so on the idx x idx block the later row wins;
# rows[r][idx[r]] is ignored): it is the composition of k one-index moves.

def pf_apply_move_k(S, rows, idx):
    """S' of a k-index move (float64 / complex128), the one-index moves applied in order."""
    S = _wide(S).copy()
    B = S.reshape((-1,) + S.shape[-2:])
    U = _wide(rows).reshape((B.shape[0],) + np.asarray(rows).shape[-2:])
    I = np.asarray(idx).reshape(B.shape[0], -1)
    for r in range(I.shape[1]):
        B[:] = pf_apply_move(B, U[:, r], I[:, r])
    return B.reshape(S.shape)


def pf_ratio_direct_k(S, rows, idx):
    """(sign, logabs) of pf(S') / pf(S) by refactoring both (float64 / complex128)."""
    S = _wide(S)
    s0, l0 = _slogpf(S)
    s1, l1 = _slogpf(pf_apply_move_k(S, rows, idx))
    return s1 / np.where(s0 == 0, 1, s0), l1 - l0


def pf_grad_direct_k(S, rows, idx):
    """S'^-T / 2 of a k-index move (float64 / complex128)."""
    return 0.5 * np.swapaxes(np.linalg.inv(pf_apply_move_k(S, rows, idx)), -1, -2)


def pf_factors_k(G, rows, idx):
    """The k-index move from G = S^-T / 2 alone (float64 / complex128): with G_t the
    gradient after t one-index moves, g_t = row idx[t] of G_t, rho_t = 2 g_t . u_t and
    y_t = e_idx[t] - 2 G_t u_t, so that G_{t+1} = G_t + (y_t g_t^T - g_t y_t^T) / rho_t.
    Every G_t u and every row of G_t follow from V = G U^T (one pass over G) and the rows
    idx of G by the rank-2 corrections, O(n k^2). Returns (rho[B, k], g[B, k, n],
    y[B, k, n]); the ratio is prod(rho) and G' = G + sum_t (y_t g_t^T - g_t y_t^T) / rho_t."""
    G = _wide(G)
    Bsh = G.shape[:-2]
    n = G.shape[-1]
    Gf = G.reshape(-1, n, n)
    U = _wide(rows).reshape(Gf.shape[0], -1, n).copy()
    I = np.asarray(idx).reshape(Gf.shape[0], -1)
    k = I.shape[1]
    for b in range(Gf.shape[0]):
        for t in range(k):
            U[b, t, I[b, t]] = 0  # u_t[idx_t] is ignored
    V = np.einsum("bjc,btc->btj", Gf, U)  # V[t] = G u_t
    rho = np.zeros((Gf.shape[0], k), dtype=G.dtype)
    gs = np.zeros((Gf.shape[0], k, n), dtype=G.dtype)
    ys = np.zeros((Gf.shape[0], k, n), dtype=G.dtype)
    for b in range(Gf.shape[0]):
        for t in range(k):
            i = I[b, t]
            g = Gf[b, i].copy()          # row i of G_t
            w = V[b, t].copy()           # G_t u_t
            for q in range(t):
                yq, gq, rq = ys[b, q], gs[b, q], rho[b, q]
                g += (yq[i] * gq - gq[i] * yq) / rq
                w += (yq * (gq @ U[b, t]) - gq * (yq @ U[b, t])) / rq
            rho[b, t] = 2 * (g @ U[b, t])
            y = -2 * w
            y[i] += 1
            gs[b, t], ys[b, t] = g, y
    return rho.reshape(Bsh + (k,)), gs.reshape(Bsh + (k, n)), ys.reshape(Bsh + (k, n))


def pf_ratio_woodbury_k(G, rows, idx):
    rho, _, _ = pf_factors_k(G, rows, idx)
    return np.prod(rho, axis=-1)


def pf_update_woodbury_k(G, rows, idx):
    rho, g, y = pf_factors_k(G, rows, idx)
    G = _wide(G)
    upd = np.einsum("...tj,...tc->...jc", y / rho[..., None], g) - np.einsum("...tj,...tc->...jc", g / rho[..., None], y)
    return G + upd
