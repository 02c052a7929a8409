"""numpy / scipy restatement of the reference's generic path (TEST INFRASTRUCTURE ONLY).

Each function restates one function of ChenAo-Phys/fermix (paths relative to that
project) with the same arithmetic conventions:

* LU: ``lax.linalg.lu`` on CPU is LAPACK ``?getrf`` (``src/fermix/_fallback.py:59``,
  ``:78``); here ``scipy.linalg.lapack.?getrf`` per matrix, i.e. the same LAPACK routine
  (OpenBLAS build, pinned by the scipy wheel in this image).
* (sign, logabs) from the LU with explicit pairwise trees (``_fallback.py:19-55``).
* the masked batched Parlett-Reid (``_fallback.py:266-300``) and its factor-keeping
  variant with the pf adjugate / inverse formulas (``_fallback.py:101-263``).
* the derivative rules of ``src/fermix/_diff.py`` (tangents ``:92-97``, permutation
  sign ``:160-176``, det from the LU pivots ``:184-202``, the singular-safe det adjugate
  ``:205-246``) and the closed forms of ``src/fermix/_poly.py``.

Gradients follow the reference's (JAX) convention: the arrays returned by the
``*_grad`` functions are ``jax.grad`` of ``sum(logabs)`` (slogdet / slogpf) or of
``sum(Re value)`` (det / pf) -- for complex inputs the holomorphic derivative, without
conjugation (``tests/test_fermix.py:329-358`` of the reference).
"""

import numpy as np
import scipy.linalg.lapack as _lapack

DET_POLY_MAX = 4  # src/fermix/_poly.py:6
PF_POLY_MAX = 6  # src/fermix/_poly.py:7

_GETRF = {
    np.dtype(np.float32): _lapack.sgetrf,
    np.dtype(np.float64): _lapack.dgetrf,
    np.dtype(np.complex64): _lapack.cgetrf,
    np.dtype(np.complex128): _lapack.zgetrf,
}
KINDS = tuple(_GETRF)


def real_dtype(dt):
    return np.finfo(np.dtype(dt)).dtype


def _check(a):
    """dtype / shape validation of ``api._prep`` (src/fermix/api.py:24-31)."""
    a = np.asarray(a)
    if a.dtype not in _GETRF:
        raise TypeError(f"fermix supports float32, float64, complex64 and complex128, got {a.dtype}")
    if a.ndim < 2 or a.shape[-1] != a.shape[-2]:
        raise ValueError(f"expected (..., n, n), got {a.shape}")
    return a


# ------------------------------------------------------------------ reductions
def _pairwise(x, op, fill):
    """Pairwise tree reduction of the last axis (src/fermix/_fallback.py:19-33)."""
    x = np.asarray(x)
    n = x.shape[-1]
    if n == 0:
        return np.full(x.shape[:-1], fill, x.dtype)
    while n > 1:
        h = (n + 1) // 2
        pad = 2 * h - n
        if pad:
            x = np.concatenate([x, np.full(x.shape[:-1] + (pad,), fill, x.dtype)], -1)
        x = op(x[..., :h], x[..., h:])
        n = h
    return x[..., 0]


def _unit(x):
    """x / |x| with 0 -> 0 (jnp.sign of a complex number)."""
    x = np.asarray(x)
    if np.iscomplexobj(x):
        m = np.abs(x)
        return np.where(m == 0, 0, x / np.where(m == 0, 1, m)).astype(x.dtype)
    return np.sign(x)


# ------------------------------------------------------------------ LU path
def lapack_lu(A):
    """Batched LAPACK getrf: (lu, piv) with 0-based LAPACK pivots (P A = L U)."""
    A = np.asarray(A)
    getrf = _GETRF[A.dtype]
    lu = np.empty_like(A)
    piv = np.empty(A.shape[:-1], np.int32)
    for b in range(A.shape[0]):
        lu[b], piv[b], _ = getrf(A[b])
    return lu, piv


def _perm_from_piv(piv):
    """The row permutation of LAPACK's interchange sequence: A[perm] = L U."""
    B, n = piv.shape
    perm = np.broadcast_to(np.arange(n), (B, n)).copy()
    rows = np.arange(B)
    for j in range(n):
        p = piv[:, j]
        a, b = perm[rows, j].copy(), perm[rows, p].copy()
        perm[rows, j], perm[rows, p] = b, a
    return perm


def _slog_from_lu(lu, piv):
    """(sign, logabs) of P L U from diag(U) and the LAPACK pivots
    (src/fermix/_fallback.py:36-55)."""
    d = np.diagonal(lu, axis1=-2, axis2=-1)
    iota = np.arange(lu.shape[-1], dtype=piv.dtype)
    swaps = np.sum(piv != iota, axis=-1)
    zero = np.any(d == 0, axis=-1)
    dsafe = np.where(d == 0, 1, d).astype(lu.dtype)
    if np.iscomplexobj(lu):
        sign = _pairwise(dsafe / np.abs(dsafe), np.multiply, 1).astype(lu.dtype)
        sign = np.where(swaps % 2 == 1, -sign, sign)
    else:
        parity = swaps + np.sum(d < 0, axis=-1)
        sign = np.where(parity % 2 == 1, -1.0, 1.0).astype(lu.dtype)
    sign = np.where(zero, 0, sign).astype(lu.dtype)
    logsum = _pairwise(np.log(np.abs(dsafe)), np.add, 0)
    logabs = np.where(zero, -np.inf, logsum)
    return sign, logabs.astype(real_dtype(lu.dtype))


def slogdet_generic(A):
    """src/fermix/_fallback.py:58-60."""
    lu, piv = lapack_lu(A)
    return _slog_from_lu(lu, piv)


def _tri_solve_lower_unit(L, X):
    import scipy.linalg as sl

    return np.stack([sl.solve_triangular(L[b], X[b], lower=True, unit_diagonal=True, check_finite=False) for b in range(L.shape[0])])


def _tri_solve_upper(U, X):
    import scipy.linalg as sl

    with np.errstate(all="ignore"):
        return np.stack([sl.solve_triangular(U[b], X[b], lower=False, check_finite=False) for b in range(U.shape[0])])


def lu_parts(A, zero_singular=True):
    """(sign, logabs, invT, LU, g0, zero) (src/fermix/_fallback.py:63-97, N == n):
    A[g0] = L U, invT = (U~^-1 L^-1 P)^T with zero pivots replaced by 1, zeroed where
    non-finite and, with zero_singular, where a pivot is exactly zero."""
    A = np.asarray(A)
    n = A.shape[-1]
    dt = A.dtype
    lu, piv = lapack_lu(A)
    perm = _perm_from_piv(piv)
    sign, logabs = _slog_from_lu(lu, piv)
    zero = np.diagonal(lu, axis1=-2, axis2=-1) == 0
    Ut = np.triu(lu) + zero.astype(dt)[..., None] * np.eye(n, dtype=dt)
    X = np.zeros_like(A)
    np.put_along_axis(X, perm[:, :, None], 1, axis=2)  # (P I)[c, :] = e_perm[c]
    X = _tri_solve_lower_unit(lu, X)
    X = _tri_solve_upper(Ut, X)
    bad = ~np.all(np.isfinite(X), axis=(-1, -2))
    if zero_singular:
        bad = bad | np.any(zero, axis=-1)
    invT = np.where(bad[:, None, None], 0, np.swapaxes(X, -1, -2)).astype(dt)
    return sign, logabs, invT, lu, perm, zero


# ------------------------------------------------------------------ det helpers
def _perm_sign(g0, dt):
    """sgn of the row permutation g0 (src/fermix/_diff.py:160-176): (-1)^(N - cycles)."""
    B, N = g0.shape
    idx = np.broadcast_to(np.arange(N), (B, N))
    lab, p = idx.copy(), g0.copy()
    for _ in range(max(N - 1, 0).bit_length()):
        lab = np.minimum(lab, np.take_along_axis(lab, p, axis=1))
        p = np.take_along_axis(p, p, axis=1)
    ncyc = np.sum(lab == idx, axis=1)
    return (1.0 - 2.0 * ((N - ncyc) % 2)).astype(dt)


def _lu_det(d, g0, dt):
    """sgn(P) prod(d) of a packed LU (src/fermix/_diff.py:184-202)."""
    dsafe = np.where(d == 0, 1, d).astype(dt)
    logsum = _pairwise(np.log(np.abs(dsafe)), np.add, 0)
    phase = _pairwise(_unit(dsafe), np.multiply, 1)
    det = _perm_sign(g0, dt) * phase * np.exp(logsum)
    return np.where(np.any(d == 0, axis=1), 0, det).astype(dt)


def _det_gradT(invT, LU, g0, zero, n):
    """adj(A)^T from the LU parts, exact for up to two zero pivots
    (src/fermix/_diff.py:205-246)."""
    B, N = LU.shape[:2]
    dt = LU.dtype
    m = np.sum(zero, axis=1)
    d = np.diagonal(LU, axis1=1, axis2=2)
    det = _lu_det(d, g0, dt)
    G = det[:, None, None] * invT
    if not np.any(m >= 1):
        return G
    idx = np.arange(N)
    k1 = np.minimum(np.min(np.where(zero, idx, N), axis=1), N - 1)
    k2 = np.maximum(np.max(np.where(zero, idx, -1), axis=1), 0)
    dsafe = np.where(zero, 1.0, d).astype(dt)
    logsum = np.sum(np.log(np.abs(dsafe)), axis=1)
    dK = np.prod(_unit(dsafe), axis=1) * np.exp(logsum)
    Ut = np.triu(LU) + zero.astype(dt)[:, :, None] * np.eye(N, dtype=dt)
    E = np.zeros((B, N, 2), dt)
    E[np.arange(B), k1, 0] = 1
    E[np.arange(B), k2, 1] = 1
    UE = _tri_solve_upper(Ut, E)
    u1 = UE[:, :n, 0]
    c = UE[np.arange(B), k1, 1]
    s = _perm_sign(g0, dt) * dK * np.where(m >= 2, c, 1.0)
    s = np.where(m >= 3, 0.0, s)
    col = invT[np.arange(B), :, k2]
    Gs = s[:, None, None] * col[:, :, None] * u1[:, None, :]
    return np.where((m >= 1)[:, None, None], Gs, G).astype(dt)


# ------------------------------------------------------------------ closed forms
def det_poly(A):
    """src/fermix/_poly.py:10-37."""
    n = A.shape[-1]
    if n == 0:
        return np.ones(A.shape[:-2], A.dtype)
    a = lambda i, j: A[..., i, j]
    m = lambda r, s, i, j: a(r, i) * a(s, j) - a(r, j) * a(s, i)
    if n == 1:
        return a(0, 0)
    if n == 2:
        return m(0, 1, 0, 1)
    if n == 3:
        return a(0, 0) * m(1, 2, 1, 2) - a(0, 1) * m(1, 2, 0, 2) + a(0, 2) * m(1, 2, 0, 1)
    if n == 4:
        p01 = m(0, 1, 0, 1) * m(2, 3, 2, 3)
        p02 = m(0, 1, 0, 2) * m(2, 3, 1, 3)
        p03 = m(0, 1, 0, 3) * m(2, 3, 1, 2)
        p12 = m(0, 1, 1, 2) * m(2, 3, 0, 3)
        p13 = m(0, 1, 1, 3) * m(2, 3, 0, 2)
        p23 = m(0, 1, 2, 3) * m(2, 3, 0, 1)
        return p01 - p02 + p03 + p12 - p13 + p23
    raise ValueError(n)


def det_poly_grad(A):
    """d det / dA = adj(A)^T for n <= 4: the cofactors (the derivative of the polynomial;
    the reference obtains it by autodiff of _det_poly, src/fermix/_diff.py:114-117)."""
    n = A.shape[-1]
    G = np.zeros_like(A)
    if n == 1:
        G[..., 0, 0] = 1
        return G
    for i in range(n):
        for j in range(n):
            M = np.delete(np.delete(A, i, -2), j, -1)
            G[..., i, j] = (-1) ** (i + j) * det_poly(M)
    return G


def pf_poly(S):
    """src/fermix/_poly.py:40-60."""
    n = S.shape[-1]
    if n == 0:
        return np.ones(S.shape[:-2], S.dtype)
    s = lambda i, j: S[..., i, j]
    pf4 = lambda a, b, c, d: s(a, b) * s(c, d) - s(a, c) * s(b, d) + s(a, d) * s(b, c)
    if n == 2:
        return s(0, 1)
    if n == 4:
        return pf4(0, 1, 2, 3)
    if n == 6:
        t1 = s(0, 1) * pf4(2, 3, 4, 5)
        t2 = s(0, 2) * pf4(1, 3, 4, 5)
        t3 = s(0, 3) * pf4(1, 2, 4, 5)
        t4 = s(0, 4) * pf4(1, 2, 3, 5)
        t5 = s(0, 5) * pf4(1, 2, 3, 4)
        return t1 - t2 + t3 - t4 + t5
    raise ValueError(n)


def pf_poly_grad_upper(S):
    """d pf / d s_ij on the strict upper triangle (zero elsewhere): the minor Pfaffian
    (-1)^(i+j+1) pf(S without rows/cols i, j) -- the vjp of _pf_poly
    (src/fermix/_diff.py:143-147, :322-324)."""
    n = S.shape[-1]
    G = np.zeros_like(S)
    for i in range(n):
        for j in range(i + 1, n):
            keep = [k for k in range(n) if k not in (i, j)]
            sub = S[..., keep, :][..., :, keep]
            G[..., i, j] = (-1) ** (i + j + 1) * pf_poly(sub)
    return G


# ------------------------------------------------------------------ Parlett-Reid
def _pr_step_pivot(A, c, idx):
    col = A[:, :, c]
    cand = np.where(idx > c, np.abs(col), -1.0)
    kp = np.argmax(cand, axis=1)  # first occurrence
    moved = np.where(idx == kp[:, None], c + 1, idx)
    p = np.where(idx == c + 1, kp[:, None], moved)
    return kp, p


def slogpf_generic(S):
    """Masked batched Parlett-Reid (src/fermix/_fallback.py:266-300)."""
    sign, log, *_ = _parlett_reid(S, keep=False)
    return sign, log


def _parlett_reid(S, keep):
    """The pair steps of src/fermix/_fallback.py:206-236 (keep=True also keeps L, the
    permutation and the parity, as _pf_parts_generic does)."""
    S = np.asarray(S)
    B, n, _ = S.shape
    dt = S.dtype
    idx = np.arange(n)[None, :]
    A = S.copy()
    L = np.zeros_like(S) if keep else None
    perm = np.broadcast_to(np.arange(n), (B, n)).copy()
    sign = np.ones(B, dt)
    log = np.zeros(B, real_dtype(dt))
    par = np.zeros(B, bool)
    rows = np.arange(B)[:, None]
    for k in range(n // 2):
        c = 2 * k
        kp, p = _pr_step_pivot(A, c, idx)
        A = A[rows, p, :]
        A = A[rows[:, :, None], np.arange(n)[None, :, None], p[:, None, :]]
        if keep:
            L = L[rows, p, :]
            perm = np.take_along_axis(perm, p, axis=1)
        swapped = kp != c + 1
        sign = np.where(swapped, -sign, sign)
        colc = A[:, :, c]
        colc1 = A[:, :, c + 1]
        d = colc1[:, c]
        with np.errstate(all="ignore"):
            inv = np.where(d == 0, 0.0, 1.0 / np.where(d == 0, 1.0, d)).astype(dt)
        mask = (idx > c + 1).astype(dt)
        tau = (-colc * inv[:, None] * mask).astype(dt)
        w = (colc1 * mask).astype(dt)
        A = (A + tau[:, :, None] * w[:, None, :] - w[:, :, None] * tau[:, None, :]).astype(dt)
        if keep:
            L[:, :, c] = w
            L[:, :, c + 1] = tau
        with np.errstate(divide="ignore"):
            sign = (sign * _unit(d)).astype(dt)
            log = (log + np.log(np.abs(d))).astype(real_dtype(dt))
        par = par ^ swapped
    return sign, log, A, L, perm, par


def _pivot_index(d, n):
    """src/fermix/_fallback.py:101-108."""
    a = np.abs(d).astype(np.float64)
    h = d.shape[1]
    if n // 2 < h:
        a[:, n // 2 :] = np.inf
    return np.argmin(a, axis=1)


def _pair_scale(d, K):
    """src/fermix/_fallback.py:111-115."""
    isK = np.arange(d.shape[1])[None, :] == K[:, None]
    return np.where(isK | (d == 0), 1, d).astype(d.dtype)


def _pf_value(d, sgnP):
    """src/fermix/_fallback.py:118-123."""
    dsafe = np.where(d == 0, 1, d).astype(d.dtype)
    with np.errstate(over="ignore"):
        mag = np.exp(_pairwise(np.log(np.abs(dsafe)), np.add, 0))
        return (sgnP * _pairwise(_unit(d), np.multiply, 1) * mag).astype(d.dtype)


def _second_zero(d, K):
    """src/fermix/_fallback.py:126-139."""
    others = (d == 0) & (np.arange(d.shape[1])[None, :] != K[:, None])
    has2 = np.any(others, axis=1)
    first = np.argmax(others, axis=1)
    is2 = has2[:, None] & (np.arange(d.shape[1])[None, :] == first[:, None])
    return has2, is2


def _pf_adj_coeffs(d, sgnP, K, adjugate):
    """src/fermix/_fallback.py:157-172."""
    h = d.shape[1]
    isK = np.arange(h)[None, :] == K[:, None]
    dK = np.take_along_axis(d, K[:, None], axis=1)[:, 0]
    dsafe = np.where(d == 0, 1, d).astype(d.dtype)
    logD = _pairwise(np.where(isK, 0, np.log(np.abs(dsafe))), np.add, 0)
    phase = _pairwise(np.where(isK, 1, _unit(d)), np.multiply, 1)
    D = phase * np.exp(logD)
    if adjugate:
        return sgnP * D * dK, sgnP * D * (1 - dK), dK
    nz = dK != 0
    with np.errstate(all="ignore"):
        a2 = np.where(nz, (1 - dK) / np.where(nz, dK, 1), 0)
    return np.ones_like(dK), a2, dK


def _pf_adj_blocks(d, Y, R, sgnP, K, adjugate):
    """-(a1 R + a2 (w v^T - v w^T)) (src/fermix/_fallback.py:175-192)."""
    a1, a2, _ = _pf_adj_coeffs(d, sgnP, K, adjugate)
    B = d.shape[0]
    aK = 2 * K
    w = R[np.arange(B), :, aK]
    v = Y[np.arange(B), aK, :]
    outer = lambda x, y: x[:, :, None] * y[:, None, :]
    PT = a1[:, None, None] * R + a2[:, None, None] * (outer(w, v) - outer(v, w))
    return -PT


def pf_parts(S, adjugate):
    """(sign, logabs, G, pf) with G = pf S^-1 (adjugate) or S^-1 (zeroed for an exactly
    singular S or a non-finite result) (src/fermix/_fallback.py:195-263)."""
    S = np.asarray(S)
    B, n, _ = S.shape
    dt = S.dtype
    h = n // 2
    sign, log, T, L0, perm, par = _parlett_reid(S, keep=True)
    d = T[:, np.arange(0, n, 2), np.arange(1, n, 2)]  # T[2s, 2s+1]
    K = _pivot_index(d, n)
    sgnP = np.where(par, -1.0, 1.0).astype(dt)
    eye = np.broadcast_to(np.eye(n, dtype=dt), (B, n, n))
    iperm = np.argsort(perm, axis=1)

    def evaluate(dd):
        dt_ = _pair_scale(dd, K)
        scale = np.stack([1 / dt_, np.ones_like(dt_)], axis=2).reshape(B, n)
        Lt = L0 * scale[:, None, :] + np.eye(n, dtype=dt)
        Y = _tri_solve_lower_unit(Lt, eye)
        Yr = Y.reshape(B, h, 2, n)
        DY = np.stack([Yr[:, :, 1], -Yr[:, :, 0]], axis=2) / dt_[:, :, None, None]
        R = np.matmul(np.swapaxes(Y, 1, 2), DY.reshape(B, n, n))
        PT = _pf_adj_blocks(dd, Y, R, sgnP, K, adjugate)
        G = np.take_along_axis(PT, iperm[:, :, None], axis=1)
        return np.take_along_axis(G, iperm[:, None, :], axis=2)

    with np.errstate(all="ignore"):
        if adjugate:
            has2, is2 = _second_zero(d, K)
            G = evaluate(d)
            if np.any(has2):  # the lifted mean of _fallback.py:142-154
                lifted = 0.5 * (evaluate(np.where(is2, 1, d).astype(dt)) + evaluate(np.where(is2, -1, d).astype(dt)))
                G = np.where(has2[:, None, None], lifted, G)
        else:
            G = evaluate(d)
            dK = np.take_along_axis(d, K[:, None], axis=1)[:, 0]
            bad = (dK == 0) | ~np.all(np.isfinite(G), axis=(1, 2))
            G = np.where(bad[:, None, None], 0, G)
    return sign, log, G.astype(dt), _pf_value(d, sgnP)


# ------------------------------------------------------------------ public surface
def _flat(a):
    batch = a.shape[:-2]
    n = a.shape[-1]
    return a.reshape((int(np.prod(batch)), n, n)), batch, n


def _sign_log(x):
    with np.errstate(divide="ignore"):
        return _unit(x).astype(x.dtype), np.log(np.abs(x)).astype(real_dtype(x.dtype))


def slogdet(a):
    """(sign, logabs) as ``fermix.slogdet`` (src/fermix/api.py:148-174, _diff.py:42-49)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n <= DET_POLY_MAX:
        s, l = _sign_log(det_poly(A))
    else:
        s, l = slogdet_generic(A)
    return s.reshape(batch), l.reshape(batch)


def _skew(A):
    return ((A - np.swapaxes(A, -1, -2)) * 0.5).astype(A.dtype)


def slogpf(a, skew_symmetrize=True):
    """(sign, logabs) as ``fermix.slogpf`` (src/fermix/api.py:177-193, _diff.py:52-59)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n % 2 == 1:
        return np.zeros(batch, a.dtype), np.full(batch, -np.inf, real_dtype(a.dtype))
    if skew_symmetrize:
        A = _skew(A)
    if n <= PF_POLY_MAX:
        s, l = _sign_log(pf_poly(A))
    else:
        s, l = slogpf_generic(A)
    return s.reshape(batch), l.reshape(batch)


def det(a):
    """``fermix.det`` (src/fermix/_diff.py:278-285)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n <= DET_POLY_MAX:
        return det_poly(A).reshape(batch)
    s, l = slogdet_generic(A)
    return (s * np.exp(l)).astype(a.dtype).reshape(batch)


def pf(a, skew_symmetrize=True):
    """``fermix.pf`` (src/fermix/_diff.py:311-316, api.py:130-145)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n % 2 == 1:
        return np.zeros(batch, a.dtype)
    if skew_symmetrize:
        A = _skew(A)
    if n <= PF_POLY_MAX:
        return pf_poly(A).reshape(batch)
    s, l = slogpf_generic(A)
    return (s * np.exp(l)).astype(a.dtype).reshape(batch)


def _safe_recip(x):
    """src/fermix/_poly.py:67-71."""
    nz = x != 0
    with np.errstate(all="ignore"):
        return np.where(nz, 1.0 / np.where(nz, x, 1.0), 0.0).astype(x.dtype)


def slogdet_grad(a):
    """jax.grad of sum(logabs): A^-T (holomorphic), zero for an exactly singular A
    (src/fermix/_diff.py:111-124)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n <= DET_POLY_MAX:
        G = det_poly_grad(A) * _safe_recip(det_poly(A))[:, None, None]
    else:
        G = lu_parts(A, True)[2]
    return G.astype(a.dtype).reshape(a.shape)


def slogpf_grad(a, skew_symmetrize=True):
    """jax.grad of sum(logabs) w.r.t. the input: S^-T / 2 (S the skew-symmetrised input),
    zero for an exactly singular S (src/fermix/_diff.py:139-154)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n % 2 == 1:
        return np.zeros_like(a)
    S = _skew(A) if skew_symmetrize else A
    if n <= PF_POLY_MAX:
        Gu = pf_poly_grad_upper(S)
        G = (Gu - np.swapaxes(Gu, -1, -2)) * _safe_recip(pf_poly(S))[:, None, None]
        G = 0.5 * G  # d logabs = 0.5 sum(G dS) for skew dS
    else:
        Sinv = pf_parts(S, False)[2]
        G = -0.5 * Sinv
    if skew_symmetrize:
        G = 0.5 * (G - np.swapaxes(G, -1, -2))
    return G.astype(a.dtype).reshape(a.shape)


def det_grad(a):
    """jax.grad of sum(Re det): adj(A)^T, finite for singular A (src/fermix/_diff.py:287-300)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n <= DET_POLY_MAX:
        G = det_poly_grad(A)
    else:
        sign, logabs, invT, LU, g0, zero = lu_parts(A, False)
        G = _det_gradT(invT, LU, g0, zero, n)
    return G.astype(a.dtype).reshape(a.shape)


def pf_grad(a, skew_symmetrize=True):
    """jax.grad of sum(Re pf): pf S^-T / 2 continued to singular S
    (src/fermix/_diff.py:318-331)."""
    a = _check(a)
    A, batch, n = _flat(a)
    if n % 2 == 1:
        return np.zeros_like(a)
    S = _skew(A) if skew_symmetrize else A
    if n <= PF_POLY_MAX:
        Gu = pf_poly_grad_upper(S)
        G = 0.5 * (Gu - np.swapaxes(Gu, -1, -2))
    else:
        adj = pf_parts(S, True)[2]
        G = -0.5 * adj
    if skew_symmetrize:
        G = 0.5 * (G - np.swapaxes(G, -1, -2))
    return G.astype(a.dtype).reshape(a.shape)
