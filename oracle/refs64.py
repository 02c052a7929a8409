"""64-bit reference oracles of the reference's own test suite (TEST INFRASTRUCTURE ONLY).

Restated from ChenAo-Phys/fermix ``tests/test_fermix.py``: the input generators
(``randn`` :35-41, ``shifted`` :44-46, ``skew`` :49-50, ``rank_deficient`` :484-492,
``skew_rank_deficient`` :535-545), the tolerances (:57-84) and the float64 /
complex128 oracles ``pf_ref64`` (:95-116), ``pf64`` (:119-121), ``adjT64`` (:124-132)
and ``pf_gradT64`` (:135-144). They pin both the numpy restatement in
``oracle.fallback`` and the CUDA path.
"""

import math

import numpy as np


def is_complex(dtype):
    return np.issubdtype(np.dtype(dtype), np.complexfloating)


def ref64(x):
    x = np.asarray(x)
    return x.astype(np.complex128 if is_complex(x.dtype) else np.float64)


def randn(shape, dtype, gen):
    z = gen.standard_normal(shape)
    if is_complex(dtype):
        z = z + 1j * gen.standard_normal(shape)
    return z.astype(dtype)


def shifted(shape, dtype, shift, gen):
    return (randn(shape, dtype, gen) + shift * np.eye(shape[-1])).astype(dtype)


def skew(A):
    return A - np.swapaxes(A, -1, -2)


def rank_deficient(shape, dtype, gen):
    A = randn(shape, np.complex128 if is_complex(dtype) else np.float64, gen)
    c = randn(shape[:-2] + (shape[-1] - 1,), A.dtype, gen)
    A[..., -1, :] = np.einsum("...i,...ij->...j", c, A[..., :-1, :])
    return A.astype(dtype)


def skew_rank_deficient(shape, dtype, gen):
    n = shape[-1]
    X = randn(shape[:-1] + (n - 2,), np.complex128 if is_complex(dtype) else np.float64, gen)
    J = np.kron(np.eye((n - 2) // 2), np.array([[0.0, 1.0], [-1.0, 0.0]]))
    S = (X @ J @ np.swapaxes(X, -1, -2)).astype(dtype)
    return S - np.swapaxes(S, -1, -2)


def relerr(x, ref):
    return float(np.max(np.abs(x - ref)) / max(np.max(np.abs(ref)), 1e-30))


def tol(dtype, t32, t64):
    return t32 if np.finfo(np.dtype(dtype)).bits == 32 else t64


def log_tol(dtype, n=1):
    return tol(dtype, 2e-3, 1e-10) * max(1.0, n / 64)


def rel_tol(dtype):
    return tol(dtype, 1e-4, 1e-10)


def assert_sign(s, ref, dtype, atol):
    s, ref = np.asarray(s), np.asarray(ref)
    if not is_complex(dtype):
        assert np.array_equal(s, ref), (s, ref)
        return
    assert np.max(np.abs(s - ref)) < atol
    nz = ref != 0
    assert np.all(s[~nz] == 0)
    assert np.all(np.abs(np.abs(s[nz]) - 1.0) < tol(dtype, 1e-5, 1e-12))


def pf_ref64(S):
    A = np.array(ref64(S))
    n = A.shape[0]
    sign, log = 1.0, 0.0
    for k in range(0, n - 1, 2):
        kp = k + 1 + np.argmax(np.abs(A[k + 1 :, k]))
        if kp != k + 1:
            A[[k + 1, kp], :] = A[[kp, k + 1], :]
            A[:, [k + 1, kp]] = A[:, [kp, k + 1]]
            sign = -sign
        d = A[k, k + 1]
        if d == 0.0:
            return 0.0, -np.inf
        sign *= d / abs(d)
        log += math.log(abs(d))
        if k + 2 < n:
            tau = -A[k + 2 :, k] / d
            w = A[k + 2 :, k + 1]
            A[k + 2 :, k + 2 :] += np.outer(tau, w) - np.outer(w, tau)
    return sign, log


def pf64(S):
    s, l = pf_ref64(S)
    return s * math.exp(l) if np.isfinite(l) else 0.0


def adjT64(A):
    n = A.shape[0]
    G = np.zeros((n, n), A.dtype)
    for i in range(n):
        for j in range(n):
            M = np.delete(np.delete(A, i, 0), j, 1)
            G[i, j] = (-1) ** (i + j) * np.linalg.det(M)
    return G


def pf_gradT64(S):
    n = S.shape[0]
    D = np.zeros((n, n), S.dtype)
    for i in range(n):
        for j in range(i + 1, n):
            keep = [k for k in range(n) if k not in (i, j)]
            D[i, j] = (-1) ** (i + j + 1) * pf64(S[np.ix_(keep, keep)])
    return 0.5 * (D - D.T)
