"""Extended-precision references for the large-n float64 / complex128 parity tests.

For each case a seeded numpy matrix (regenerated bit for bit by the tests from the same
seed: numpy's PCG64 stream is stable across machines) is factorised by LU with partial
pivoting in np.longdouble / np.clongdouble (x87 80-bit: a 64-bit mantissa, eps 5.4e-20),
and log|det| and the sign of det are written to longdouble.json with 20 significant
digits. For a skew-symmetric S, log|pf(S)| = log|det(S)| / 2. The float64 LAPACK error of
the same quantity is recorded beside it (`lapack_err`), which is the yardstick for the
1e-10 logabs tolerance at n = 4096.

    python tests/golden/make_longdouble.py [--quick]   # --quick: the n <= 1040 cases only

Runtime: a few minutes per n = 4096 case on one core (longdouble arithmetic is not
vectorised by BLAS).
"""

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "longdouble.json")

# (name, kind, n, seed): kind "det" = iid N(0, 1) float64; "skew" = C - C^T with C complex
# N(0, 1) (real and imaginary parts), complex128
CASES = [
    ("f64_det_n1040", "det", 1040, 1040),
    ("c128_skew_n1040", "skew", 1040, 1041),
    ("f64_det_n4096", "det", 4096, 4096),
    ("c128_skew_n4096", "skew", 4096, 4097),
]


def matrix(kind, n, seed):
    """The test matrix of a case (float64 or complex128), as the tests build it."""
    g = np.random.default_rng(seed)
    if kind == "det":
        return g.standard_normal((n, n))
    C = g.standard_normal((n, n)) + 1j * g.standard_normal((n, n))
    return C - C.T


def lu_logdet(M):
    """(sign, log|det|) of M by LU with partial pivoting in extended precision."""
    cx = np.iscomplexobj(M)
    A = M.astype(np.clongdouble if cx else np.longdouble)
    n = A.shape[0]
    logabs = np.longdouble(0)
    sign = np.clongdouble(1) if cx else np.longdouble(1)
    for k in range(n):
        col = np.abs(A[k:, k])
        p = k + int(np.argmax(col))
        if col[p - k] == 0:
            return 0, -np.inf
        if p != k:
            A[[k, p]] = A[[p, k]]
            sign = -sign
        d = A[k, k]
        ad = np.abs(d)
        logabs += np.log(ad)
        sign = sign * (d / ad)
        if k + 1 < n:
            l = A[k + 1:, k] / d
            A[k + 1:, k + 1:] -= np.outer(l, A[k, k + 1:])
    return sign, logabs


def main():
    quick = "--quick" in sys.argv
    res = json.load(open(OUT)) if os.path.exists(OUT) else {}
    for name, kind, n, seed in CASES:
        if quick and n > 1040:
            continue
        M = matrix(kind, n, seed)
        t0 = time.time()
        s, l = lu_logdet(M)
        s64, l64 = np.linalg.slogdet(M)
        half = 0.5 if kind == "skew" else 1.0
        res[name] = {
            "kind": kind, "n": n, "seed": seed,
            "det_sign_re": repr(float(np.real(s))), "det_sign_im": repr(float(np.imag(s))),
            "logabs": np.format_float_positional(np.longdouble(half) * l, precision=20, unique=False),
            "lapack_err": float(abs(half * (np.longdouble(l64) - l))),
            "seconds": round(time.time() - t0, 1),
        }
        print(name, res[name], flush=True)
        json.dump(res, open(OUT, "w"), indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
