"""Golden fixtures for the slogdet / slogpf / det / pf path (TEST INFRASTRUCTURE).

    python tests/golden/make_golden.py      # rewrites tests/golden/golden.npz

Each case stores seeded inputs (generated as in the reference's test suite,
ChenAo-Phys/fermix tests/test_fermix.py:35-50, :459-545) together with answers that do
not come from this repository's code: numpy float64 / complex128 LAPACK
(np.linalg.slogdet / det / inv) and the reference test suite's own 64-bit oracles
(pf_ref64, adjT64, pf_gradT64, restated in oracle/refs64.py), plus closed-form known
answers. check_case() compares any implementation exposing the oracle's API (the numpy
oracle, or the CUDA path through the adapter in tests/test_golden_gpu.py) against them
with the reference's tolerances.
"""

import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle.refs64 import (  # noqa: E402
    adjT64,
    pf64,
    pf_gradT64,
    pf_ref64,
    randn,
    ref64,
    shifted,
    skew,
)

PATH = os.path.join(HERE, "golden.npz")
DT = {"f32": np.float32, "f64": np.float64, "c64": np.complex64, "c128": np.complex128}


def _tol(dt, t32, t64):
    return t32 if np.finfo(dt).bits == 32 else t64


def _cases():
    """name -> (kind, inputs dict, expected dict); deterministic."""
    out = {}
    for key, dt in DT.items():
        g = np.random.default_rng(1234)
        A = randn((4, 13, 13), dt, g)
        s, l = np.linalg.slogdet(ref64(A))
        out[f"slogdet_{key}"] = ("slogdet", {"a": A}, {"sign": s, "logabs": l})
        A = randn((2, 40, 40), dt, g)
        A[0, 7] = 0.0  # zero row: exactly singular
        A[1, :, 11] = 0.0  # zero column
        out[f"slogdet_singular_{key}"] = (
            "slogdet",
            {"a": A},
            {"sign": np.zeros(2), "logabs": np.full(2, -np.inf)},
        )
        S = skew(randn((4, 14, 14), dt, g))
        ref = [pf_ref64(S[i]) for i in range(4)]
        out[f"slogpf_{key}"] = (
            "slogpf",
            {"a": S},
            {"sign": np.array([r[0] for r in ref]), "logabs": np.array([r[1] for r in ref])},
        )
        A = shifted((3, 12, 12), dt, 3, g)
        out[f"slogdet_grad_{key}"] = (
            "slogdet_grad",
            {"a": A},
            {"grad": np.swapaxes(np.linalg.inv(ref64(A)), -1, -2)},
        )
        A = randn((3, 12, 12), dt, g)
        Sh = 0.5 * skew(ref64(A))
        out[f"slogpf_grad_{key}"] = (
            "slogpf_grad",
            {"a": A},
            {"grad": 0.5 * np.swapaxes(np.linalg.inv(Sh), -1, -2)},
        )
        A = shifted((4, 8, 8), dt, 2, g)
        A[0, :, 1] = 0.0
        A[1, 2] = 0.0
        A[2, :, 0] = 0.0
        A[2, :, 1] = 0.0
        out[f"det_grad_singular_{key}"] = (
            "det_grad",
            {"a": A},
            {"grad": np.stack([adjT64(x) for x in ref64(A)])},
        )
        S = skew(randn((3, 8, 8), dt, g))
        S[0, 3, :] = 0.0
        S[0, :, 3] = 0.0
        S[1, 1, :] = 0.0
        S[1, :, 1] = 0.0
        S[1, 5, :] = 0.0
        S[1, :, 5] = 0.0
        out[f"pf_grad_singular_{key}"] = (
            "pf_grad",
            {"a": S},
            {"grad": np.stack([pf_gradT64(x) for x in ref64(S)])},
        )
        S = skew(randn((3, 10, 10), dt, g))
        out[f"pf_{key}"] = ("pf", {"a": S}, {"value": np.array([pf64(x) for x in ref64(S)])})
        A = randn((3, 9, 9), dt, g)
        out[f"det_{key}"] = ("det", {"a": A}, {"value": np.linalg.det(ref64(A))})
    # closed forms: det(diag(1..n)) = n!, a permutation matrix has det = its sign, the
    # Pfaffian of the direct sum of [[0, c_k], [-c_k, 0]] is prod c_k
    n = 10
    D = np.diag(np.arange(1, n + 1, dtype=np.float64))[None]
    out["known_det_diag"] = ("slogdet", {"a": D}, {"sign": np.array([1.0]), "logabs": np.array([math.lgamma(n + 1)])})
    P = np.eye(7)[[2, 0, 1, 4, 3, 6, 5]][None]  # cycles (0 2 1)(3 4)(5 6): sign +1 * -1 * -1
    out["known_det_perm"] = ("slogdet", {"a": P}, {"sign": np.array([1.0]), "logabs": np.array([0.0])})
    c = np.array([2.0, -0.5, 3.0, 1.5, -4.0])
    J = np.zeros((1, 10, 10))
    for k, ck in enumerate(c):
        J[0, 2 * k, 2 * k + 1], J[0, 2 * k + 1, 2 * k] = ck, -ck
    out["known_pf_blocks"] = (
        "slogpf",
        {"a": J},
        {"sign": np.array([np.sign(np.prod(c))]), "logabs": np.array([np.sum(np.log(np.abs(c)))])},
    )
    return out


CASES = tuple(_cases().keys())


def write():
    arrays = {}
    for name, (kind, ins, exp) in _cases().items():
        for k, v in ins.items():
            arrays[f"{name}/in/{k}"] = v
        for k, v in exp.items():
            arrays[f"{name}/out/{k}"] = np.asarray(v)
        arrays[f"{name}/kind"] = np.array(kind)
    np.savez_compressed(PATH, **arrays)
    return PATH


def check_case(name, z, F):
    """Compare implementation F (oracle API: slogdet, slogpf, det, pf, slogdet_grad,
    slogpf_grad, det_grad, pf_grad; grads in the reference's JAX convention) with the
    stored answers of case `name` from the loaded npz `z`."""
    kind = str(z[f"{name}/kind"])
    a = z[f"{name}/in/a"]
    dt = a.dtype
    n = a.shape[-1]
    if kind in ("slogdet", "slogpf"):
        s, l = (F.slogdet(a) if kind == "slogdet" else F.slogpf(a, skew_symmetrize=False))
        s, l = np.asarray(s), np.asarray(l)
        es, el = z[f"{name}/out/sign"], z[f"{name}/out/logabs"]
        lt = _tol(dt, 2e-3, 1e-10) * max(1.0, n / 64)
        fin = np.isfinite(el)
        assert np.all(np.isneginf(l[~fin])) and np.all(s[~fin] == 0), (name, s, l)
        if np.iscomplexobj(s):
            assert np.max(np.abs(s[fin] - es[fin]), initial=0) < lt, (name, s, es)
        else:
            assert np.array_equal(s[fin], es[fin].astype(s.dtype)), (name, s, es)
        assert np.max(np.abs(l[fin] - el[fin]), initial=0) < lt, (name, l, el)
        return
    rt = _tol(dt, 1e-4, 1e-10)
    if kind in ("det", "pf"):
        v = np.asarray(F.det(a) if kind == "det" else F.pf(a, skew_symmetrize=False))
        e = z[f"{name}/out/value"]
        assert np.allclose(v, e, rtol=rt, atol=rt / 10), (name, v, e)
        return
    if kind == "slogdet_grad":
        g = F.slogdet_grad(a)
    elif kind == "slogpf_grad":
        g = F.slogpf_grad(a)
    elif kind == "det_grad":
        g = F.det_grad(a)
    else:
        g = F.pf_grad(a, skew_symmetrize=False)
    g = np.asarray(g)
    e = z[f"{name}/out/grad"]
    scale = max(np.abs(e).max(), 1e-30)
    assert np.all(np.isfinite(g)), name
    assert np.max(np.abs(g - e)) < rt * scale * 10, (name, np.max(np.abs(g - e)) / scale)


if __name__ == "__main__":
    print(write())
