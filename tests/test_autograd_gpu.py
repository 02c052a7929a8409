"""One factorisation per differentiated call: under autograd the forward launches the
fused factorisation + gradient kernel once and keeps the derivative matrix; the backward
only scales it (the reference's rule: primal and inverse from one _parts call,
src/fermix/_diff.py:111-124). Primal and gradient equal the separate forward and gradient
launches bit for bit (real dtypes) or to rounding of the complex product (complex)."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx
from fermix_b200 import _lib
from tests.helpers import cuda, host

pytestmark = pytest.mark.gpu

ENTRIES = ["fermix_slogdet", "fermix_slogdet_grad", "fermix_slogpf", "fermix_slogpf_grad"]


@pytest.fixture
def calls(monkeypatch):
    L = _lib.lib()
    seen = []
    for name in ENTRIES:
        fn = getattr(L, name)

        def wrap(*args, _fn=fn, _name=name):
            seen.append(_name)
            return _fn(*args)

        monkeypatch.setattr(L, name, wrap)
    return seen


def _inputs(op, dtype, B, n, seed):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((B, n, n))
    if np.dtype(dtype).kind == "c":
        A = A + 1j * rng.standard_normal((B, n, n))
    if op == "slogpf":
        A = A - np.swapaxes(A, -1, -2)
    return A.astype(dtype)


@pytest.mark.parametrize("op", ["slogdet", "slogpf"])
@pytest.mark.parametrize("dtype,n", [(np.float32, 128), (np.float64, 64), (np.complex64, 32), (np.float32, 300)],
                         ids=["f32-n128", "f64-n64", "c64-n32", "f32-n300"])
def test_backward_is_one_launch_with_identical_bits(calls, op, dtype, n):
    X = _inputs(op, dtype, 16, n, 11)
    f = getattr(fx, op)
    parts = getattr(fx, op + "_parts")
    with torch.no_grad():
        s0, l0 = host(f(cuda(X)))
        _, _, d0 = host(parts(cuda(X)))
    calls.clear()
    x = cuda(X, requires_grad=True)
    s, l = f(x)
    l.sum().backward()
    torch.cuda.synchronize()
    assert calls == [f"fermix_{op}_grad"], calls
    assert np.array_equal(host(s), s0) and np.array_equal(host(l), l0)
    g = host(x.grad)
    if np.dtype(dtype).kind == "c":
        np.testing.assert_allclose(g, np.conj(d0), rtol=1e-5, atol=1e-6 * np.abs(d0).max())
    else:
        assert np.array_equal(g, d0)


@pytest.mark.parametrize("op", ["det", "pf"])
def test_value_backward_is_one_launch(calls, op):
    X = _inputs("slogpf" if op == "pf" else "slogdet", np.float64, 8, 20, 12)
    x = cuda(X, requires_grad=True)
    v = getattr(fx, op)(x)
    v.sum().backward()
    torch.cuda.synchronize()
    base = "slogpf" if op == "pf" else "slogdet"
    assert calls == [f"fermix_{base}_grad"], calls
    with torch.no_grad():
        v0, d0 = host(getattr(fx, op + "_parts")(cuda(X)))
    assert np.array_equal(host(v), v0) and np.array_equal(host(x.grad), d0)


def test_large_derivative_recomputes_in_backward(calls, monkeypatch):
    from fermix_b200 import api

    monkeypatch.setattr(api, "KEEP_GRAD_BYTES", 0)
    X = _inputs("slogdet", np.float32, 4, 64, 13)
    x = cuda(X, requires_grad=True)
    s, l = fx.slogdet(x)
    l.sum().backward()
    torch.cuda.synchronize()
    assert calls == ["fermix_slogdet", "fermix_slogdet_grad"], calls
    with torch.no_grad():
        _, _, d0 = host(fx.slogdet_parts(cuda(X)))
    assert np.array_equal(host(x.grad), d0)
