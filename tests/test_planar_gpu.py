"""Complex inputs as split real / imaginary planes (fermix_*_planar): equal bit for bit to
the interleaved entry points on the same values -- the blocked engines' direct plane
reads and writes (n > 256) and the chunked converting route (other sizes, adjugates)."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx

pytestmark = pytest.mark.gpu


def _data(dtype, B, n, seed, skew):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn((B, n, n), generator=g, device="cuda", dtype=dtype)
    if skew:
        a = (a - a.transpose(-1, -2)).contiguous()
    return a, a.real.contiguous(), a.imag.contiguous()


def _eq(x, y):
    assert x.shape == y.shape
    assert torch.equal(torch.nan_to_num(x), torch.nan_to_num(y)), (x - y).abs().max()


CASES = [(torch.complex64, 20, 5), (torch.complex128, 40, 3), (torch.complex64, 300, 3), (torch.complex128, 260, 2),
         (torch.complex64, 512, 2)]


@pytest.mark.parametrize("op", ["slogdet", "slogpf"])
@pytest.mark.parametrize("dtype,n,B", CASES, ids=[f"{str(c[0])[6:]}-n{c[1]}" for c in CASES])
def test_planar_equals_interleaved(op, dtype, n, B):
    a, re, im = _data(dtype, B, n, n, skew=False)
    f = getattr(fx, op)
    fp = getattr(fx, op + "_planar")
    parts = getattr(fx, op + "_parts")
    with torch.no_grad():
        s0, l0 = f(a)
        s1, l1 = fp(re, im)
        _eq(s1, s0)
        _eq(l1, l0)
        coef = torch.randn(B, device="cuda", dtype=dtype)
        s0, l0, g0 = parts(a, coef=coef)
        s1, l1, g_re, g_im = fp(re, im, grad=True, coef=coef)
        _eq(s1, s0)
        _eq(l1, l0)
        _eq(g_re, g0.real.contiguous())
        _eq(g_im, g0.imag.contiguous())


@pytest.mark.parametrize("op", ["det", "pf"])
def test_planar_adjugate_and_prec(op):
    a, re, im = _data(torch.complex64, 4, 64, 9, skew=(op == "pf"))
    f = getattr(fx, op + "_parts")
    fp = getattr(fx, op + "_planar")
    with torch.no_grad():
        v0, g0 = f(a, prec="ieee")
        v1, g_re, g_im = fp(re, im, prec="ieee", grad=True)
        (v2,) = fp(re, im, prec="ieee")
    _eq(v1, v0)
    _eq(v2, v0)
    _eq(g_re, g0.real.contiguous())
    _eq(g_im, g0.imag.contiguous())


def test_planar_multi_chunk_route():
    """complex128 n = 256 (converting route): 1030 matrices are more than one ~1 GiB chunk."""
    a, re, im = _data(torch.complex128, 1030, 256, 4, skew=False)
    with torch.no_grad():
        s0, l0, g0 = fx.slogdet_parts(a)
        s1, l1, g_re, g_im = fx.slogdet_planar(re, im, grad=True)
    _eq(s1, s0)
    _eq(l1, l0)
    _eq(g_re, g0.real.contiguous())
    _eq(g_im, g0.imag.contiguous())


def test_planar_rejects_real_dtypes():
    from fermix_b200 import _lib

    L = _lib.lib()
    assert L.fermix_slogdet_planar(None, _lib.FX_F32, 0, 1, 4, None, None, None, None, None, None, 0) == 1
    x = torch.zeros((2, 4, 4), device="cuda", dtype=torch.float32)
    with pytest.raises(TypeError):
        fx.slogdet_planar(x, x.double())
