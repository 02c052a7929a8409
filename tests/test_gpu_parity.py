"""Parity of the CUDA path (through the public API and the C ABI) with the oracle and the
64-bit references, case by case as in ChenAo-Phys/fermix tests/test_fermix.py."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx
import oracle
from oracle.refs64 import (
    adjT64,
    assert_sign,
    is_complex,
    log_tol,
    pf64,
    pf_gradT64,
    pf_ref64,
    randn,
    rank_deficient,
    ref64,
    rel_tol,
    relerr,
    shifted,
    skew,
    skew_rank_deficient,
    tol,
)
from tests.helpers import DTYPES, IDS, cuda, host, jgrad

pytestmark = pytest.mark.gpu
dtypes = pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
complex_dtypes = pytest.mark.parametrize("dtype", DTYPES[2:], ids=IDS[2:])


def slogdet(a, **kw):
    return host(fx.slogdet(cuda(a), **kw))


def slogpf(a, **kw):
    return host(fx.slogpf(cuda(a), **kw))


# ------------------------------------------------------------ forward
@pytest.mark.parametrize("n", [0, 1, 3, 5, 8, 24, 40, 96, 128])
@dtypes
def test_slogdet_matches_numpy_and_oracle(n, dtype):
    A = randn((5, n, n), dtype, np.random.default_rng(100 + n))
    s, l = slogdet(A)
    assert s.dtype == dtype and l.dtype == np.finfo(dtype).dtype
    s64, l64 = np.linalg.slogdet(ref64(A))
    assert_sign(s, s64, dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - l64)) < log_tol(dtype, n)
    so, lo = oracle.slogdet(A)
    assert_sign(s, so, dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - lo)) < log_tol(dtype, n)


@pytest.mark.parametrize("n", [0, 2, 4, 6, 8, 34, 64, 128])
@dtypes
def test_slogpf_matches_reference(n, dtype):
    S = skew(randn((5, n, n), dtype, np.random.default_rng(200 + n)))
    s, l = slogpf(S, skew_symmetrize=False)
    ref = [pf_ref64(S[i]) for i in range(5)]
    assert_sign(s, [r[0] for r in ref], dtype, log_tol(dtype))
    assert np.max(np.abs(l - [r[1] for r in ref])) < log_tol(dtype)
    so, lo = oracle.slogpf(S, skew_symmetrize=False)
    assert np.max(np.abs(l - lo)) < log_tol(dtype)


@dtypes
def test_n192_forward_and_grad(dtype):
    """n = 192: the gradient's two work buffers no longer fit in shared memory for any
    dtype, so this runs the global-workspace variant; the primal under the gradient is
    bit-identical to the forward."""
    n = 192
    gen = np.random.default_rng(17)
    A = randn((3, n, n), dtype, gen)
    s, l = slogdet(A)
    s64, l64 = np.linalg.slogdet(ref64(A))
    assert_sign(s, s64, dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - l64)) < log_tol(dtype, n)
    S = skew(randn((3, n, n), dtype, gen))
    s, l = slogpf(S)
    ref = [pf_ref64(S[i]) for i in range(3)]
    assert_sign(s, [r[0] for r in ref], dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - [r[1] for r in ref])) < log_tol(dtype, n)
    W = (randn((3, n, n), dtype, gen) / np.sqrt(n) + 2 * np.eye(n)).astype(dtype)
    s2, l2, g = host(fx.slogdet_parts(cuda(W)))
    s1, l1 = slogdet(W)
    assert np.array_equal(s1, s2) and np.array_equal(l1, l2)
    ref_g = np.swapaxes(np.linalg.inv(ref64(W)), -1, -2)
    assert relerr(g, ref_g) < rel_tol(dtype)


@dtypes
def test_det_pf_values_batch_dims_and_odd_n(dtype):
    gen = np.random.default_rng(3)
    rt = rel_tol(dtype)
    A = randn((2, 3, 5, 5), dtype, gen)
    d = host(fx.det(cuda(A)))
    assert d.shape == (2, 3) and d.dtype == dtype
    assert np.allclose(d, np.linalg.det(ref64(A)), rtol=rt, atol=rt / 10)
    S = skew(randn((4, 12, 12), dtype, gen))
    p = host(fx.pf(cuda(S)))
    assert np.allclose(p, [pf64(S[i]) for i in range(4)], rtol=rt, atol=rt / 10)
    odd = np.zeros((3, 7, 7), dtype)
    assert np.all(host(fx.pf(cuda(odd))) == 0)
    s, l = slogpf(odd)
    assert np.all(s == 0) and np.all(np.isneginf(l))


@dtypes
def test_output_dtypes(dtype):
    real = np.finfo(dtype).dtype
    gen = np.random.default_rng(4)
    for n in (4, 12):
        A = randn((2, n, n), dtype, gen)
        s, l = slogdet(A)
        assert s.dtype == dtype and l.dtype == real
        assert host(fx.det(cuda(A))).dtype == dtype
        s, l = slogpf(A)
        assert s.dtype == dtype and l.dtype == real
        assert host(fx.pf(cuda(A))).dtype == dtype
    odd = np.zeros((2, 7, 7), dtype)
    s, l = slogpf(odd)
    assert s.dtype == dtype and l.dtype == real


@pytest.mark.parametrize("bad", [torch.float16, torch.bfloat16, torch.int32])
def test_rejects_unsupported_dtype(bad):
    with pytest.raises(TypeError):
        fx.slogdet(torch.eye(4, dtype=bad, device="cuda"))


def test_rejects_bad_shape_block_prec_and_cpu():
    with pytest.raises(ValueError):
        fx.slogdet(torch.zeros((3, 4), device="cuda"))
    with pytest.raises(ValueError):
        fx.slogdet(torch.zeros((5,), device="cuda"))
    for block in (16, 48, 256):
        with pytest.raises(ValueError):
            fx.slogdet(torch.eye(40, device="cuda"), block=block)
        with pytest.raises(ValueError):
            fx.det(torch.eye(40, device="cuda"), block=block)
    with pytest.raises(ValueError):
        fx.det(torch.eye(8, device="cuda"), prec="fast")
    with pytest.raises(ValueError):
        fx.slogdet(torch.eye(8, dtype=torch.float64, device="cuda"), prec="tf32x3")
    with pytest.raises(ValueError):
        fx.pf(torch.eye(8, dtype=torch.complex128, device="cuda"), prec="tf32x3")
    with pytest.raises(RuntimeError):
        fx.slogdet(torch.eye(8))  # a CPU tensor: no fallback


def test_public_kwargs_match_defaults():
    n = 72
    gen = np.random.default_rng(21)
    A = shifted((3, n, n), np.float32, 2, gen)
    s0, l0 = slogdet(A)
    for kw in (dict(block=32), dict(block=64), dict(block=128), dict(unroll_steps=True), dict(unroll_steps=False)):
        s, l = slogdet(A, **kw)
        assert np.array_equal(s, s0) and np.max(np.abs(l - l0)) < log_tol(np.float32, n)
    S = skew(randn((3, n, n), np.float32, gen))
    s0, l0 = slogpf(S)
    for warps in (2, 8):
        s, l = slogpf(S, upd_warps=warps)
        assert np.array_equal(s, s0) and np.max(np.abs(l - l0)) < log_tol(np.float32, n)


@dtypes
def test_prec_option(dtype):
    n = 8
    A = randn((2, n, n), dtype, np.random.default_rng(22))
    S = skew(A)
    s64, l64 = np.linalg.slogdet(ref64(A))
    for prec in ("ieee",) + (("tf32x3", None) if np.finfo(dtype).bits == 32 else (None,)):
        s, l = slogdet(A, prec=prec)
        assert_sign(s, s64, dtype, log_tol(dtype))
        assert np.max(np.abs(l - l64)) < log_tol(dtype)
        s, l = slogpf(S, prec=prec)
        ref = [pf_ref64(S[i]) for i in range(2)]
        assert_sign(s, [r[0] for r in ref], dtype, log_tol(dtype))
        assert np.max(np.abs(l - [r[1] for r in ref])) < log_tol(dtype)


# ------------------------------------------------------------ gradients, regular
@pytest.mark.parametrize("n", [3, 48, 128])
@dtypes
def test_slogdet_grad_and_jvp(n, dtype):
    rt = rel_tol(dtype)
    A = shifted((4, n, n), dtype, max(3.0, np.sqrt(n) + 2), np.random.default_rng(23))
    g = jgrad(lambda a: fx.slogdet(a)[1], A)
    inv = np.linalg.inv(ref64(A))
    assert relerr(g, np.swapaxes(inv, -1, -2)) < rt
    assert relerr(g, oracle.slogdet_grad(A)) < rt
    dA = randn(A.shape, dtype, np.random.default_rng(24))
    (s, _), (ds, dl) = torch.func.jvp(fx.slogdet, (cuda(A),), (cuda(dA),))
    s, ds, dl = host(s), host(ds), host(dl)
    tr = np.einsum("bij,bji->b", inv, ref64(dA))
    assert np.allclose(dl, tr.real, rtol=rt, atol=rt)
    if is_complex(dtype):
        assert np.allclose(ds, 1j * tr.imag * s, rtol=rt, atol=rt)
    else:
        assert np.all(ds == 0)


@complex_dtypes
def test_complex_conventions(dtype):
    """torch.autograd matches torch.linalg.slogdet's convention (the conjugate of
    JAX's); the sign cotangent enters as in torch.linalg.slogdet."""
    n = 16
    rt = rel_tol(dtype)
    A = shifted((3, n, n), dtype, 3, np.random.default_rng(25))
    gs = randn((3,), dtype, np.random.default_rng(26))
    gl = np.random.default_rng(27).standard_normal(3)
    x = cuda(A, requires_grad=True)
    s, l = fx.slogdet(x)
    (g,) = torch.autograd.grad((s, l), x, (cuda(gs), cuda(gl.astype(np.finfo(dtype).dtype))))
    x2 = cuda(A.astype(np.complex128), requires_grad=True)
    s2, l2 = torch.linalg.slogdet(x2)
    (g2,) = torch.autograd.grad((s2, l2), x2, (cuda(gs.astype(np.complex128)), cuda(gl)))
    assert relerr(host(g), host(g2)) < rt
    x = cuda(A, requires_grad=True)
    (g,) = torch.autograd.grad(torch.real(fx.det(x)).sum(), x)
    x2 = cuda(A.astype(np.complex128), requires_grad=True)
    (g2,) = torch.autograd.grad(torch.real(torch.linalg.det(x2)).sum(), x2)
    assert relerr(host(g), host(g2)) < rt


@pytest.mark.parametrize("n", [6, 32, 96, 128])
@dtypes
def test_slogpf_grad(n, dtype):
    A = randn((4, n, n), dtype, np.random.default_rng(1000 + n))
    g = jgrad(lambda a: fx.slogpf(a)[1], A)
    S = 0.5 * skew(ref64(A))
    assert relerr(g, 0.5 * np.swapaxes(np.linalg.inv(S), -1, -2)) < rel_tol(dtype)


@pytest.mark.parametrize("n", [4, 6, 16, 40, 130])
@dtypes
def test_grad_primal_is_bit_identical_to_forward(n, dtype):
    gen = np.random.default_rng(11)
    A = shifted((3, n, n), dtype, 3, gen)
    for parts, f, a in ((fx.slogdet_parts, fx.slogdet, A), (fx.slogpf_parts, fx.slogpf, skew(A))):
        s1, l1 = host(f(cuda(a)))
        s2, l2, _ = host(parts(cuda(a)))
        assert np.array_equal(s1, s2) and np.array_equal(l1, l2)
    for parts, f, a in ((fx.det_parts, fx.det, A), (fx.pf_parts, fx.pf, skew(A))):
        v1 = host(f(cuda(a)))
        v2, _ = host(parts(cuda(a)))
        assert np.array_equal(v1, v2)


@dtypes
def test_det_pf_grad_regular(dtype):
    gen = np.random.default_rng(28)
    n = 12
    A = shifted((3, n, n), dtype, 2, gen)
    g = jgrad(fx.det, A)
    ref = np.stack([np.linalg.det(a) * np.linalg.inv(a).T for a in ref64(A)])
    assert relerr(g, ref) < rel_tol(dtype)
    S = skew(randn((3, n, n), dtype, gen))
    g = jgrad(lambda a: fx.pf(a, skew_symmetrize=False), S)
    ref = np.stack([0.5 * pf64(s) * np.linalg.inv(s).T for s in ref64(S)])
    assert relerr(g, ref) < rel_tol(dtype)


# ------------------------------------------------------------ gradients, singular
@dtypes
def test_slogdet_slogpf_singular_grad_is_zero_and_finite(dtype):
    n = 40
    gen = np.random.default_rng(29)
    A = randn((3, n, n), dtype, gen)
    A[0, :, 5] = 0.0
    A[1] = 0.0
    s, l = slogdet(A)
    assert np.all(s[:2] == 0) and np.all(np.isneginf(l[:2]))
    g = jgrad(lambda a: fx.slogdet(a)[1], A)
    assert np.all(np.isfinite(g)) and np.all(g[:2] == 0)
    assert relerr(g[2], np.linalg.inv(ref64(A[2])).T) < rel_tol(dtype) * 10
    S = skew(randn((3, n, n), dtype, gen))
    S[0, 7, :] = 0.0
    S[0, :, 7] = 0.0
    g = jgrad(lambda a: fx.slogpf(a, skew_symmetrize=False)[1], S)
    assert np.all(np.isfinite(g)) and np.all(g[0] == 0)


@pytest.mark.parametrize("n", [3, 8, 40])
@dtypes
def test_det_grad_singular(n, dtype):
    B = 6
    A = shifted((B, n, n), dtype, 2, np.random.default_rng(30))
    A[0, :, 1] = 0.0
    A[1, 2 % n] = 0.0
    A[2] = 0.0
    A[3, :, 0] = 0.0
    A[3, :, 1] = 0.0
    A[4, :, 0] = 0.0
    A[4, 1] = 0.0
    g = jgrad(fx.det, A)
    assert np.all(np.isfinite(g))
    ref = np.stack([adjT64(a) for a in ref64(A)])
    scale = max(np.abs(ref).max(), 1e-30)
    assert np.max(np.abs(g - ref)) < rel_tol(dtype) * scale
    assert np.all(g[2] == 0) and np.all(g[3] == 0)
    for k in (0, 1, 4):
        assert np.abs(ref[k]).max() > 0 and relerr(g[k], ref[k]) < rel_tol(dtype)


@pytest.mark.parametrize("n", [8, 24])
@dtypes
def test_det_grad_near_singular(n, dtype):
    A = rank_deficient((4, n, n), dtype, np.random.default_rng(31))
    g = jgrad(fx.det, A)
    ref = np.stack([adjT64(a) for a in ref64(A)])
    for k in range(len(A)):
        assert relerr(g[k], ref[k]) < tol(dtype, 1e-4, 1e-9)


@pytest.mark.parametrize("n", [4, 8, 14])
@dtypes
def test_pf_grad_singular(n, dtype):
    B = 4
    S = skew(randn((B, n, n), dtype, np.random.default_rng(32)))
    S[0, 3 % n, :] = 0.0
    S[0, :, 3 % n] = 0.0
    S[1] = 0.0
    S[2, 1, :] = 0.0
    S[2, :, 1] = 0.0
    S[2, 3 % n, :] = 0.0
    S[2, :, 3 % n] = 0.0
    g = jgrad(lambda a: fx.pf(a, skew_symmetrize=False), S)
    assert np.all(np.isfinite(g))
    ref = np.stack([pf_gradT64(s) for s in ref64(S)])
    scale = max(np.abs(ref).max(), 1e-30)
    assert np.max(np.abs(g - ref)) < rel_tol(dtype) * scale
    assert np.all(g[1] == 0) and np.abs(ref[0]).max() > 0
    if n > 4:
        assert np.abs(ref[2]).max() > 0


@pytest.mark.parametrize("n", [8, 24])
@dtypes
def test_pf_grad_near_singular(n, dtype):
    S = skew_rank_deficient((4, n, n), dtype, np.random.default_rng(33))
    g = jgrad(lambda a: fx.pf(a, skew_symmetrize=False), S)
    ref = np.stack([pf_gradT64(s) for s in ref64(S)])
    for k in range(len(S)):
        assert relerr(g[k], ref[k]) < tol(dtype, 1e-4, 1e-9)


# ------------------------------------------------------------ vmap
@dtypes
def test_vmap_matches_batched(dtype):
    n = 12
    gen = np.random.default_rng(5)
    A = shifted((4, n, n), dtype, 2, gen)
    A[0, :, 3] = 0.0
    S = skew(randn((4, n, n), dtype, gen))
    S[0, 2, :] = 0.0
    S[0, :, 2] = 0.0
    S[1, 5, :] = 0.0
    S[1, :, 5] = 0.0
    S[1, 7, :] = 0.0
    S[1, :, 7] = 0.0
    cases = [
        (fx.slogdet, lambda o: o[1], A),
        (fx.det, lambda o: torch.real(o), A),
        (lambda a: fx.slogpf(a, skew_symmetrize=False), lambda o: o[1], S),
        (lambda a: fx.pf(a, skew_symmetrize=False), lambda o: torch.real(o), S),
    ]
    for f, sel, x in cases:
        x = cuda(x)
        out_b = f(x)
        out_v = torch.func.vmap(f)(x)
        for b, v in zip(torch.utils._pytree.tree_leaves(out_b), torch.utils._pytree.tree_leaves(out_v)):
            assert torch.equal(b, v)
        gb = host(torch.func.grad(lambda a: sel(f(a)).sum())(x))
        gv = host(torch.func.vmap(torch.func.grad(lambda a: sel(f(a))))(x))
        assert np.all(np.isfinite(gb))
        assert relerr(gv, gb) < tol(dtype, 1e-6, 1e-14)


# ------------------------------------------------------------ larger n
@dtypes
def test_n300_forward_and_grad(dtype):
    n = 300
    gen = np.random.default_rng(11)
    A = randn((2, n, n), dtype, gen)
    s, l = slogdet(A)
    s64, l64 = np.linalg.slogdet(ref64(A))
    assert_sign(s, s64, dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - l64)) < log_tol(dtype, n)
    s2, l2, g = host(fx.slogdet_parts(cuda(A)))
    assert np.array_equal(s, s2) and np.array_equal(l, l2)
    inv = np.linalg.inv(ref64(A))
    assert relerr(g, np.swapaxes(inv, -1, -2)) < tol(dtype, 1e-3, 1e-9)


@pytest.mark.parametrize(
    "dtype,n",
    [(np.float32, 236), (np.float32, 240), (np.float64, 170), (np.complex64, 170), (np.complex128, 120)],
    ids=["f32-236-smem", "f32-240-ws", "f64-170-ws", "c64-170-ws", "c128-120-ws"],
)
def test_register_panel_shared_and_workspace_modes(dtype, n):
    """The register-panel kernels (n <= 256) with the matrix in shared memory and, once
    it no longer fits, in the global workspace: forward, primal under the gradient, and
    both gradients against the 64-bit references."""
    gen = np.random.default_rng(40 + n)
    A = randn((2, n, n), dtype, gen)
    s, l = slogdet(A)
    s64, l64 = np.linalg.slogdet(ref64(A))
    assert_sign(s, s64, dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - l64)) < log_tol(dtype, n)
    s2, l2, g = host(fx.slogdet_parts(cuda(A)))
    assert np.array_equal(s, s2) and np.array_equal(l, l2)
    assert relerr(g, np.swapaxes(np.linalg.inv(ref64(A)), -1, -2)) < tol(dtype, 3e-3, 1e-9)
    S = skew(randn((2, n, n), dtype, gen))
    s, l = slogpf(S, skew_symmetrize=False)
    ref = [pf_ref64(S[i]) for i in range(2)]
    assert_sign(s, [r[0] for r in ref], dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - [r[1] for r in ref])) < log_tol(dtype, n)
    s2, l2, g = host(fx.slogpf_parts(cuda(S), skew_symmetrize=False))
    assert np.array_equal(s, s2) and np.array_equal(l, l2)
    assert relerr(g, 0.5 * np.swapaxes(np.linalg.inv(ref64(S)), -1, -2)) < tol(dtype, 3e-3, 1e-9)


@dtypes
def test_n300_slogpf_large_engine(dtype):
    """n = 300 (> 256): the blocked Parlett-Reid forward and the Gauss-Jordan gradient of
    the large-n engine; the primal of slogpf_parts / pf_parts equals slogpf's bits, and an
    exactly singular skew input gives (0, -inf) with a zero gradient."""
    n = 300
    gen = np.random.default_rng(23)
    S = skew(randn((2, n, n), dtype, gen))
    s, l = slogpf(S)
    ref = [pf_ref64(S[i]) for i in range(2)]
    assert_sign(s, [r[0] for r in ref], dtype, log_tol(dtype, n))
    assert np.max(np.abs(l - [r[1] for r in ref])) < log_tol(dtype, n)
    s2, l2, g = host(fx.slogpf_parts(cuda(S)))
    assert np.array_equal(s, s2) and np.array_equal(l, l2)
    Sh = 0.5 * (ref64(S) - np.swapaxes(ref64(S), -1, -2))
    assert relerr(g, 0.5 * np.swapaxes(np.linalg.inv(Sh), -1, -2)) < tol(dtype, 1e-3, 1e-9)
    v1 = host(fx.pf(cuda(S)))
    v2, _ = host(fx.pf_parts(cuda(S)))
    assert np.array_equal(v1, v2)
    Z = skew(randn((1, n, n), dtype, gen))
    Z[0, 7, :] = 0.0
    Z[0, :, 7] = 0.0
    sz, lz, gz = host(fx.slogpf_parts(cuda(Z)))
    assert sz[0] == 0 and lz[0] == -np.inf and np.all(np.isfinite(gz)) and not np.any(gz)


@dtypes
def test_n300_det_adjugate_primal_matches_forward(dtype):
    """n = 300: det_parts runs the generic adjugate kernel and rewrites the primal with the
    large-n forward, so det equals det_parts' value bit for bit."""
    n = 300
    gen = np.random.default_rng(29)
    A = (randn((2, n, n), dtype, gen) / np.sqrt(n) + np.eye(n)).astype(dtype)
    v1 = host(fx.det(cuda(A)))
    v2, g = host(fx.det_parts(cuda(A)))
    assert np.array_equal(v1, v2)
    s64, l64 = np.linalg.slogdet(ref64(A))
    want = np.swapaxes(np.linalg.inv(ref64(A)), -1, -2) * (s64 * np.exp(l64))[:, None, None]
    assert relerr(g, want) < tol(dtype, 1e-3, 1e-9)


def test_cluster_panel_pfaffian_known_value():
    """n = 4200 > 4096: the large-n Parlett-Reid panel spans a cluster of five blocks at
    first. S = Q J Q^T with J = diag([[0, 1], [-1, 0]]) and Q = D L (D diagonal, L unit
    lower) has pf(S) = det(Q) = prod(D)."""
    n = 4200
    gen = np.random.default_rng(43)
    d = gen.uniform(0.7, 1.4, n) * gen.choice([-1.0, 1.0], n)
    Lw = np.tril(gen.standard_normal((n, n)) * (0.3 / np.sqrt(n)), -1) + np.eye(n)
    Q = d[:, None] * Lw
    J = np.kron(np.eye(n // 2), np.array([[0.0, 1.0], [-1.0, 0.0]]))
    M = Q @ J @ Q.T
    S = 0.5 * (M - M.T)
    s, l = host(fx.slogpf(cuda(S[None])))
    want_s = np.prod(np.sign(d))
    want_l = np.sum(np.log(np.abs(d)))
    assert s[0] == want_s
    assert abs(l[0] - want_l) < 1e-8 * max(1.0, abs(want_l))
