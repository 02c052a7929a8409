"""fermix_slogdet_grad_static (the workspace-free variant of fermix_slogdet_grad, for
callers that cannot allocate device memory when they call) against fermix_slogdet_grad
with a caller workspace: two calls in a row on one stream, bit for bit.

The file name makes pytest collect it last, so it runs after every other test has used
the library on the device, and it also passes on its own."""

import ctypes

import numpy as np
import pytest
import torch

from fermix_b200 import _lib

from tests.helpers import TORCH

CODE = {np.float32: _lib.FX_F32, np.float64: _lib.FX_F64, np.complex64: _lib.FX_C64, np.complex128: _lib.FX_C128}
REAL = {np.float32: torch.float32, np.float64: torch.float64, np.complex64: torch.float32, np.complex128: torch.float64}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _matrices(dtype, batch, n, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, n, n))
    if np.iscomplexobj(np.zeros(1, dtype)):
        x = x + 1j * rng.standard_normal((batch, n, n))
    x = x.astype(dtype)
    x[0, 1] = x[0, 0]  # an exactly singular member (two equal rows)
    return torch.from_numpy(x).cuda()


def _outputs(dtype, batch, n):
    td = TORCH[np.dtype(dtype)]
    return (
        torch.empty(batch, dtype=td, device="cuda"),
        torch.empty(batch, dtype=REAL[dtype], device="cuda"),
        torch.empty(batch, dtype=td, device="cuda"),
        torch.empty(batch, n, n, dtype=td, device="cuda"),
    )


def _with_workspace(L, stream, dtype, a, coef, adjugate):
    batch, n = a.shape[0], a.shape[1]
    sign, logabs, value, grad = _outputs(dtype, batch, n)
    wsb = L.fermix_workspace_bytes(_lib.FX_OP_SLOGDET, CODE[dtype], batch, n, 1)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device="cuda")
    _lib.check(
        L.fermix_slogdet_grad(
            stream, CODE[dtype], 0, batch, n, _ptr(a), _ptr(coef), 0, adjugate,
            _ptr(sign), _ptr(logabs), _ptr(value), _ptr(grad), _ptr(ws), wsb,
        )
    )
    return wsb, (sign, logabs, value, grad)


def _static(L, stream, dtype, a, coef, adjugate):
    batch, n = a.shape[0], a.shape[1]
    sign, logabs, value, grad = _outputs(dtype, batch, n)
    _lib.check(
        L.fermix_slogdet_grad_static(
            stream, CODE[dtype], 0, batch, n, _ptr(a), _ptr(coef), 0, adjugate,
            _ptr(sign), _ptr(logabs), _ptr(value), _ptr(grad),
        )
    )
    return sign, logabs, value, grad


@pytest.mark.gpu
@pytest.mark.parametrize(
    "dtype,batch,n,adjugate",
    [
        (np.float64, 40, 300, 0),  # blocked kernel, slots in the static array (11 fit)
        (np.complex128, 24, 160, 1),  # register-panel kernel, slots in the static array
        (np.complex64, 3, 1024, 0),  # exactly one slot fits: one block in flight
        (np.float32, 64, 64, 0),  # fits in shared memory: the array is not touched
    ],
    ids=["f64-n300", "c128-n160-adj", "c64-n1024-one-slot", "f32-n64-smem"],
)
def test_static_scratch_matches_workspace_entry(dtype, batch, n, adjugate):
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    a1 = _matrices(dtype, batch, n, seed=11)
    a2 = _matrices(dtype, batch, n, seed=12)
    rng = np.random.default_rng(13)
    coef = torch.from_numpy((rng.standard_normal(batch) + 0.5).astype(dtype)).cuda()
    # two calls in a row on one stream: the second reuses the slots the first wrote
    s1 = _static(L, stream, dtype, a1, coef, adjugate)
    s2 = _static(L, stream, dtype, a2, coef, adjugate)
    wsb, r1 = _with_workspace(L, stream, dtype, a1, coef, adjugate)
    _, r2 = _with_workspace(L, stream, dtype, a2, coef, adjugate)
    torch.cuda.synchronize()
    if n >= 160:
        assert wsb > 0  # the case runs in slot mode
    for got, want in ((s1, r1), (s2, r2)):
        for g, w, name in zip(got, want, ("sign", "logabs", "value", "grad")):
            assert torch.equal(g.contiguous().view(torch.uint8), w.contiguous().view(torch.uint8)), name
    # the singular member takes the documented values
    assert s1[0][0].item() == 0 and s1[1][0].item() == -np.inf


@pytest.mark.gpu
def test_static_scratch_rejects_oversize_before_launch():
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    n = 800  # complex128: one slot is 2 * 800^2 * 16 bytes > 16 MiB
    a = torch.zeros(1, n, n, dtype=torch.complex128, device="cuda")
    sign, logabs, value, grad = _outputs(np.complex128, 1, n)
    rc = L.fermix_slogdet_grad_static(
        stream, _lib.FX_C128, 0, 1, n, _ptr(a), None, 0, 0, _ptr(sign), _ptr(logabs), _ptr(value), _ptr(grad)
    )
    assert rc == 4  # FX_ERR_WORKSPACE
    # the rejection queued no work: the device context is clean
    torch.cuda.synchronize()
    assert L.fermix_slogdet_grad_static(stream, _lib.FX_C128, 0, 0, n, None, None, 0, 0, None, None, None, None) == 0
