"""Failure paths of the C ABI on the GPU, without faulting it:

* bounded waits: with the wait limit set to 0 polls every tensor-core completion wait and
  the Pfaffian move's bulk-copy wait give up at once. The kernels then wait once more with
  the default limit (so nothing is in flight when they go on), write NaN for the affected
  members and record FX_ERR_TIMEOUT in the device status word, which fermix_device_status
  reports. After the limit is restored the same calls give the normal results again;
* a workspace at an odd (8-byte) offset gives the same bits as a 256-byte aligned one."""

import ctypes

import numpy as np
import pytest
import torch

import fermix_b200 as fx
from fermix_b200 import _lib
from tests.helpers import cuda, host

pytestmark = pytest.mark.gpu


@pytest.fixture
def zero_polls():
    L = _lib.lib()
    assert _lib.device_status(clear=True) == 0
    prev = L.fermix_set_wait_polls(0)
    try:
        yield L
    finally:
        L.fermix_set_wait_polls(prev)
        _lib.device_status(clear=True)


def _skew(B, n, seed):
    A = np.random.default_rng(seed).standard_normal((B, n, n)).astype(np.float32)
    return A - np.swapaxes(A, -1, -2)


@pytest.mark.parametrize("op", ["slogdet", "slogpf"])
@pytest.mark.parametrize("n", [64, 200])
def test_tensor_core_wait_timeout_gives_nan_and_status(zero_polls, op, n):
    if op == "slogpf" and n > 128:
        n = 128  # the tensor-memory Parlett-Reid kernel covers n <= 128
    X = _skew(8, n, 1) if op == "slogpf" else np.random.default_rng(2).standard_normal((8, n, n)).astype(np.float32)
    parts = fx.slogpf_parts if op == "slogpf" else fx.slogdet_parts
    s, l, g = host(parts(cuda(X), prec="tf32x3"))
    assert np.all(np.isnan(s)) and np.all(np.isnan(l))
    assert np.all(g == 0)  # a member that gave up gets a zero gradient
    assert _lib.device_status() == _lib.FX_ERR_TIMEOUT
    assert _lib.device_status(clear=True) == _lib.FX_ERR_TIMEOUT
    assert _lib.device_status() == 0
    # the forward kernels take the same path
    s, l = host((fx.slogpf if op == "slogpf" else fx.slogdet)(cuda(X), prec="tf32x3"))
    assert np.all(np.isnan(s)) and _lib.device_status(clear=True) == _lib.FX_ERR_TIMEOUT
    # limit restored: normal results, status stays clear (the context is still usable)
    zero_polls.fermix_set_wait_polls(_lib.FX_WAIT_POLLS_DEFAULT)
    s, l, g = host(parts(cuda(X), prec="tf32x3"))
    ref = np.linalg.slogdet(X.astype(np.float64))
    if op == "slogdet":
        assert np.array_equal(s, ref[0].astype(np.float32))
        assert np.abs(l - ref[1]).max() < 1e-3
    assert np.all(np.isfinite(l)) and np.all(np.isfinite(g))
    assert _lib.device_status() == 0


def test_pfaffian_move_copy_wait_timeout_leaves_g_and_reports(zero_polls):
    n, B = 64, 12  # G fits one block's shared memory: the bulk-copy path
    S = _skew(B, n, 3).astype(np.float64) + 0.0
    J = np.zeros((n, n))
    r = np.arange(0, n, 2)
    J[r, r + 1], J[r + 1, r] = 4.0, -4.0
    S = (S / np.sqrt(n) + J).astype(np.float32)
    G = (0.5 * np.swapaxes(np.linalg.inv(S.astype(np.float64)), -1, -2)).astype(np.float32)
    rng = np.random.default_rng(4)
    idx = rng.integers(0, n, B).astype(np.int32)
    row = S[np.arange(B), idx] + 0.05 * rng.standard_normal((B, n)).astype(np.float32)
    g = cuda(G)
    s, l, out = fx.slogpf_update(g, cuda(row), cuda(idx), inplace=True)
    assert np.all(np.isnan(host(s))) and np.all(np.isnan(host(l)))
    assert np.array_equal(host(out), G)  # no member was updated
    assert _lib.device_status(clear=True) == _lib.FX_ERR_TIMEOUT
    zero_polls.fermix_set_wait_polls(_lib.FX_WAIT_POLLS_DEFAULT)
    s, l, out = fx.slogpf_update(g, cuda(row), cuda(idx), inplace=True)
    assert np.all(np.isfinite(host(l))) and _lib.device_status() == 0


def _offset_ws(nbytes, offset, dev):
    buf = torch.empty(nbytes + 512, dtype=torch.uint8, device=dev)
    base = (buf.data_ptr() + 255) // 256 * 256
    return buf, base + offset


@pytest.mark.parametrize("offset", [8, 136])
def test_unaligned_workspace_matches_aligned(offset):
    L = _lib.lib()
    dev = torch.device("cuda")
    sp = torch.cuda.current_stream().cuda_stream
    # large-n slogdet gradient (the blocked engine lives in the workspace), complex128
    n, B = 300, 3
    rng = np.random.default_rng(7)
    A = cuda((rng.standard_normal((B, n, n)) + 1j * rng.standard_normal((B, n, n))).astype(np.complex128))
    nb = L.fermix_workspace_bytes(_lib.FX_OP_SLOGDET, _lib.FX_C128, B, n, 1)
    outs = []
    for off in (0, offset):
        buf, ws = _offset_ws(nb, off, dev)
        sg = torch.empty(B, dtype=A.dtype, device=dev)
        la = torch.empty(B, dtype=torch.float64, device=dev)
        G = torch.empty_like(A)
        _lib.check(L.fermix_slogdet_grad(sp, _lib.FX_C128, 0, B, n, A.data_ptr(), None, 0, 0, sg.data_ptr(),
                                         la.data_ptr(), None, G.data_ptr(), ctypes.c_void_p(ws), nb))
        outs.append(host((sg, la, G)))
        del buf
    for x, y in zip(*outs):
        assert np.array_equal(x, y)
    # k-row move (H in the workspace, read as 16-byte pieces) and Pfaffian move (three launches)
    for pf in (False, True):
        n, k, B = 256, (1 if pf else 3), 8
        X = rng.standard_normal((B, n, n)) / np.sqrt(n)
        if pf:
            X = X - np.swapaxes(X, -1, -2)
            X[:, np.arange(0, n, 2), np.arange(1, n, 2)] += 3.0
            X[:, np.arange(1, n, 2), np.arange(0, n, 2)] -= 3.0
            G0 = 0.5 * np.swapaxes(np.linalg.inv(X), -1, -2)
        else:
            X = X + 2 * np.eye(n)
            G0 = np.swapaxes(np.linalg.inv(X), -1, -2)
        G0 = G0.astype(np.float32)
        idx = np.stack([rng.choice(n, k, replace=False) for _ in range(B)]).astype(np.int32)
        U = (X[np.arange(B)[:, None], idx] + 0.1 * rng.standard_normal((B, k, n)) / np.sqrt(n)).astype(np.float32)
        res = []
        for off in (0, offset):
            g = cuda(G0)
            u = cuda(U[:, 0] if pf else U)
            ix = cuda(idx[:, 0] if pf else idx)
            sg = torch.empty(B, dtype=torch.float32, device=dev)
            la = torch.empty(B, dtype=torch.float32, device=dev)
            if pf:
                nb = L.fermix_slogpf_update_workspace_bytes(_lib.FX_F32, B, n)
                buf, ws = _offset_ws(nb, off, dev)
                st = L.fermix_slogpf_update(sp, _lib.FX_F32, B, n, g.data_ptr(), u.data_ptr(), ix.data_ptr(), None,
                                            sg.data_ptr(), la.data_ptr(), ctypes.c_void_p(ws), nb)
            else:
                nb = L.fermix_slogdet_update_workspace_bytes(_lib.FX_F32, B, n, k)
                buf, ws = _offset_ws(nb, off, dev)
                st = L.fermix_slogdet_update(sp, _lib.FX_F32, B, n, k, g.data_ptr(), u.data_ptr(), ix.data_ptr(),
                                             None, sg.data_ptr(), la.data_ptr(), ctypes.c_void_p(ws), nb)
            _lib.check(st)
            res.append(host((sg, la, g)))
            del buf
        for x, y in zip(*res):
            assert np.array_equal(x, y)
        assert np.all(np.isfinite(res[0][1]))
