"""The XLA custom-call adapter (include/fermix_b200_xla.h) called the way XLA calls it:
an array of device pointers plus the packed descriptor, through ctypes. On the GPU its
outputs must equal the direct C entry point's bit for bit; without a GPU, malformed
descriptors are rejected before any buffer is read."""

import ctypes

import numpy as np
import pytest
import torch

from fermix_b200 import _lib, jax_ffi

KIND = {torch.float32: 0, torch.float64: 1, torch.complex64: 2, torch.complex128: 3}


def _call(desc, ptrs):
    L = _lib.lib()
    arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs) if ptrs is not None else None
    L.fermix_xla_custom_call(None, ctypes.cast(arr, ctypes.c_void_p) if arr is not None else None, desc, len(desc))
    return L.fermix_xla_last_error(1)


def test_descriptor_layout_and_rejections():
    L = _lib.lib()
    L.fermix_xla_last_error(1)
    d = jax_ffi.descriptor(jax_ffi.SLOGPF, 0, 1, 3, 8, flags=jax_ffi.F_SKEW, workspace_bytes=512)
    assert len(d) == 48 and d[:4] == (0x46584231).to_bytes(4, "little")
    assert _call(d[:40], [0] * 4) == 2          # short descriptor: FX_ERR_SHAPE
    bad = bytearray(d)
    bad[0] ^= 1
    assert _call(bytes(bad), [0] * 4) == 2      # wrong magic
    assert _call(jax_ffi.descriptor(7, 0, 1, 3, 8), [0] * 4) == 2  # unknown op
    assert _call(d, None) == 5                  # no buffer array: FX_ERR_NULL
    # a valid empty call reaches the entry point, which returns at once
    assert _call(jax_ffi.descriptor(jax_ffi.SLOGDET, 0, 0, 0, 8), [0] * 3) == 0
    # the entry point's own argument errors are recorded
    assert _call(jax_ffi.descriptor(jax_ffi.SLOGDET, 1, 1, 2, 8), [0] * 3) == 3  # tf32x3 on float64


CASES = [
    ("slogdet", torch.float32, 64, 0), ("slogdet", torch.complex128, 300, 0),
    ("slogpf", torch.float32, 128, 0), ("slogpf", torch.complex64, 40, 0),
    ("slogdet_grad", torch.float32, 100, 0), ("slogdet_grad", torch.float64, 300, jax_ffi.F_COEF),
    ("slogdet_grad", torch.complex64, 24, jax_ffi.F_ADJUGATE | jax_ffi.F_VALUE | jax_ffi.F_CONJ_OUT),
    ("slogpf_grad", torch.float32, 128, jax_ffi.F_SKEW), ("slogpf_grad", torch.complex128, 260, jax_ffi.F_SKEW),
    ("slogpf_grad", torch.float64, 30, jax_ffi.F_ADJUGATE | jax_ffi.F_VALUE | jax_ffi.F_COEF),
]


@pytest.mark.gpu
@pytest.mark.parametrize("name,dtype,n,flags", CASES, ids=[f"{c[0]}-{str(c[1])[6:]}-n{c[2]}-f{c[3]}" for c in CASES])
def test_adapter_equals_direct_entry_point(name, dtype, n, flags):
    L = _lib.lib()
    L.fermix_xla_last_error(1)
    op = {"slogdet": jax_ffi.SLOGDET, "slogdet_grad": jax_ffi.SLOGDET_GRAD, "slogpf": jax_ffi.SLOGPF,
          "slogpf_grad": jax_ffi.SLOGPF_GRAD}[name]
    grad = name.endswith("grad")
    pf = name.startswith("slogpf")
    B, dev = 6, torch.device("cuda")
    kind = KIND[dtype]
    g = torch.Generator(device=dev).manual_seed(n)
    a = torch.randn((B, n, n), generator=g, device=dev, dtype=dtype)
    if pf and not flags & jax_ffi.F_SKEW:
        a = (a - a.transpose(-1, -2)).contiguous()
    coef = torch.randn(B, generator=g, device=dev, dtype=dtype) if flags & jax_ffi.F_COEF else None
    real = torch.float32 if dtype in (torch.float32, torch.complex64) else torch.float64
    ws = jax_ffi.workspace_bytes(op, kind, B, n)

    def outputs():
        return (torch.full((B,), 7.0, device=dev, dtype=dtype), torch.full((B,), 7.0, device=dev, dtype=real),
                torch.full((B,), 7.0, device=dev, dtype=dtype) if flags & jax_ffi.F_VALUE else None,
                torch.full_like(a, 7.0) if grad else None,
                torch.empty(ws, dtype=torch.uint8, device=dev) if ws else None)

    # through the adapter
    sg, la, val, G, w = outputs()
    ptrs = [a.data_ptr()] + ([coef.data_ptr()] if coef is not None and grad else []) + [sg.data_ptr(), la.data_ptr()]
    ptrs += ([val.data_ptr()] if val is not None else []) + ([G.data_ptr()] if grad else [])
    ptrs += [w.data_ptr()] if ws else []
    desc = jax_ffi.descriptor(op, kind, 0, B, n, flags=flags, workspace_bytes=ws)
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    L.fermix_xla_custom_call(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                             ctypes.cast(arr, ctypes.c_void_p), desc, len(desc))
    assert L.fermix_xla_last_error(1) == 0
    # direct
    s2, l2, v2, G2, w2 = outputs()
    sp = torch.cuda.current_stream().cuda_stream
    P = lambda t: None if t is None else t.data_ptr()
    skew, conj, adj = int(bool(flags & jax_ffi.F_SKEW)), int(bool(flags & jax_ffi.F_CONJ_OUT)), int(
        bool(flags & jax_ffi.F_ADJUGATE))
    if name == "slogdet":
        st = L.fermix_slogdet(sp, kind, 0, B, n, P(a), P(s2), P(l2), P(v2), P(w2), ws)
    elif name == "slogpf":
        st = L.fermix_slogpf(sp, kind, 0, B, n, skew, P(a), P(s2), P(l2), P(v2), P(w2), ws)
    elif name == "slogdet_grad":
        st = L.fermix_slogdet_grad(sp, kind, 0, B, n, P(a), P(coef), conj, adj, P(s2), P(l2), P(v2), P(G2), P(w2), ws)
    else:
        st = L.fermix_slogpf_grad(sp, kind, 0, B, n, skew, P(a), P(coef), conj, adj, P(s2), P(l2), P(v2), P(G2),
                                  P(w2), ws)
    _lib.check(st)
    torch.cuda.synchronize()
    for x, y in ((sg, s2), (la, l2), (val, v2), (G, G2)):
        if x is not None:
            assert torch.equal(x, y) or (torch.isnan(x) == torch.isnan(y)).all() and torch.equal(
                torch.nan_to_num(x), torch.nan_to_num(y))
    assert torch.isfinite(la).all() or not torch.isfinite(l2).all()
