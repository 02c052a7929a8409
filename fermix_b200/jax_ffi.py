"""JAX binding of libfermix_b200.so through XLA's legacy custom-call ABI
(include/fermix_b200_xla.h), the host the reference itself runs on.

:func:`descriptor` packs the opaque bytes of one call; :func:`register` registers the
adapter ``fermix_xla_custom_call`` with ``jax.ffi`` (api_version 0, which needs no XLA
headers); :func:`slogdet` / :func:`slogpf` are jitted JAX functions with the reference's
custom_jvp conventions (src/fermix/_diff.py:92-156) on top of the custom calls.

The descriptor packing and the adapter are tested through ctypes against the direct C
entry points (tests/test_xla_adapter.py). The JAX part needs jax / jaxlib, which this
image does not have: it is the binding a JAX user would import, and it is unverified here.
"""

import ctypes
import struct

from . import _lib

MAGIC, VERSION = 0x46584231, 1
SLOGDET, SLOGDET_GRAD, SLOGPF, SLOGPF_GRAD = 0, 1, 2, 3
F_VALUE, F_COEF, F_CONJ_OUT, F_ADJUGATE, F_SKEW = 1, 2, 4, 8, 16
_DESC = struct.Struct("<IiiiiIqqQ")
assert _DESC.size == 48


def descriptor(op, dtype, prec, batch, n, *, flags=0, workspace_bytes=0):
    """The 48 opaque bytes of one custom call (fermix_xla_descriptor)."""
    return _DESC.pack(MAGIC, VERSION, op, dtype, prec, flags, batch, n, workspace_bytes)


def workspace_bytes(op, dtype, batch, n):
    """Scratch the call needs (the extra uint8 output buffer; 0 means none)."""
    grad = op in (SLOGDET_GRAD, SLOGPF_GRAD)
    kind = _lib.FX_OP_SLOGPF if op in (SLOGPF, SLOGPF_GRAD) else _lib.FX_OP_SLOGDET
    return int(_lib.lib().fermix_workspace_bytes(kind, dtype, batch, n, int(grad)))


def target():
    """The adapter's address as a C function pointer."""
    return ctypes.cast(_lib.lib().fermix_xla_custom_call, ctypes.c_void_p).value


_registered = False
_fn_keep = None  # the ctypes function object must outlive the registration


def register(name="fermix_b200"):
    """Register the adapter as an XLA custom-call target for CUDA (needs jax)."""
    global _registered, _fn_keep
    import jax

    if not _registered:
        fn = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t)(target())
        _fn_keep = fn
        jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(fn), platform="CUDA", api_version=0)
        _registered = True
    return name


def _call(op, a, prec, flags):
    import jax
    import jax.numpy as jnp
    import numpy as np

    kinds = {np.dtype(np.float32): 0, np.dtype(np.float64): 1, np.dtype(np.complex64): 2,
             np.dtype(np.complex128): 3}
    B, n = a.shape[0], a.shape[-1]
    dt = kinds[np.dtype(a.dtype)]
    p = {None: 0, "tf32x3": 1, "ieee": 2}[prec]
    ws = workspace_bytes(op, dt, B, n)
    real = jnp.finfo(a.dtype).dtype
    outs = [jax.ShapeDtypeStruct((B,), a.dtype), jax.ShapeDtypeStruct((B,), real)]
    if op in (SLOGDET_GRAD, SLOGPF_GRAD):
        outs.append(jax.ShapeDtypeStruct(a.shape, a.dtype))
    if ws:
        outs.append(jax.ShapeDtypeStruct((ws,), jnp.uint8))
    res = jax.ffi.ffi_call(register(), tuple(outs), vmap_method="broadcast_all",
                           legacy_backend_config=descriptor(op, dt, p, B, n, flags=flags, workspace_bytes=ws))(a)
    return res[:3] if op in (SLOGDET_GRAD, SLOGPF_GRAD) else res[:2]


def _slog(op_fwd, op_grad, flags):
    import functools

    import jax
    import jax.numpy as jnp

    @functools.partial(jax.custom_jvp, nondiff_argnums=(1,))
    def f(a, prec):
        return _call(op_fwd, a, prec, flags)

    def jvp(prec, primals, tangents):
        (a,), (da,) = primals, tangents
        sign, logabs, D = _call(op_grad, a, prec, flags)  # D = d logabs / d a (holomorphic)
        t = jnp.sum(D * da, axis=(-1, -2))
        dsign = (1j * jnp.imag(t)).astype(sign.dtype) * sign if jnp.iscomplexobj(a) else jnp.zeros_like(sign)
        return (sign, logabs), (dsign, jnp.real(t).astype(logabs.dtype))

    f.defjvp(jvp)
    return f


def slogdet(a, *, prec=None):
    """(sign, logabs) of a (..., n, n) JAX array on a CUDA device, as fermix.slogdet."""
    import jax.numpy as jnp

    batch, n = a.shape[:-2], a.shape[-1]
    s, l = _slog(SLOGDET, SLOGDET_GRAD, 0)(jnp.reshape(a, (-1, n, n)), prec)
    return jnp.reshape(s, batch), jnp.reshape(l, batch)


def slogpf(a, *, prec=None, skew_symmetrize=True):
    """(sign, logabs) of the Pfaffian of a (..., n, n) JAX array, as fermix.slogpf."""
    import jax.numpy as jnp

    batch, n = a.shape[:-2], a.shape[-1]
    s, l = _slog(SLOGPF, SLOGPF_GRAD, F_SKEW if skew_symmetrize else 0)(jnp.reshape(a, (-1, n, n)), prec)
    return jnp.reshape(s, batch), jnp.reshape(l, batch)
