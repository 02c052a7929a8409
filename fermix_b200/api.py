"""Public API: slogdet, slogpf, det, pf -- the signatures, argument meanings, return
dtypes and errors of ChenAo-Phys/fermix's ``src/fermix/api.py:148-227``, on torch CUDA
tensors, computed by the hand-written sm_100a kernels of libfermix_b200.so.

Differences from the reference, which is JAX-only:

* inputs are torch tensors on a CUDA device (numpy arrays are copied to the current
  CUDA device); a CPU tensor raises -- there is no CPU fallback, so
  ``FermixFallbackWarning`` is exported for compatibility but never emitted;
* derivatives go through torch autograd (``backward``, ``torch.autograd.grad``),
  forward-mode AD (``torch.func.jvp`` via ``jvp``) and ``torch.func.vmap``. For complex
  inputs torch's gradient convention is the conjugate of JAX's: where the reference's
  ``jax.grad`` of ``sum(logabs)`` returns ``A^-T``, ``torch.autograd.grad`` returns
  ``conj(A^-T)`` (the same convention as ``torch.linalg.slogdet``). Tangents (jvp) are
  identical to the reference's.
* ``slogdet_parts`` / ``slogpf_parts`` / ``det_parts`` / ``pf_parts`` return the
  reference's (JAX-convention) derivative arrays directly -- the values of the reference's
  ``jax.grad`` -- together with the forward, from one kernel launch.
"""

import numpy as np
import torch

from . import _lib

_KIND = {
    torch.float32: _lib.FX_F32,
    torch.float64: _lib.FX_F64,
    torch.complex64: _lib.FX_C64,
    torch.complex128: _lib.FX_C128,
}
_PREC = {None: _lib.FX_PREC_DEFAULT, "tf32x3": _lib.FX_PREC_TF32X3, "ieee": _lib.FX_PREC_IEEE}


class FermixFallbackWarning(UserWarning):
    """Kept for API compatibility with the reference (src/fermix/api.py:19-21). This
    build has no fallback path: non-CUDA inputs raise instead, so it is never emitted."""


# ------------------------------------------------------------------ validation
def _prep(a, square=True):
    """dtype / shape checks of the reference's _prep (src/fermix/api.py:24-31); square=False
    only requires a matrix (the shared phi of slogdet_gather)."""
    from_host = False
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
        from_host = True
    elif not isinstance(a, torch.Tensor):
        a = torch.as_tensor(a)
        from_host = True
    if a.dtype not in _KIND:
        raise TypeError(f"fermix supports float32, float64, complex64 and complex128, got {a.dtype}")
    if a.ndim < 2 or (square and a.shape[-1] != a.shape[-2]):
        raise ValueError(f"expected (..., n, n), got {tuple(a.shape)}")
    if a.device.type != "cuda":
        if from_host and torch.cuda.is_available():
            return a.cuda()  # like jnp.asarray: host data goes to the default device
        raise RuntimeError(
            f"fermix_b200 runs on CUDA devices only (got a tensor on {a.device}); "
            "move it with .cuda() -- there is no CPU fallback"
        )
    return a


def _check_block(block):
    """src/fermix/api.py:92-97."""
    if block is not None and block not in (32, 64, 128):
        raise ValueError(f"block must be None, 32, 64 or 128, got {block!r}")
    return block


def _check_prec(dtype, prec):
    """Field.check_prec (src/fermix/_field.py:265-275)."""
    if prec not in _PREC:
        raise ValueError(f"prec must be 'tf32x3' or 'ieee', got {prec!r}")
    if prec == "tf32x3" and dtype in (torch.float64, torch.complex128):
        raise ValueError(
            "prec='tf32x3' applies to float32 / complex64 only; float64 and complex128 run "
            "their block updates in IEEE fp64 (prec='ieee')"
        )
    return _PREC[prec]


def _check_unroll(unroll_steps):
    if unroll_steps is not None and not isinstance(unroll_steps, (bool, int)):
        raise ValueError(f"unroll_steps must be None or a bool, got {unroll_steps!r}")


def _check_upd_warps(upd_warps):
    if upd_warps is not None and (not isinstance(upd_warps, int) or upd_warps < 1):
        raise ValueError(f"upd_warps must be None or a positive int, got {upd_warps!r}")


def _real(dtype):
    return torch.float32 if dtype in (torch.float32, torch.complex64) else torch.float64


# ------------------------------------------------------------------ library calls
def _stream_ptr(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _workspace(op, kind, B, n, grad, dev):
    nbytes = _lib.lib().fermix_workspace_bytes(op, kind, B, n, int(grad))
    if nbytes == 0:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=dev), nbytes


def _ptr(t):
    return None if t is None else t.data_ptr()


def _run(op, A, prec, *, skew=True, grad=False, coef=None, conj_out=False, adjugate=False, value=False):
    """One library call on the contiguous (B, n, n) CUDA tensor A: returns (sign,
    logabs, value or None, grad or None)."""
    L = _lib.lib()
    B, n = A.shape[0], A.shape[-1]
    kind = _KIND[A.dtype]
    dev = A.device
    sign = torch.empty(B, dtype=A.dtype, device=dev)
    logabs = torch.empty(B, dtype=_real(A.dtype), device=dev)
    val = torch.empty(B, dtype=A.dtype, device=dev) if value else None
    G = torch.empty_like(A) if grad else None
    if coef is not None:
        coef = coef.to(dtype=A.dtype, device=dev).contiguous()
    with torch.cuda.device(dev):
        ws, wsb = _workspace(op, kind, B, n, grad, dev)
        s = _stream_ptr(dev)
        if op == _lib.FX_OP_SLOGDET:
            if grad:
                st = L.fermix_slogdet_grad(s, kind, prec, B, n, _ptr(A), _ptr(coef), int(conj_out), int(adjugate),
                                           _ptr(sign), _ptr(logabs), _ptr(val), _ptr(G), _ptr(ws), wsb)
            else:
                st = L.fermix_slogdet(s, kind, prec, B, n, _ptr(A), _ptr(sign), _ptr(logabs), _ptr(val), _ptr(ws), wsb)
        else:
            if grad:
                st = L.fermix_slogpf_grad(s, kind, prec, B, n, int(skew), _ptr(A), _ptr(coef), int(conj_out),
                                          int(adjugate), _ptr(sign), _ptr(logabs), _ptr(val), _ptr(G), _ptr(ws), wsb)
            else:
                st = L.fermix_slogpf(s, kind, prec, B, n, int(skew), _ptr(A), _ptr(sign), _ptr(logabs), _ptr(val),
                                     _ptr(ws), wsb)
    _lib.check(st)
    return sign, logabs, val, G


def _run_gather(phi, occ, prec, *, grad=False, coef=None, conj_out=False):
    """fermix_slogdet_gather on phi (rows, cols) and occ (B, n) int32, both contiguous
    CUDA tensors: returns (sign, logabs, grad or None)."""
    L = _lib.lib()
    B, n = occ.shape
    kind = _KIND[phi.dtype]
    dev = phi.device
    sign = torch.empty(B, dtype=phi.dtype, device=dev)
    logabs = torch.empty(B, dtype=_real(phi.dtype), device=dev)
    G = torch.empty((B, n, n), dtype=phi.dtype, device=dev) if grad else None
    if coef is not None:
        coef = coef.to(dtype=phi.dtype, device=dev).contiguous()
    with torch.cuda.device(dev):
        nbytes = L.fermix_slogdet_gather_workspace_bytes(kind, prec, B, n, int(grad))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev) if nbytes else None
        st = L.fermix_slogdet_gather(_stream_ptr(dev), kind, prec, B, n, _ptr(phi), phi.shape[0], phi.shape[1],
                                     _ptr(occ), _ptr(coef), int(conj_out), _ptr(sign), _ptr(logabs), None, _ptr(G),
                                     _ptr(ws), nbytes)
    _lib.check(st)
    return sign, logabs, G


def _flat(a):
    batch = tuple(a.shape[:-2])
    n = a.shape[-1]
    B = int(np.prod(batch)) if batch else 1
    return a.reshape(B, n, n).contiguous(), batch, n


def _slog_coef(sign, g_sign, g_logabs, cplx):
    """Per-matrix coefficient c with torch grad = conj(c * D), D the holomorphic
    derivative of logabs: c = g_logabs + i Im(conj(g_sign) sign) (complex), g_logabs
    (real). The sign's tangent is i Im(tr) sign (src/fermix/_diff.py:92-97)."""
    if g_logabs is None:
        g_logabs = torch.zeros(sign.shape, dtype=_real(sign.dtype), device=sign.device)
    if not cplx:
        return g_logabs
    c = g_logabs.to(sign.dtype)
    if g_sign is not None:
        q = torch.imag(torch.conj(g_sign) * sign)
        c = c + 1j * q.to(sign.dtype)
    return c


# ------------------------------------------------------------------ autograd
def _fold(A, in_dim):
    """vmap helper: move the vmapped axis first and fold it into the batch."""
    A = A.movedim(in_dim, 0)
    V, rest, n = A.shape[0], tuple(A.shape[1:-2]), A.shape[-1]
    return A.reshape((-1, n, n)).contiguous(), V, rest


class _FwdKernel(torch.autograd.Function):
    """Non-differentiable forward launch: (sign, logabs, value) of a (B, n, n) batch."""

    @staticmethod
    def forward(A, op, prec, skew):
        sign, logabs, val, _ = _run(op, A, prec, skew=skew, value=True)
        return sign, logabs, val

    @staticmethod
    def setup_context(ctx, inputs, output):
        ctx.mark_non_differentiable(*output)

    @staticmethod
    def vmap(info, in_dims, A, op, prec, skew):
        if in_dims[0] is None:
            return _FwdKernel.apply(A, op, prec, skew), (None, None, None)
        X, V, rest = _fold(A, in_dims[0])
        out = _FwdKernel.apply(X, op, prec, skew)
        return tuple(o.reshape((V,) + rest) for o in out), (0, 0, 0)


class _GradKernel(torch.autograd.Function):
    """Non-differentiable gradient launch: G = coef * D (conjugated if conj_out) with D
    the derivative matrix of the op (A^-T, adj(A)^T, S^-T/2 or pf S^-T/2)."""

    @staticmethod
    def forward(A, coef, op, prec, skew, conj_out, adjugate):
        _, _, _, G = _run(op, A, prec, skew=skew, grad=True, coef=coef, conj_out=conj_out, adjugate=adjugate)
        return G

    @staticmethod
    def setup_context(ctx, inputs, output):
        ctx.mark_non_differentiable(output)

    @staticmethod
    def vmap(info, in_dims, A, coef, op, prec, skew, conj_out, adjugate):
        da, dc = in_dims[0], in_dims[1]
        if da is None and dc is None:
            return _GradKernel.apply(A, coef, op, prec, skew, conj_out, adjugate), None
        V = info.batch_size
        if da is None:
            A = A.unsqueeze(0).expand((V,) + tuple(A.shape))
            da = 0
        X, V, rest = _fold(A, da)
        if coef is not None:
            c = coef.movedim(dc, 0) if dc is not None else coef.unsqueeze(0).expand((V,) + tuple(coef.shape))
            c = c.reshape(-1).contiguous()
        else:
            c = None
        G = _GradKernel.apply(X, c, op, prec, skew, conj_out, adjugate)
        n = X.shape[-1]
        return G.reshape((V,) + rest + (n, n)), 0


# Derivative matrices (B, n, n) up to this many bytes are computed by the forward launch
# and kept for the backward, so that one factorisation serves both (the reference's rule,
# src/fermix/_diff.py:111-124). Larger ones are not kept: the backward factorises again,
# which holds no (B, n, n) residual between the passes.
KEEP_GRAD_BYTES = 8 << 30


def _keep(A):
    """Whether the forward should also produce the derivative matrix for the backward."""
    return (torch.is_grad_enabled() and A.requires_grad and
            A.numel() * A.element_size() <= KEEP_GRAD_BYTES)


def _scale_grad(D, c):
    """The gradient conj(c * D) from the kept derivative matrix D (torch's complex
    convention; the same product the kernels form when given coef and conj_out)."""
    G = c.to(D.dtype)[:, None, None] * D
    return torch.conj(G) if D.is_complex() else G


class _Slog(torch.autograd.Function):
    """(sign, logabs) of slogdet (op=SLOGDET) or slogpf (op=SLOGPF) on a (B, n, n)
    batch. With keep (the input requires grad and the derivative fits KEEP_GRAD_BYTES) the
    forward is one launch of the fused factorisation + gradient kernel, whose primal is
    bit-identical to the forward kernel's, and the backward scales the kept derivative;
    otherwise the backward re-runs the factorisation with the gradient epilogue."""

    @staticmethod
    def forward(A, op, prec, skew, keep):
        if keep:
            sign, logabs, _, D = _run(op, A, prec, skew=skew, grad=True)
            return sign, logabs, D
        sign, logabs, _ = _FwdKernel.apply(A, op, prec, skew)
        return sign, logabs, None

    @staticmethod
    def setup_context(ctx, inputs, output):
        A, op, prec, skew, keep = inputs
        D = output[2]
        if D is not None:
            ctx.mark_non_differentiable(D)
        ctx.save_for_backward(A, output[0], D)
        ctx.save_for_forward(A, output[0], D)
        ctx.op, ctx.prec, ctx.skew = op, prec, skew

    @staticmethod
    def backward(ctx, g_sign, g_logabs, _g_d):
        A, sign, D = ctx.saved_tensors
        c = _slog_coef(sign, g_sign, g_logabs, A.is_complex())
        if D is not None:
            return _scale_grad(D, c), None, None, None, None
        G = _GradKernel.apply(A, c, ctx.op, ctx.prec, ctx.skew, True, False)
        return G, None, None, None, None

    @staticmethod
    def jvp(ctx, dA, *_):
        A, sign, D = ctx.saved_tensors
        if D is None:
            D = _GradKernel.apply(A, None, ctx.op, ctx.prec, ctx.skew, False, False)
        t = (D * dA).sum(dim=(-1, -2))
        if A.is_complex():
            return (1j * t.imag).to(sign.dtype) * sign, t.real, None
        return torch.zeros_like(sign), t, None

    @staticmethod
    def vmap(info, in_dims, A, op, prec, skew, keep):
        if in_dims[0] is None:
            return _Slog.apply(A, op, prec, skew, keep), (None, None, None)
        X, V, rest = _fold(A, in_dims[0])
        s, l, D = _Slog.apply(X, op, prec, skew, keep)
        n = X.shape[-1]
        out = (s.reshape((V,) + rest), l.reshape((V,) + rest), None if D is None else D.reshape((V,) + rest + (n, n)))
        return out, (0, 0, None if D is None else 0)


class _Value(torch.autograd.Function):
    """det (op=SLOGDET) or pf (op=SLOGPF) value on a (B, n, n) batch, with the
    singular-safe adjugate gradient (kept from the forward launch under the same rule as
    _Slog)."""

    @staticmethod
    def forward(A, op, prec, skew, keep):
        if keep:
            _, _, val, D = _run(op, A, prec, skew=skew, grad=True, adjugate=True, value=True)
            return val, D
        return _FwdKernel.apply(A, op, prec, skew)[2], None

    @staticmethod
    def setup_context(ctx, inputs, output):
        A, op, prec, skew, keep = inputs
        D = output[1]
        if D is not None:
            ctx.mark_non_differentiable(D)
        ctx.save_for_backward(A, D)
        ctx.save_for_forward(A, D)
        ctx.op, ctx.prec, ctx.skew = op, prec, skew

    @staticmethod
    def backward(ctx, g, _g_d):
        A, D = ctx.saved_tensors
        c = torch.conj(g) if A.is_complex() else g
        if D is not None:
            return _scale_grad(D, c), None, None, None, None
        G = _GradKernel.apply(A, c, ctx.op, ctx.prec, ctx.skew, True, True)
        return G, None, None, None, None

    @staticmethod
    def jvp(ctx, dA, *_):
        A, D = ctx.saved_tensors
        if D is None:
            D = _GradKernel.apply(A, None, ctx.op, ctx.prec, ctx.skew, False, True)
        return (D * dA).sum(dim=(-1, -2)), None

    @staticmethod
    def vmap(info, in_dims, A, op, prec, skew, keep):
        if in_dims[0] is None:
            return _Value.apply(A, op, prec, skew, keep), (None, None)
        X, V, rest = _fold(A, in_dims[0])
        v, D = _Value.apply(X, op, prec, skew, keep)
        n = X.shape[-1]
        return (v.reshape((V,) + rest), None if D is None else D.reshape((V,) + rest + (n, n))), (0, None if D is None else 0)


# ------------------------------------------------------------------ public functions
class _SlogGather(torch.autograd.Function):
    """(sign, logabs) of the matrices phi[occ[b]] (rows of a shared phi), differentiable
    in phi: the backward runs the gathered gradient kernel and adds each matrix's rows
    of coef * A^-T into the phi rows they came from."""

    @staticmethod
    def forward(phi, occ, prec):
        sign, logabs, _ = _run_gather(phi, occ, prec)
        return sign, logabs

    @staticmethod
    def setup_context(ctx, inputs, output):
        phi, occ, prec = inputs
        ctx.save_for_backward(phi, occ, output[0])
        ctx.prec = prec
        ctx.mark_non_differentiable(output[0])

    @staticmethod
    def backward(ctx, g_sign, g_logabs):
        phi, occ, sign = ctx.saved_tensors
        c = _slog_coef(sign, g_sign, g_logabs, phi.is_complex())
        _, _, G = _run_gather(phi, occ, ctx.prec, grad=True, coef=c, conj_out=True)
        B, n = occ.shape
        rows = torch.zeros((phi.shape[0], n), dtype=phi.dtype, device=phi.device)
        rows.index_add_(0, occ.reshape(-1).long(), G.reshape(B * n, n))
        dphi = torch.zeros_like(phi)
        dphi[:, :n] = rows
        return dphi, None, None


def slogdet_gather(phi, occ, *, prec=None):
    """slogdet of the matrices whose rows are gathered from a shared ``phi``: matrix
    ``b`` is ``phi[occ[b, :], :n]`` with n = occ.shape[-1] (the QMC pattern of an orbital
    matrix and electron occupations), without materialising the batch. ``phi`` is a 2-D
    CUDA tensor (rows, cols >= n), ``occ`` an integer tensor of shape (..., n). Returns
    (sign, logabs) of shape occ.shape[:-1], equal to ``slogdet(phi[occ][..., :n])`` bit for
    bit and differentiable in ``phi``. An index outside [0, rows) makes that member NaN
    (and is not allowed when differentiating)."""
    phi = _prep(phi, square=False)
    if phi.dim() != 2:
        raise ValueError("phi must be a 2-D tensor (rows, cols)")
    if not isinstance(occ, torch.Tensor):
        occ = torch.as_tensor(np.asarray(occ))
    if occ.dtype not in (torch.int32, torch.int64, torch.int16, torch.uint8):
        raise TypeError("occ must be an integer tensor")
    if occ.dim() < 1:
        raise ValueError("occ must have shape (..., n)")
    n = occ.shape[-1]
    if phi.shape[1] < n:
        raise ValueError(f"phi has {phi.shape[1]} columns, fewer than n = {n}")
    batch = tuple(occ.shape[:-1])
    p = _check_prec(phi.dtype, prec)
    O = occ.to(device=phi.device, dtype=torch.int32).reshape(-1, n).contiguous()
    sign, logabs = _SlogGather.apply(phi.contiguous(), O, p)
    return sign.reshape(batch), logabs.reshape(batch)


def _move_args(g, rows, idx):
    """Checks of the rank-k move functions: g (..., n, n), rows (..., k, n), idx (..., k)."""
    g = _prep(g)
    n = g.shape[-1]
    batch = tuple(g.shape[:-2])
    rows = torch.as_tensor(rows, device=g.device)
    if rows.dtype != g.dtype:
        raise TypeError(f"rows must have the dtype of g ({g.dtype}), got {rows.dtype}")
    if rows.dim() < 2 or rows.shape[-1] != n or tuple(rows.shape[:-2]) != batch:
        raise ValueError(f"rows must have shape {batch + ('k', n)}, got {tuple(rows.shape)}")
    k = rows.shape[-2]
    if k > 16 or k > n:
        raise ValueError(f"a move replaces at most min(16, n) rows, got k = {k}")
    if not isinstance(idx, torch.Tensor):
        idx = torch.as_tensor(np.asarray(idx))
    if idx.dtype not in (torch.int32, torch.int64, torch.int16, torch.uint8):
        raise TypeError("idx must be an integer tensor")
    if tuple(idx.shape) != batch + (k,):
        raise ValueError(f"idx must have shape {batch + (k,)}, got {tuple(idx.shape)}")
    B = int(np.prod(batch)) if batch else 1
    U = rows.detach().reshape(B, k, n).contiguous()
    I = idx.to(device=g.device, dtype=torch.int32).reshape(B, k).contiguous()
    return g, U, I, batch, B, n, k


def slogdet_ratio(g, rows, idx):
    """Determinant ratio of a k-row move (no reference counterpart: the single- and
    multi-electron moves of a QMC caller). ``g`` (..., n, n) holds A^-T -- the gradient
    ``slogdet_parts`` returns -- ``rows`` (..., k, n) the new rows and ``idx`` (..., k)
    the distinct rows of A they replace, k <= min(16, n). Returns (sign, logabs) of
    det(A') / det(A) = det(U A^-1 E) in the slogdet conventions; reads only k rows of each
    g."""
    g, U, I, batch, B, n, k = _move_args(g, rows, idx)
    G = g.detach().reshape(B, n, n).contiguous()
    sign = torch.empty(B, dtype=g.dtype, device=g.device)
    logabs = torch.empty(B, dtype=_real(g.dtype), device=g.device)
    with torch.cuda.device(g.device):
        st = _lib.lib().fermix_slogdet_ratio(_stream_ptr(g.device), _KIND[g.dtype], B, n, k, _ptr(G), _ptr(U),
                                             _ptr(I), _ptr(sign), _ptr(logabs))
    _lib.check(st)
    return sign.reshape(batch), logabs.reshape(batch)


def slogdet_update(g, rows, idx, *, accept=None, inplace=False):
    """Apply a k-row move to the inverse: as ``slogdet_ratio``, and also the new
    A'^-T by the Woodbury identity for the members where ``accept`` (bool, shape
    g.shape[:-2]; None = all) is true; the others keep g. A member whose ratio is exactly
    0 gets a zero matrix (the slogdet gradient convention for a singular matrix). Returns
    (sign, logabs, g_new); with ``inplace=True`` g (a contiguous CUDA tensor) is updated
    and returned. Not differentiable."""
    g, U, I, batch, B, n, k = _move_args(g, rows, idx)
    if inplace:
        if not g.is_contiguous():
            raise ValueError("inplace=True needs a contiguous g")
        G = g.detach().view(B, n, n)
    else:
        G = g.detach().reshape(B, n, n).clone()
    acc = None
    if accept is not None:
        acc = torch.as_tensor(accept, device=g.device)
        if tuple(acc.shape) != batch:
            raise ValueError(f"accept must have shape {batch}, got {tuple(acc.shape)}")
        acc = acc.to(torch.uint8).reshape(B).contiguous()
    sign = torch.empty(B, dtype=g.dtype, device=g.device)
    logabs = torch.empty(B, dtype=_real(g.dtype), device=g.device)
    L = _lib.lib()
    kind = _KIND[g.dtype]
    with torch.cuda.device(g.device):
        nbytes = L.fermix_slogdet_update_workspace_bytes(kind, B, n, k)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=g.device) if nbytes else None
        st = L.fermix_slogdet_update(_stream_ptr(g.device), kind, B, n, k, _ptr(G), _ptr(U), _ptr(I), _ptr(acc),
                                     _ptr(sign), _ptr(logabs), _ptr(ws), nbytes)
    _lib.check(st)
    return sign.reshape(batch), logabs.reshape(batch), (g if inplace else G.reshape(g.shape))


def _pf_move_args(g, row, idx):
    """Checks of the Pfaffian move functions: g (..., n, n), row (..., n), idx (...)."""
    g = _prep(g)
    n = g.shape[-1]
    if n < 2:
        raise ValueError("a Pfaffian move needs n >= 2")
    batch = tuple(g.shape[:-2])
    row = torch.as_tensor(row, device=g.device)
    if row.dtype != g.dtype:
        raise TypeError(f"row must have the dtype of g ({g.dtype}), got {row.dtype}")
    if tuple(row.shape) != batch + (n,):
        raise ValueError(f"row must have shape {batch + (n,)}, got {tuple(row.shape)}")
    if not isinstance(idx, torch.Tensor):
        idx = torch.as_tensor(np.asarray(idx))
    if idx.dtype not in (torch.int32, torch.int64, torch.int16, torch.uint8):
        raise TypeError("idx must be an integer tensor")
    if tuple(idx.shape) != batch:
        raise ValueError(f"idx must have shape {batch}, got {tuple(idx.shape)}")
    B = int(np.prod(batch)) if batch else 1
    U = row.detach().reshape(B, n).contiguous()
    I = idx.to(device=g.device, dtype=torch.int32).reshape(B).contiguous()
    return g, U, I, batch, B, n


def slogpf_ratio(g, row, idx):
    """Pfaffian ratio of a one-index move (no reference counterpart: the one-electron move
    of a Pfaffian wavefunction). ``g`` (..., n, n) holds S^-T / 2 -- the gradient
    ``slogpf_parts`` returns -- and the move replaces row ``idx`` of the skew S by ``row``
    (..., n) and column ``idx`` by -row (row[idx] is ignored). Returns (sign, logabs) of
    pf(S') / pf(S) = 2 g[idx] . row in the slogpf conventions; reads one row of each g."""
    g, U, I, batch, B, n = _pf_move_args(g, row, idx)
    G = g.detach().reshape(B, n, n).contiguous()
    sign = torch.empty(B, dtype=g.dtype, device=g.device)
    logabs = torch.empty(B, dtype=_real(g.dtype), device=g.device)
    with torch.cuda.device(g.device):
        st = _lib.lib().fermix_slogpf_ratio(_stream_ptr(g.device), _KIND[g.dtype], B, n, _ptr(G), _ptr(U), _ptr(I),
                                            _ptr(sign), _ptr(logabs))
    _lib.check(st)
    return sign.reshape(batch), logabs.reshape(batch)


def slogpf_update(g, row, idx, *, accept=None, inplace=False):
    """Apply a one-index Pfaffian move to the gradient: as ``slogpf_ratio``, and also
    g <- S'^-T / 2 (rank-2 skew Woodbury) where ``accept`` (bool, shape g.shape[:-2]; None =
    all) is true; the others keep g. A member whose ratio is exactly 0 gets a zero matrix.
    Returns (sign, logabs, g_new); with ``inplace=True`` g (a contiguous CUDA tensor) is
    updated and returned. Not differentiable."""
    g, U, I, batch, B, n = _pf_move_args(g, row, idx)
    if inplace:
        if not g.is_contiguous():
            raise ValueError("inplace=True needs a contiguous g")
        G = g.detach().view(B, n, n)
    else:
        G = g.detach().reshape(B, n, n).clone()
    acc = None
    if accept is not None:
        acc = torch.as_tensor(accept, device=g.device)
        if tuple(acc.shape) != batch:
            raise ValueError(f"accept must have shape {batch}, got {tuple(acc.shape)}")
        acc = acc.to(torch.uint8).reshape(B).contiguous()
    sign = torch.empty(B, dtype=g.dtype, device=g.device)
    logabs = torch.empty(B, dtype=_real(g.dtype), device=g.device)
    L = _lib.lib()
    kind = _KIND[g.dtype]
    with torch.cuda.device(g.device):
        nbytes = L.fermix_slogpf_update_workspace_bytes(kind, B, n)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=g.device) if nbytes else None
        st = L.fermix_slogpf_update(_stream_ptr(g.device), kind, B, n, _ptr(G), _ptr(U), _ptr(I), _ptr(acc),
                                    _ptr(sign), _ptr(logabs), _ptr(ws), nbytes)
    _lib.check(st)
    return sign.reshape(batch), logabs.reshape(batch), (g if inplace else G.reshape(g.shape))


def _pf_move_k_args(g, rows, idx):
    """Checks of the k-index Pfaffian move functions: g (..., n, n), rows (..., k, n), idx (..., k)."""
    g, U, I, batch, B, n, k = _move_args(g, rows, idx)
    if n < 2:
        raise ValueError("a Pfaffian move needs n >= 2")
    return g, U, I, batch, B, n, k


def slogpf_ratio_k(g, rows, idx):
    """Pfaffian ratio of a k-index move (no reference counterpart: the multi-electron move
    of a Pfaffian wavefunction). ``g`` (..., n, n) holds S^-T / 2 -- the gradient
    ``slogpf_parts`` returns -- and the move replaces rows ``idx`` (..., k) of the skew S by
    ``rows`` (..., k, n) and the same columns by -rows, applied in order (k one-index moves;
    on the idx x idx block the later row wins). Returns (sign, logabs) of pf(S') / pf(S) in
    the slogpf conventions; reads all of each g once."""
    g, U, I, batch, B, n, k = _pf_move_k_args(g, rows, idx)
    G = g.detach().reshape(B, n, n).contiguous()
    sign = torch.empty(B, dtype=g.dtype, device=g.device)
    logabs = torch.empty(B, dtype=_real(g.dtype), device=g.device)
    L = _lib.lib()
    kind = _KIND[g.dtype]
    with torch.cuda.device(g.device):
        nb = L.fermix_slogpf_move_k_workspace_bytes(kind, B, n, k)
        ws = torch.empty(nb, dtype=torch.uint8, device=g.device) if nb else None
        st = L.fermix_slogpf_ratio_k(_stream_ptr(g.device), kind, B, n, k, _ptr(G), _ptr(U), _ptr(I), _ptr(sign),
                                     _ptr(logabs), _ptr(ws), nb)
    _lib.check(st)
    return sign.reshape(batch), logabs.reshape(batch)


def slogpf_update_k(g, rows, idx, *, accept=None, inplace=False):
    """Apply a k-index Pfaffian move to the gradient: as ``slogpf_ratio_k``, and also
    g <- S'^-T / 2 where ``accept`` (bool, shape g.shape[:-2]; None = all) is true; the
    others keep g. A member whose ratio is exactly 0 gets a zero matrix. Returns
    (sign, logabs, g_new); with ``inplace=True`` g (a contiguous CUDA tensor) is updated
    and returned. Not differentiable."""
    g, U, I, batch, B, n, k = _pf_move_k_args(g, rows, idx)
    if inplace:
        if not g.is_contiguous():
            raise ValueError("inplace=True needs a contiguous g")
        G = g.detach().view(B, n, n)
    else:
        G = g.detach().reshape(B, n, n).clone()
    acc = None
    if accept is not None:
        acc = torch.as_tensor(accept, device=g.device)
        if tuple(acc.shape) != batch:
            raise ValueError(f"accept must have shape {batch}, got {tuple(acc.shape)}")
        acc = acc.to(torch.uint8).reshape(B).contiguous()
    sign = torch.empty(B, dtype=g.dtype, device=g.device)
    logabs = torch.empty(B, dtype=_real(g.dtype), device=g.device)
    L = _lib.lib()
    kind = _KIND[g.dtype]
    with torch.cuda.device(g.device):
        nb = L.fermix_slogpf_move_k_workspace_bytes(kind, B, n, k)
        ws = torch.empty(nb, dtype=torch.uint8, device=g.device) if nb else None
        st = L.fermix_slogpf_update_k(_stream_ptr(g.device), kind, B, n, k, _ptr(G), _ptr(U), _ptr(I), _ptr(acc),
                                      _ptr(sign), _ptr(logabs), _ptr(ws), nb)
    _lib.check(st)
    return sign.reshape(batch), logabs.reshape(batch), (g if inplace else G.reshape(g.shape))


def slogdet(a, *, prec=None, unroll_steps=None, block=None):
    """Sign and log|det| of a batch of matrices ``a`` of shape (..., n, n)
    (src/fermix/api.py:148-174). Returns (sign, logabsdet): sign has the dtype of ``a``
    (exactly +-1 / 0 for real dtypes, a unit complex number for complex ones),
    logabsdet the corresponding real dtype -- the conventions of
    ``jnp.linalg.slogdet``. Exactly singular matrices give (0, -inf) and a zero
    gradient. ``prec`` ("tf32x3" | "ieee"; "tf32x3" only for float32 / complex64) is
    validated as in the reference: "tf32x3" on float32 with 8 <= n <= 256 runs the
    tensor-core kernels (3 TF32 products per update, fp32 accumulation), every other
    case IEEE FMA. ``block`` (None, 32, 64, 128) and ``unroll_steps`` are validated
    launch hints."""
    a = _prep(a)
    _check_block(block)
    _check_unroll(unroll_steps)
    p = _check_prec(a.dtype, prec)
    A, batch, n = _flat(a)
    sign, logabs, _ = _Slog.apply(A, _lib.FX_OP_SLOGDET, p, True, _keep(a))
    return sign.reshape(batch), logabs.reshape(batch)


def slogpf(a, *, prec=None, skew_symmetrize=True, upd_warps=None):
    """Sign and log|pf| of a batch of skew-symmetric matrices (S^T = -S, also for
    complex dtypes; odd n gives (0, -inf)) (src/fermix/api.py:177-193). The input is
    skew-symmetrised as (a - a^T)/2 unless ``skew_symmetrize=False`` (then it must be
    exactly skew-symmetric). Gradient: S^-T / 2 (skew), zero for an exactly singular S."""
    a = _prep(a)
    _check_upd_warps(upd_warps)
    p = _check_prec(a.dtype, prec)
    A, batch, n = _flat(a)
    sign, logabs, _ = _Slog.apply(A, _lib.FX_OP_SLOGPF, p, bool(skew_symmetrize), _keep(a))
    return sign.reshape(batch), logabs.reshape(batch)


def det(a, *, prec=None, unroll_steps=None, block=None):
    """Determinant of a batch of matrices (src/fermix/api.py:196-212); differentiable
    with d det = tr(adj(A) dA), finite and exact for singular A of rank n-1 (up to two
    exact zero pivots) and zero for rank <= n-2."""
    a = _prep(a)
    _check_block(block)
    _check_unroll(unroll_steps)
    p = _check_prec(a.dtype, prec)
    A, batch, n = _flat(a)
    return _Value.apply(A, _lib.FX_OP_SLOGDET, p, True, _keep(a))[0].reshape(batch)


def pf(a, *, prec=None, skew_symmetrize=True, upd_warps=None):
    """Pfaffian of a batch of skew-symmetric matrices (src/fermix/api.py:215-227); odd n
    gives 0. Differentiable with d pf = sum(G dS), G = pf S^-T / 2 continued to singular
    S (rank n-2: the rank-2 Pfaffian adjugate; rank <= n-4: 0)."""
    a = _prep(a)
    _check_upd_warps(upd_warps)
    p = _check_prec(a.dtype, prec)
    A, batch, n = _flat(a)
    return _Value.apply(A, _lib.FX_OP_SLOGPF, p, bool(skew_symmetrize), _keep(a))[0].reshape(batch)


# ------------------------------------------------------------------ one-launch parts
def _parts(op, a, prec, skew, adjugate, coef):
    a = _prep(a)
    p = _check_prec(a.dtype, prec)
    A, batch, n = _flat(a)
    if coef is not None:
        coef = torch.as_tensor(coef, device=A.device).reshape(-1)
    sign, logabs, val, G = _run(op, A, p, skew=skew, grad=True, coef=coef, adjugate=adjugate, value=adjugate)
    shape = batch + (n, n)
    if adjugate:
        return val.reshape(batch), G.reshape(shape)
    return sign.reshape(batch), logabs.reshape(batch), G.reshape(shape)


def slogdet_parts(a, *, prec=None, coef=None):
    """(sign, logabs, G) from one launch, G = coef * A^-T (the reference's jax.grad of
    sum(logabs); zero for exactly singular members)."""
    return _parts(_lib.FX_OP_SLOGDET, a, prec, True, False, coef)


def slogpf_parts(a, *, prec=None, skew_symmetrize=True, coef=None):
    """(sign, logabs, G) from one launch, G = coef * S^-T / 2 (the reference's jax.grad
    of sum(logabs) w.r.t. a)."""
    return _parts(_lib.FX_OP_SLOGPF, a, prec, skew_symmetrize, False, coef)


def det_parts(a, *, prec=None, coef=None):
    """(det, G) from one launch, G = coef * adj(A)^T (the reference's jax.grad of
    sum(Re det))."""
    return _parts(_lib.FX_OP_SLOGDET, a, prec, True, True, coef)


def pf_parts(a, *, prec=None, skew_symmetrize=True, coef=None):
    """(pf, G) from one launch, G = coef * pf(S) S^-T / 2 (the reference's jax.grad of
    sum(Re pf))."""
    return _parts(_lib.FX_OP_SLOGPF, a, prec, skew_symmetrize, True, coef)


# ------------------------------------------------------------------ split planes
def _planar(op, a_re, a_im, prec, skew, grad, adjugate, coef):
    a_re, a_im = _prep(a_re), _prep(a_im)
    if a_re.dtype not in (torch.float32, torch.float64) or a_im.dtype != a_re.dtype:
        raise TypeError("a_re and a_im must both be float32 (complex64) or both float64 (complex128)")
    if a_re.shape != a_im.shape or a_re.device != a_im.device:
        raise ValueError("a_re and a_im must have the same shape and device")
    cdt = torch.complex64 if a_re.dtype == torch.float32 else torch.complex128
    p = _check_prec(cdt, prec)
    re, batch, n = _flat(a_re)
    im, _, _ = _flat(a_im)
    B, dev, kind = re.shape[0], re.device, _KIND[cdt]
    L = _lib.lib()
    sign = torch.empty(B, dtype=cdt, device=dev)
    logabs = torch.empty(B, dtype=a_re.dtype, device=dev)
    val = torch.empty(B, dtype=cdt, device=dev) if adjugate else None
    g_re = torch.empty_like(re) if grad else None
    g_im = torch.empty_like(im) if grad else None
    if coef is not None:
        coef = torch.as_tensor(coef, device=dev).to(cdt).reshape(-1).contiguous()
    with torch.cuda.device(dev):
        nb = L.fermix_workspace_bytes_planar(op, kind, B, n, int(grad))
        ws = torch.empty(nb, dtype=torch.uint8, device=dev) if nb else None
        s = _stream_ptr(dev)
        if op == _lib.FX_OP_SLOGDET:
            st = (L.fermix_slogdet_grad_planar(s, kind, p, B, n, _ptr(re), _ptr(im), _ptr(coef), 0, int(adjugate),
                                               _ptr(sign), _ptr(logabs), _ptr(val), _ptr(g_re), _ptr(g_im), _ptr(ws), nb)
                  if grad else
                  L.fermix_slogdet_planar(s, kind, p, B, n, _ptr(re), _ptr(im), _ptr(sign), _ptr(logabs), _ptr(val),
                                          _ptr(ws), nb))
        else:
            st = (L.fermix_slogpf_grad_planar(s, kind, p, B, n, int(skew), _ptr(re), _ptr(im), _ptr(coef), 0,
                                              int(adjugate), _ptr(sign), _ptr(logabs), _ptr(val), _ptr(g_re),
                                              _ptr(g_im), _ptr(ws), nb)
                  if grad else
                  L.fermix_slogpf_planar(s, kind, p, B, n, int(skew), _ptr(re), _ptr(im), _ptr(sign), _ptr(logabs),
                                         _ptr(val), _ptr(ws), nb))
    _lib.check(st)
    shape = batch + (n, n)
    out = (sign.reshape(batch), logabs.reshape(batch))
    if adjugate:
        out = (val.reshape(batch),)
    if grad:
        out = out + (g_re.reshape(shape), g_im.reshape(shape))
    return out


def slogdet_planar(a_re, a_im, *, prec=None, grad=False, coef=None):
    """slogdet of complex matrices given as split real and imaginary planes a_re, a_im
    (float32 for complex64, float64 for complex128; shape (..., n, n)). Returns (sign,
    logabs), plus (g_re, g_im) -- the planes of coef * A^-T, the reference's jax.grad of
    sum(logabs) -- when grad. Equal bit for bit to slogdet / slogdet_parts on a_re + i a_im;
    for n > 256 the kernels read and write the planes directly. Not differentiable."""
    return _planar(_lib.FX_OP_SLOGDET, a_re, a_im, prec, True, grad, False, coef)


def slogpf_planar(a_re, a_im, *, prec=None, skew_symmetrize=True, grad=False, coef=None):
    """slogpf of complex skew matrices given as split real and imaginary planes (see
    slogdet_planar); the gradient planes are those of coef * S^-T / 2."""
    return _planar(_lib.FX_OP_SLOGPF, a_re, a_im, prec, skew_symmetrize, grad, False, coef)


def det_planar(a_re, a_im, *, prec=None, grad=False, coef=None):
    """det of complex matrices given as split planes: (det,) plus the planes of
    coef * adj(A)^T when grad."""
    return _planar(_lib.FX_OP_SLOGDET, a_re, a_im, prec, True, grad, True, coef)


def pf_planar(a_re, a_im, *, prec=None, skew_symmetrize=True, grad=False, coef=None):
    """pf of complex skew matrices given as split planes: (pf,) plus the planes of
    coef * pf(S) S^-T / 2 when grad."""
    return _planar(_lib.FX_OP_SLOGPF, a_re, a_im, prec, skew_symmetrize, grad, True, coef)
