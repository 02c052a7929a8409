"""Shared helpers of the GPU parity tests."""

import numpy as np
import torch

DTYPES = [np.float32, np.float64, np.complex64, np.complex128]
IDS = ["f32", "f64", "c64", "c128"]
TORCH = {
    np.dtype(np.float32): torch.float32,
    np.dtype(np.float64): torch.float64,
    np.dtype(np.complex64): torch.complex64,
    np.dtype(np.complex128): torch.complex128,
}


def cuda(x, requires_grad=False):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    if requires_grad:
        t.requires_grad_(True)
    return t


def host(t):
    if isinstance(t, (tuple, list)):
        return type(t)(host(x) for x in t)
    return t.detach().cpu().numpy()


def jgrad(f, x):
    """The reference's ``grad_real_sum``: jax.grad of sum(Re f(x)). torch's gradient of a
    real loss w.r.t. a complex input is the conjugate of JAX's, so conjugate it back."""
    t = cuda(x, requires_grad=True)
    out = f(t)
    loss = torch.real(out).sum()
    (g,) = torch.autograd.grad(loss, t)
    g = host(g)
    return np.conj(g) if np.iscomplexobj(g) else g
