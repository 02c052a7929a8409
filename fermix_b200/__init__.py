"""fermix_b200: batched determinants and Pfaffians (float32 / float64 / complex64 /
complex128) on NVIDIA B200, with singular-safe gradients -- a drop-in for the public API
of ChenAo-Phys/fermix (src/fermix/__init__.py:1-10) on torch CUDA tensors, computed by
hand-written sm_100a kernels behind a C ABI (include/fermix_b200.h).

Public functions: :func:`slogdet`, :func:`slogpf`, :func:`det`, :func:`pf`.
"""

from .api import (
    FermixFallbackWarning,
    det,
    det_parts,
    pf,
    pf_parts,
    slogdet,
    slogdet_gather,
    slogdet_ratio,
    slogdet_update,
    slogpf_ratio,
    slogpf_ratio_k,
    slogpf_update,
    slogpf_update_k,
    slogdet_parts,
    slogdet_planar,
    slogpf,
    slogpf_parts,
    slogpf_planar,
    det_planar,
    pf_planar,
)

__version__ = "0.1.0"
__all__ = [
    "slogdet",
    "slogpf",
    "det",
    "pf",
    "slogdet_parts",
    "slogpf_parts",
    "det_parts",
    "pf_parts",
    "slogdet_gather",
    "slogdet_ratio",
    "slogdet_update",
    "slogpf_ratio",
    "slogpf_update",
    "slogpf_ratio_k",
    "slogpf_update_k",
    "slogdet_planar",
    "slogpf_planar",
    "det_planar",
    "pf_planar",
    "FermixFallbackWarning",
    "__version__",
]
