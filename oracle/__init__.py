"""CPU oracle for the batched slogdet / slogpf / det / pf path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the ``fermix_b200`` package and its
CUDA library) imports, links or runs this package; only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` use it, and only
as the checker / the timed CPU reference.

``oracle.fallback`` restates the reference's generic (jax.numpy / LAPACK) path in numpy
and scipy; ``oracle.refs64`` restates the float64 / complex128 reference oracles of the
reference's own test suite, which pin the restatement (see ``tests/test_oracle.py``).
"""

from .fallback import (  # noqa: F401
    det,
    det_grad,
    lu_parts,
    pf,
    pf_grad,
    pf_parts,
    slogdet,
    slogdet_grad,
    slogpf,
    slogpf_grad,
)
