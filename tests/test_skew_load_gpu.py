"""skew_symmetrize=True on a general (not skew) float32 input equals the same call on
S = (A - A^T) / 2 formed beforehand, bit for bit, for the tensor-memory Parlett-Reid's two
input paths: 32-row chunks staged in shared memory by bulk copies (n % 4 == 0, 16-byte
aligned input) and direct loads (any other n or alignment). The reference skew-symmetrises
as (a - a^T) * 0.5 (src/fermix/api.py:177-193)."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx
import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prec", ["tf32x3", "ieee"])
@pytest.mark.parametrize("n", [8, 12, 32, 34, 64, 100, 126, 128])
def test_skew_symmetrize_matches_preformed_skew(n, prec):
    g = torch.Generator(device="cuda").manual_seed(1000 + n)
    A = torch.randn(9, n, n, device="cuda", generator=g)
    S = ((A - A.transpose(-1, -2)) * 0.5).contiguous()
    s1, l1, G1 = fx.slogpf_parts(A, prec=prec)
    s2, l2, G2 = fx.slogpf_parts(S, prec=prec, skew_symmetrize=False)
    assert torch.equal(s1, s2) and torch.equal(l1, l2) and torch.equal(G1, G2)
    f1 = fx.slogpf(A, prec=prec)
    assert torch.equal(f1[0], s1) and torch.equal(f1[1], l1)
    # against the float64 restatement of the reference's path on the same input: logabs
    # within 1e-4 max(1, |logabs|), or 2 cond(S) eps32 for an ill-conditioned member
    S64 = S.cpu().numpy().astype(np.float64)
    so, lo = oracle.slogpf(A.cpu().numpy().astype(np.float64))
    assert np.array_equal(s1.cpu().numpy(), so.astype(np.float32))
    err = np.abs(l1.cpu().numpy() - lo)
    for i in range(len(err)):
        lim = max(1e-4 * max(1.0, abs(lo[i])), 2 * np.linalg.cond(S64[i]) * np.finfo(np.float32).eps)
        assert err[i] <= lim, (i, err[i], lim)


def test_skew_symmetrize_unaligned_input():
    """A matrix batch starting 4 bytes into its buffer takes the direct-load path."""
    n = 64
    g = torch.Generator(device="cuda").manual_seed(77)
    buf = torch.randn(5 * n * n + 1, device="cuda", generator=g)
    A = buf[1:].view(5, n, n)
    assert A.data_ptr() % 16 != 0
    S = ((A - A.transpose(-1, -2)) * 0.5).contiguous()
    s1, l1 = fx.slogpf(A)
    s2, l2 = fx.slogpf(S, skew_symmetrize=False)
    assert torch.equal(s1, s2) and torch.equal(l1, l2)
