"""The fused gather-slogdet (the QMC caller step of configuration C3): slogdet of rows of
a shared orbital matrix phi picked by occupations, against slogdet of the materialised
batch (bit for bit) and its phi gradient against the scattered per-matrix gradients."""

import numpy as np
import pytest
import torch

import fermix_b200 as fx
from oracle.refs64 import randn
from tests.helpers import DTYPES, IDS, host

pytestmark = pytest.mark.gpu


def _occ(gen, batch, sites, n):
    return np.stack([np.sort(gen.choice(sites, n, replace=False)) for _ in range(batch)]).astype(np.int32)


@pytest.mark.parametrize("dtype", DTYPES, ids=IDS)
@pytest.mark.parametrize("n", [64, 256, 300])
def test_gather_matches_materialised(dtype, n):
    gen = np.random.default_rng(31 + n)
    sites = 2 * n
    phi = (randn((sites, n), dtype, gen) / np.sqrt(n)).astype(dtype)
    occ = _occ(gen, 6, sites, n)
    occ[2, 5] = occ[2, 9]  # a duplicated row: exactly singular
    P = torch.from_numpy(phi).cuda()
    O = torch.from_numpy(occ).cuda()
    s, l = host(fx.slogdet_gather(P, O))
    A = torch.from_numpy(np.ascontiguousarray(phi[occ])).cuda()
    s2, l2 = host(fx.slogdet(A))
    assert np.array_equal(s, s2) and np.array_equal(l, l2)
    assert s[2] == 0 and l[2] == -np.inf


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["f32", "f64"])
def test_gather_phi_gradient(dtype):
    gen = np.random.default_rng(7)
    n, sites = 128, 200
    phi = (randn((sites, n + 3), dtype, gen) / np.sqrt(n) + 0.0).astype(dtype)
    occ = _occ(gen, 5, sites, n)
    P = torch.from_numpy(phi).cuda().requires_grad_(True)
    O = torch.from_numpy(occ).cuda()
    _, l = fx.slogdet_gather(P, O)
    (g,) = torch.autograd.grad(l.sum(), P)
    g = host(g)
    # reference: per-matrix A^-T rows scattered back into phi's rows (first n columns)
    want = np.zeros_like(phi, dtype=np.float64)
    for b in range(occ.shape[0]):
        A = phi[occ[b], :n].astype(np.float64)
        np.add.at(want, (occ[b][:, None], np.arange(n)[None, :]), np.linalg.inv(A).T)
    err = np.abs(g - want).max() / np.abs(want).max()
    assert err < (2e-3 if dtype == np.float32 else 1e-9)
    assert not np.any(g[:, n:])


def test_gather_bad_index_gives_nan_and_shape_errors():
    gen = np.random.default_rng(3)
    phi = torch.from_numpy(randn((40, 32), np.float32, gen)).cuda()
    occ = torch.arange(32, dtype=torch.int32, device="cuda").reshape(1, 32).repeat(2, 1)
    occ[1, 4] = 99
    s, l = host(fx.slogdet_gather(phi, occ))
    assert np.isfinite(l[0]) and np.isnan(l[1])
    with pytest.raises(ValueError):
        fx.slogdet_gather(phi[:, :16], occ)
    with pytest.raises(TypeError):
        fx.slogdet_gather(phi, occ.float())
