"""The tensor-core building blocks (tcgen05 MMA into tensor memory, shared-memory operand
descriptors, 3xTF32 split) against a float64 product: D = C +- A B^T at 128 x 128 x 16."""

import ctypes

import numpy as np
import pytest
import torch

from fermix_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("negate", [0, 1])
def test_umma_3xtf32_update(negate):
    g = np.random.default_rng(7 + negate)
    A = g.standard_normal((128, 16)).astype(np.float32)
    B = g.standard_normal((128, 16)).astype(np.float32)
    C = g.standard_normal((128, 128)).astype(np.float32)
    tA, tB, tC = (torch.from_numpy(x).cuda() for x in (A, B, C))
    tD = torch.empty((128, 128), dtype=torch.float32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(L.fermix_selftest_umma(s, tA.data_ptr(), tB.data_ptr(), tC.data_ptr(), tD.data_ptr(), negate,
                                      st.data_ptr()))
    torch.cuda.synchronize()
    assert int(st.item()) == 0, "MMA completion wait timed out"
    ref = C.astype(np.float64) + (-1.0 if negate else 1.0) * (A.astype(np.float64) @ B.astype(np.float64).T)
    D = tD.cpu().numpy()
    err = np.abs(D - ref).max() / np.abs(ref).max()
    assert err < 2e-6, err
