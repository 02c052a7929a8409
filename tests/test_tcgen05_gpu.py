"""The tensor-core building blocks (tcgen05 MMA into tensor memory, shared-memory operand
descriptors, 3xTF32 split) against a float64 product: D = C +- A B^T at 128 x 128 x 16."""

import ctypes

import numpy as np
import pytest
import torch

from fermix_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("negate,accumulate,masked", [(0, 1, 0), (1, 1, 0), (1, 0, 0), (0, 0, 1), (1, 1, 1)])
def test_umma_3xtf32_update(negate, accumulate, masked):
    g = np.random.default_rng(7 + negate)
    A = g.standard_normal((128, 16)).astype(np.float32)
    B = g.standard_normal((128, 16)).astype(np.float32)
    C = g.standard_normal((128, 128)).astype(np.float32)
    tA, tB, tC = (torch.from_numpy(x).cuda() for x in (A, B, C))
    tD = torch.empty((128, 128), dtype=torch.float32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    dis = (ctypes.c_uint * 4)(*([0x0F0F00F1, 0, 0xFFFF0000, 0x80000001] if masked else [0, 0, 0, 0]))
    _lib.check(L.fermix_selftest_umma(s, tA.data_ptr(), tB.data_ptr(), tC.data_ptr(), tD.data_ptr(), negate,
                                      accumulate, ctypes.cast(dis, ctypes.c_void_p), st.data_ptr()))
    torch.cuda.synchronize()
    assert int(st.item()) == 0, "MMA completion wait timed out"
    prod = (-1.0 if negate else 1.0) * (A.astype(np.float64) @ B.astype(np.float64).T)
    ref = (C.astype(np.float64) if accumulate else 0.0) + prod
    D = tD.cpu().numpy()
    keep = np.array([(dis[r // 32] >> (r % 32)) & 1 for r in range(128)], bool)
    assert np.array_equal(D[keep], C[keep])  # disabled lanes untouched
    err = np.abs(D[~keep] - ref[~keep]).max() / np.abs(ref[~keep]).max()
    assert err < 2e-6, err
