"""The CUDA path against the committed golden fixtures (tests/golden/golden.npz), through
the public API (forward) and the one-launch parts functions (JAX-convention gradients)."""

import os

import numpy as np
import pytest

import fermix_b200 as fx
from tests.helpers import cuda, host

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")


class CudaPath:
    """The oracle's API backed by the CUDA library."""

    @staticmethod
    def slogdet(a):
        return host(fx.slogdet(cuda(a)))

    @staticmethod
    def slogpf(a, skew_symmetrize=True):
        return host(fx.slogpf(cuda(a), skew_symmetrize=skew_symmetrize))

    @staticmethod
    def det(a):
        return host(fx.det(cuda(a)))

    @staticmethod
    def pf(a, skew_symmetrize=True):
        return host(fx.pf(cuda(a), skew_symmetrize=skew_symmetrize))

    @staticmethod
    def slogdet_grad(a):
        return host(fx.slogdet_parts(cuda(a))[2])

    @staticmethod
    def slogpf_grad(a, skew_symmetrize=True):
        return host(fx.slogpf_parts(cuda(a), skew_symmetrize=skew_symmetrize)[2])

    @staticmethod
    def det_grad(a):
        return host(fx.det_parts(cuda(a))[1])

    @staticmethod
    def pf_grad(a, skew_symmetrize=True):
        return host(fx.pf_parts(cuda(a), skew_symmetrize=skew_symmetrize)[1])


def _names():
    from tests.golden.make_golden import CASES

    return CASES


@pytest.mark.parametrize("name", _names())
def test_cuda_matches_golden(name):
    from tests.golden.make_golden import check_case

    check_case(name, np.load(GOLDEN), CudaPath)
