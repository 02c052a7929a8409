"""bench.py's attribution of each workload to its dominant kernel (the roofline's kernel name and
the committed ncu summary its DRAM traffic figure comes from). CPU only: nothing is launched."""

import importlib.util
import os
import types

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _args(**kw):
    base = dict(op="slogpf", dtype="f32", n=128, prec="tf32x3", fwd_only=False, gather=0, batch=4096)
    base.update(kw)
    return types.SimpleNamespace(**base)


@pytest.mark.parametrize("kw,kernel", [
    (dict(), "pf_tc_kernel"),
    (dict(prec="ieee"), "pf_tc_kernel"),
    (dict(op="slogdet"), "lu_tc_kernel"),
    (dict(op="slogdet", n=256), "lu_tc_kernel"),
    (dict(op="slogdet", prec="ieee"), "lu_tc_kernel"),
    (dict(op="slogdet", dtype="f64"), "lu_small_kernel"),
    (dict(op="slogpf", n=130), "pf_small_kernel"),
    (dict(dtype="c64", n=512), "lg_tc_update_kernel"),
    (dict(dtype="c64", n=512, prec="ieee"), "lg_update_kernel"),
    (dict(op="slogdet", dtype="f64", n=4096, prec="ieee"), "lg_update_kernel"),
    (dict(dtype="c128", n=4096, prec="ieee"), "lg_dmma_update_kernel"),
])
def test_kernel_attribution(bench, kw, kernel):
    assert bench.kernel_name(_args(**kw)) == kernel


def test_headline_traffic_comes_from_its_profile(bench):
    t = bench.traffic_from_profiles(_args())
    assert t is not None and 4096 * 64 * 1024 <= t <= 4096 * 2 * 128 * 128 * 4
    # prec ieee runs the FMA variant of the same kernel: the tf32x3 capture does not apply
    assert bench.traffic_from_profiles(_args(prec="ieee")) is None
    assert bench.traffic_from_profiles(_args(op="slogdet", prec="ieee", fwd_only=True)) is None
    assert bench.traffic_from_profiles(_args(op="slogdet", fwd_only=True)) is not None
