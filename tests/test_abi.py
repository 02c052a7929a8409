"""The C-ABI library loads and exports every entry point include/*.h declares; the
host-only entry points behave as documented (no GPU needed)."""

import glob
import os
import re

import pytest

from fermix_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(fermix_\w+)\s*\(", src))
    return names


@pytest.fixture(scope="module")
def lib():
    from fermix_b200.build import build

    build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(lib):
    names = _declared()
    assert names, "no declarations found"
    for name in sorted(names):
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_check_prec_and_strerror(lib):
    assert lib.fermix_check_prec(_lib.FX_F32, _lib.FX_PREC_TF32X3) == 0
    assert lib.fermix_check_prec(_lib.FX_C64, _lib.FX_PREC_IEEE) == 0
    assert lib.fermix_check_prec(_lib.FX_F64, _lib.FX_PREC_TF32X3) == 3
    assert lib.fermix_check_prec(_lib.FX_C128, _lib.FX_PREC_TF32X3) == 3
    assert lib.fermix_check_prec(_lib.FX_F32, 9) == 3
    for code in range(9):
        assert lib.fermix_strerror(code)
        assert lib.fermix_strerror(code) != b"unknown error code"
    assert lib.fermix_version() >= 200


def test_argument_errors_before_any_device_work(lib):
    # invalid dtype / shape / prec are rejected on the host, before touching a device
    assert lib.fermix_slogdet(None, 7, 0, 1, 4, None, None, None, None, None, 0) == 1
    assert lib.fermix_slogdet(None, 0, 0, -1, 4, None, None, None, None, None, 0) == 2
    assert lib.fermix_slogdet(None, 1, 1, 1, 4, None, None, None, None, None, 0) == 3
    assert lib.fermix_slogpf(None, 0, 0, 2, 8, 1, None, None, None, None, None, 0) == 5
    # an empty batch is a no-op
    assert lib.fermix_slogdet(None, 0, 0, 0, 4, None, None, None, None, None, 0) == 0


def test_missing_library_raises(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(_lib.FermixError):
        _lib.lib()
