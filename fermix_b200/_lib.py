"""ctypes binding of libfermix_b200.so (the C ABI declared in include/fermix_b200.h).

The library is built in-tree (``python -m fermix_b200.build``) and loaded from
``fermix_b200/_lib/``. There is no fallback: if the library is missing or cannot be
loaded, every call raises.
"""

import ctypes
import os
import threading

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libfermix_b200.so")

FX_F32, FX_F64, FX_C64, FX_C128 = 0, 1, 2, 3
FX_PREC_DEFAULT, FX_PREC_TF32X3, FX_PREC_IEEE = 0, 1, 2
FX_OP_SLOGDET, FX_OP_SLOGPF = 0, 1
FX_ERR_TIMEOUT = 8
FX_WAIT_POLLS_DEFAULT = 1 << 26

# every symbol include/fermix_b200.h declares, with its ctypes signature
_vp, _i, _i64, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "fermix_slogdet": (_i, [_vp, _i, _i, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogdet_grad": (_i, [_vp, _i, _i, _i64, _i64, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogpf": (_i, [_vp, _i, _i, _i64, _i64, _i, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogpf_grad": (_i, [_vp, _i, _i, _i64, _i64, _i, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogdet_grad_static": (_i, [_vp, _i, _i, _i64, _i64, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp]),
    "fermix_slogdet_gather": (
        _i, [_vp, _i, _i, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogdet_gather_workspace_bytes": (_sz, [_i, _i, _i64, _i64, _i]),
    "fermix_slogdet_ratio": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "fermix_slogdet_update": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogdet_update_workspace_bytes": (_sz, [_i, _i64, _i64, _i64]),
    "fermix_slogpf_ratio": (_i, [_vp, _i, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    "fermix_slogpf_update": (_i, [_vp, _i, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogpf_update_workspace_bytes": (_sz, [_i, _i64, _i64]),
    "fermix_slogpf_ratio_k": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogpf_update_k": (_i, [_vp, _i, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogpf_move_k_workspace_bytes": (_sz, [_i, _i64, _i64, _i64]),
    "fermix_workspace_bytes": (_sz, [_i, _i, _i64, _i64, _i]),
    "fermix_check_prec": (_i, [_i, _i]),
    "fermix_strerror": (ctypes.c_char_p, [_i]),
    "fermix_version": (_i, []),
    "fermix_selftest_umma": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _vp]),
    "fermix_selftest_fma_rate": (_i, [_vp, _i, _i, _i, _vp]),
    "fermix_device_status": (_i, [_i]),
    "fermix_set_wait_polls": (ctypes.c_uint, [ctypes.c_uint]),
    "fermix_slogdet_planar": (_i, [_vp, _i, _i, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogdet_grad_planar": (
        _i, [_vp, _i, _i, _i64, _i64, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogpf_planar": (_i, [_vp, _i, _i, _i64, _i64, _i, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_slogpf_grad_planar": (
        _i, [_vp, _i, _i, _i64, _i64, _i, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _sz]),
    "fermix_workspace_bytes_planar": (_sz, [_i, _i, _i64, _i64, _i]),
    # include/fermix_b200_xla.h
    "fermix_xla_custom_call": (None, [_vp, _vp, ctypes.c_char_p, _sz]),
    "fermix_xla_last_error": (_i, [_i]),
}

_lib = None
_lock = threading.Lock()


class FermixError(RuntimeError):
    """A non-zero status from the CUDA library."""


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise FermixError(
                    f"{LIB_PATH} is missing: build it with `python -m fermix_b200.build` "
                    "(fermix_b200 has no CPU fallback)"
                )
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def device_status(clear=False):
    """The kernels' status on the current CUDA device (synchronises it): 0, or
    FX_ERR_TIMEOUT when a kernel gave up a bounded wait since the last clear (its members'
    outputs are NaN). Entry points are stream-ordered, so they cannot return it."""
    return lib().fermix_device_status(int(clear))


def check(status):
    if status != 0:
        msg = lib().fermix_strerror(status).decode()
        raise FermixError(f"fermix_b200 error {status}: {msg}")
