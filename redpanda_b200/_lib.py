"""ctypes binding of ``libm3scan.so`` (the C ABI declared in ``include/m3scan.h``).

The library is loaded from this package directory.  There is no fallback: if
it is missing or cannot be loaded, every op raises ``RuntimeError`` naming the
build command.
"""

import ctypes
import os
import threading

# M3_LIBRARY names another build of the same library (e.g. one compiled with a
# tuning macro by build.build_library(out=..., extra_flags=[...])).
LIB_PATH = os.environ.get("M3_LIBRARY") or os.path.join(
    os.path.dirname(os.path.abspath(__file__)), "libm3scan.so")

M3_F32, M3_BF16 = 0, 1
M3_DIR_FWD, M3_DIR_REV, M3_DIR_BIDIR = 0, 1, 2

# Every entry point the header declares: name -> (restype, argtypes).
_P = ctypes.c_void_p
_I = ctypes.c_int32
_Z = ctypes.c_size_t


class ScanDesc(ctypes.Structure):
    """``m3_scan_desc``."""
    _fields_ = [("batch", _I), ("seqlen", _I), ("d_inner", _I), ("d_state", _I),
                ("n_rot", _I), ("dtype_du", _I), ("dtype_bc", _I), ("direction", _I)]


class StepDesc(ctypes.Structure):
    """``m3_step_desc``."""
    _fields_ = [("batch", _I), ("d_inner", _I), ("d_state", _I), ("n_rot", _I),
                ("dtype_du", _I), ("dtype_bc", _I)]


_D = ctypes.POINTER(ScanDesc)
_S = ctypes.POINTER(StepDesc)

SIGNATURES = {
    "m3_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "m3_version": (ctypes.c_int, []),
    "m3_scan_ckpt_floats": (_Z, [_D]),
    "m3_scan_fwd": (ctypes.c_int, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "m3_scan_fwd_typed": (ctypes.c_int, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P,
                                         _P]),
    "m3_scan_fwd_fused": (ctypes.c_int, [_D, _I, _P, _P, ctypes.c_int64, _I, _I, _P, _P,
                                         ctypes.c_float, _P, _P, _P, _P, _P, _I, _P, _P]),
    "m3_scan_bwd_workspace_bytes": (_Z, [_D]),
    "m3_scan_bwd_fused_workspace_bytes": (_Z, [_D, _I]),
    "m3_scan_bwd_fused": (ctypes.c_int, [_D, _I, _P, _P, ctypes.c_int64, _I, _I, _P, _P,
                                         ctypes.c_float, _P, _P, _P, _P, _P, _I, _P, _P, _P,
                                         _P, _P, _P, _P, _P, _P, _P, _Z, _P]),
    "m3_scan_bwd": (ctypes.c_int, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P,
                                   _P, _P, _P, _P, _P, _P, _P, _P, _Z, _P]),
    "m3_step": (ctypes.c_int, [_S, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "m3_step_factored": (ctypes.c_int, [_S, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "m3_scan_bwd_noalloc": (ctypes.c_int, [_D, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P,
                                           _P, _P, _P, _P, _P, _P, _P, _P]),
    "m3_device_error": (ctypes.c_int, [ctypes.POINTER(_I), _I]),
    "m3_step_inputs": (ctypes.c_int, [_S, _I, _P, ctypes.c_int64, _P, _P, ctypes.c_int64, _I,
                                      _I, _P, _P, ctypes.c_float, _P, _P, _P, _P]),
    "m3_silu": (ctypes.c_int, [ctypes.c_int64, _I, _P, ctypes.c_int64, _P, _P]),
    "m3_rows_linear": (ctypes.c_int, [_I, _I, _I, _P, ctypes.c_int64, _P, ctypes.c_float, _P,
                                      _P, _P, ctypes.c_int64, _I, _I, _P, ctypes.c_int64, _P,
                                      ctypes.c_int64, _I, _P]),
    "m3_xdt_proj": (ctypes.c_int, [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P]),
    "m3_step_inputs_bwd_workspace_bytes": (_Z, [_S, _I]),
    "m3_step_inputs_bwd": (ctypes.c_int, [_S, _I, _P, ctypes.c_int64, _P, ctypes.c_int64, _I,
                                          _I, _P, _P, ctypes.c_float, _P, _P, _P, _P, _P, _P,
                                          _P, _P, _Z, _P]),
    "m3_gate": (ctypes.c_int, [ctypes.c_int64, _I, _P, _P, _I, _P, ctypes.c_int64, _P,
                               ctypes.c_float, _P, _P]),
    "m3_gate_typed": (ctypes.c_int, [ctypes.c_int64, _I, _P, _I, _P, _I, _P, _I,
                                     ctypes.c_int64, _P, ctypes.c_float, _I, _P, _I, _P]),
    "m3_gate_bwd_workspace_bytes": (_Z, [ctypes.c_int64, _I]),
    "m3_gate_bwd": (ctypes.c_int, [ctypes.c_int64, _I, _P, _I, _P, _I, _P, _I, ctypes.c_int64,
                                   _P, ctypes.c_float, _I, _P, _I, _P, _P, _P, _P, _P, _Z,
                                   _P]),
    "m3_step_gated": (ctypes.c_int, [_S, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                     ctypes.c_int64, _P, _P, _P]),
    "m3_step_gated_fused": (ctypes.c_int, [_S, _I, _P, _P, _P, _P, _P, ctypes.c_int64, _P, _P,
                                           ctypes.c_int64, _I, _I, _P, _P, ctypes.c_float,
                                           _P, _P, _P, _P, _P, ctypes.c_int64, _P, _P, _P]),
    "m3_step_gated_fused_proj": (ctypes.c_int, [_S, _I, _P, _P, _P, _P, _P, _I, _P, _P,
                                                ctypes.c_int64, _I, _I, _P, _P, ctypes.c_float,
                                                _P, _P, _P, _P, _P, ctypes.c_int64, _P, _P, _I,
                                                _P]),
}

_lock = threading.Lock()
_lib = None
_load_error = None


def load():
    """Load the library once and return the ctypes handle (raises if absent)."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            _load_error = (f"{LIB_PATH} is missing; build it with "
                           "`python -m redpanda_b200.build`")
            raise RuntimeError(_load_error)
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def available():
    """True when the library loads (no GPU needed)."""
    try:
        load()
        return True
    except (RuntimeError, OSError, AttributeError):   # AttributeError: a stale build
        return False


def strerror(code):
    return load().m3_strerror(int(code)).decode()


def check(code):
    """Raise RuntimeError for a non-zero status code."""
    if code != 0:
        raise RuntimeError(f"{strerror(code)} (status {code})")
