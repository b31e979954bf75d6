"""The C-ABI library loads and exports exactly what include/m3scan.h declares.

Host-side checks only (no kernel launches): symbol table, status strings,
argument validation that fails before any device work, checkpoint sizing.
"""

import ctypes
import os
import re

import pytest

from redpanda_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "m3scan.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"M3_API\s+[\w\s\*]+?\b(m3_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("m3_scan_fwd", "m3_scan_bwd", "m3_step", "m3_scan_bwd_workspace_bytes",
              "m3_scan_ckpt_floats", "m3_strerror", "m3_version", "m3_device_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for n in declared_functions():
        assert hasattr(lib, n), n
    # and the binding table covers every declared symbol
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_library_exports_nothing_else():
    out = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert exported == set(declared_functions())


def test_strerror_and_version():
    lib = _lib.load()
    assert lib.m3_version() >> 16 == 1
    assert _lib.strerror(0) == "ok"
    for code in range(1, 10):
        assert _lib.strerror(code).startswith("m3:")


def _desc(**kw):
    base = dict(batch=2, seqlen=64, d_inner=256, d_state=16, n_rot=12, dtype_du=0,
                dtype_bc=0, direction=0)
    base.update(kw)
    return _lib.ScanDesc(**base)


def test_validation_fails_before_device_work():
    lib = _lib.load()
    null = None
    # NULL descriptor
    assert lib.m3_scan_fwd(None, *([null] * 11), null) == 1
    # bad shapes / dtypes are rejected by the host checks
    for kw, code in [(dict(batch=0), 2), (dict(d_state=0), 2), (dict(d_state=200), 2),
                     (dict(n_rot=17), 2), (dict(dtype_du=7), 3), (dict(direction=5), 2)]:
        d = _desc(**kw)
        assert lib.m3_scan_fwd(ctypes.byref(d), *([null] * 11), null) == code, kw
    # NULL data pointers
    d = _desc()
    assert lib.m3_scan_fwd(ctypes.byref(d), *([null] * 11), null) == 1


def test_checkpoint_sizing():
    lib = _lib.load()
    # L <= 16: no checkpoints; otherwise (L/16 - 1) chunk states of padded lanes
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=16))) == 0
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=64))) == 2 * 3 * 256 * 16
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=64, direction=2))) == 2 * 2 * 3 * 256 * 16
    # virtual lanes: N=8 with 6 rotational + 2 tracking pads to 4*(2+1) = 12 lanes
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=33, d_state=8, n_rot=6))) == 2 * 2 * 256 * 12


@pytest.mark.parametrize("fn", ["m3_trapezoidal_scan", "m3_bidir_scan"])
def test_ops_refuse_cpu_tensors(fn):
    import torch
    from redpanda_b200 import scan as S
    x = torch.zeros(1, 4, 8)
    b = torch.zeros(1, 4, 4)
    A = torch.zeros(8, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        getattr(S, fn)(x, x, b, b, A, A, A, 2, 4)
