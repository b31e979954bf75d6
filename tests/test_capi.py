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


def test_checkpoint_interval_of_the_gate_storing_layout():
    """The (16 rotational + 16 tracking) lane layout checkpoints every 8 steps
    (its backward keeps the gates in Tensor Memory), others every 16."""
    lib = _lib.load()
    c1 = dict(d_state=32, n_rot=16, d_inner=1536)
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=8, **c1))) == 0
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=64, **c1))) == 2 * 7 * 1536 * 32
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=64, direction=2, **c1))) == \
        2 * 2 * 7 * 1536 * 32
    c3 = dict(d_state=32, n_rot=24, d_inner=1024)
    assert lib.m3_scan_ckpt_floats(ctypes.byref(_desc(seqlen=64, **c3))) == 2 * 3 * 1024 * 32


def _sdesc(**kw):
    base = dict(batch=4, d_inner=64, d_state=16, n_rot=12, dtype_du=0, dtype_bc=0)
    base.update(kw)
    return _lib.StepDesc(**base)


def test_layer_entry_points_validate_before_device_work():
    """m3_step_inputs, m3_step_inputs_bwd, m3_gate and m3_step_gated reject bad
    arguments with their status codes before touching a device."""
    lib = _lib.load()
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.cast(buf, ctypes.c_void_p).value    # host memory: never dereferenced
    d = _sdesc()
    # m3_step_inputs(desc, p, dt, ld_dt, dt_bias, xbc, ld_x, off_b, off_c, wb, wc, eps,
    #                delta, Bc, Cc, s)
    assert lib.m3_step_inputs(None, 2, p, 64, None, p, 72, 8, 40, None, None, 1e-5, p, p, p,
                              None) == 1
    assert lib.m3_step_inputs(ctypes.byref(d), 2, p, 32, None, p, 72, 8, 40, None, None, 1e-5,
                              p, p, p, None) == 2          # ld_dt < d_inner
    assert lib.m3_step_inputs(ctypes.byref(d), 2, p, 64, None, p, 60, 8, 40, None, None, 1e-5,
                              p, p, p, None) == 2          # C_raw past the row
    assert lib.m3_step_inputs(ctypes.byref(d), 2, p, 64, None, p, 72, 8, 40, p, None, 1e-5,
                              p, p, p, None) == 1          # one BCNorm weight without the other
    assert lib.m3_step_inputs(ctypes.byref(d), 0, p, 64, None, p, 72, 8, 40, None, None, 1e-5,
                              p, p, p, None) == 2          # mimo_p = 0
    assert lib.m3_step_inputs(ctypes.byref(d), 2, p, 64, p + 2, p, 72, 8, 40, None, None, 1e-5,
                              p, p, p, None) == 5          # misaligned dt_bias
    # m3_silu(rows, d, x, ld_x, out, s)
    assert lib.m3_silu(0, 64, p, 64, p, None) == 2
    assert lib.m3_silu(4, 64, p, 32, p, None) == 2       # ld_x < d
    assert lib.m3_silu(4, 64, None, 64, p, None) == 1
    assert lib.m3_silu(4, 64, p + 1, 64, p, None) == 5
    # m3_step_inputs_bwd: a BCNorm backward without a workspace
    args = [ctypes.byref(d), 2, p, 64, p, 72, 8, 40, p, p, 1e-5, p, p, p, p, p, p, p, None, 0,
            None]
    assert lib.m3_step_inputs_bwd(*args) == 6
    assert lib.m3_step_inputs_bwd_workspace_bytes(ctypes.byref(d), 2) > 0
    # m3_gate_bwd(rows, D, y, dty, u, dtu, z, dtz, ld_z, d_skip, coef, round, g, dtg,
    #             d_y, d_u, d_z, d_dskip, ws, ws_bytes, s)
    need = lib.m3_gate_bwd_workspace_bytes(64, 96)
    assert need >= 96 * 4 and lib.m3_gate_bwd_workspace_bytes(0, 96) == 0
    gb = [64, 96, p, 1, p, 1, p, 1, 192, p, 2.0, 1, p, 0, p, p, p, p, p, need, None]
    assert lib.m3_gate_bwd(*(gb[:8] + [64] + gb[9:])) == 2                 # ld_z < D
    assert lib.m3_gate_bwd(*(gb[:13] + [7] + gb[14:])) == 3                # dtype of g
    assert lib.m3_gate_bwd(*(gb[:12] + [None] + gb[13:])) == 1             # no g
    assert lib.m3_gate_bwd(*(gb[:19] + [need - 4] + gb[20:])) == 6         # workspace
    assert lib.m3_gate_bwd(*(gb[:2] + [p + 1] + gb[3:])) == 5              # misaligned y
    # m3_gate(rows, D, y, u, dtype_u, z, ld_z, d_skip, coef, out, s)
    assert lib.m3_gate(0, 64, p, p, 0, p, 64, p, 1.0, p, None) == 2
    assert lib.m3_gate(4, 64, p, p, 0, p, 32, p, 1.0, p, None) == 2    # ld_z < D
    assert lib.m3_gate(4, 64, p, p, 9, p, 64, p, 1.0, p, None) == 3    # dtype
    assert lib.m3_gate(4, 64, None, p, 0, p, 64, p, 1.0, p, None) == 1
    # m3_step_gated: exactly one state form, a z row stride >= D
    g = [ctypes.byref(d), p, p, p, p, p, p, p, p, p, p, p, p, 64, p, p, None]
    assert lib.m3_step_gated(*g) == 1                                  # both forms given
    g[2] = None
    g[4] = None
    assert lib.m3_step_gated(*g) == 1                                  # neither form
    g[2] = p
    g[13] = 32
    assert lib.m3_step_gated(*g) == 2                                  # ld_z < D


def test_small_batch_projections_validate_before_device_work():
    """m3_rows_linear and m3_xdt_proj reject bad arguments, shapes past their
    staging limits (M3_ERR_UNSUPPORTED) and overlapping buffers before any
    device work."""
    lib = _lib.load()
    buf = ctypes.create_string_buffer(1 << 16)
    p = (ctypes.cast(buf, ctypes.c_void_p).value + 15) & ~15   # host memory, never read
    q = p + 8192
    # m3_rows_linear(rows, d_in, d_out, x, ld_x, norm_w, eps, W, bias, residual, ld_r,
    #                split, silu, out0, ld0, out1, ld1, overlap, s)
    a = [2, 64, 96, p, 64, None, 1e-5, p + 4096, None, None, 0, 96, 0, q, 96, None, 0, 0, None]

    def rl(**kw):
        names = ["rows", "d_in", "d_out", "x", "ld_x", "norm_w", "eps", "W", "bias",
                 "residual", "ld_r", "split", "silu", "out0", "ld0", "out1", "ld1", "overlap",
                 "s"]
        v = dict(zip(names, a))
        v.update(kw)
        return lib.m3_rows_linear(*[v[n] for n in names])

    assert rl(rows=0) == 2
    assert rl(rows=9) == 4                     # more rows than the kernels take
    assert rl(d_in=66, ld_x=66) == 4           # d_in not a multiple of 4
    assert rl(rows=8, d_in=2048, ld_x=2048) == 4   # 64 KB of staged input
    assert rl(W=None) == 1
    assert rl(W=p + 4100) == 5                 # weight rows not 16-byte aligned
    assert rl(split=97) == 2
    assert rl(split=64) == 1                   # columns past split need out1
    assert rl(ld_x=32) == 2
    assert rl(out0=p + 64) == 11               # output overlaps the staged input
    # m3_xdt_proj(rows, d_inner, n_x, dt_rank, u, W_x, b_x, W_dt, x_dbl, dt, overlap, s)
    x = [2, 64, 40, 8, p, p + 4096, None, p + 4096, q, q + 4096, 0, None]
    assert lib.m3_xdt_proj(*(x[:2] + [6] + x[3:])) == 2           # n_x < dt_rank
    assert lib.m3_xdt_proj(*([9] + x[1:])) == 4
    assert lib.m3_xdt_proj(*(x[:4] + [None] + x[5:])) == 1
    assert lib.m3_xdt_proj(*(x[:5] + [p + 4100] + x[6:])) == 5    # misaligned W_x
    assert lib.m3_xdt_proj(*(x[:9] + [q] + x[10:])) == 11          # dt overlaps x_dbl


def test_step_gated_fused_proj_validates_before_device_work():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(4096)
    p = (ctypes.cast(buf, ctypes.c_void_p).value + 15) & ~15
    d = _sdesc()
    # (desc, mimo_p, h, dbu, fac_prev, fac_next, W_dt, dt_rank, dt_bias, xbc, ld_x, off_b,
    #  off_c, wb, wc, eps, u, Ar, Ai, Tk, z, ld_z, d_skip, out, overlap, s)
    a = [ctypes.byref(d), 2, p, p, None, None, p, 8, None, p, 72, 8, 40, None, None, 1e-5,
         p, p, p, p, p, 64, p, p, 0, None]
    assert lib.m3_step_gated_fused_proj(*(a[:6] + [None] + a[7:])) == 1      # no W_dt
    assert lib.m3_step_gated_fused_proj(*(a[:7] + [0] + a[8:])) == 2         # dt_rank 0
    assert lib.m3_step_gated_fused_proj(*(a[:7] + [80] + a[8:])) == 2        # past the row
    big = a[:7] + [68] + a[8:10] + [136] + a[11:]
    assert lib.m3_step_gated_fused_proj(*big) == 4                           # dt_rank > 64
    assert lib.m3_step_gated_fused_proj(*(a[:6] + [p + 2] + a[7:])) == 5     # misaligned W_dt


def test_small_step_eligibility_is_host_logic():
    """Which lockstep batches take the small-batch layer (decided on the host
    before any launch, so a layer never stops half way)."""
    import torch
    from redpanda_b200.mamba import Mamba3Block, MambaConfig
    blk = Mamba3Block(MambaConfig(d_model=512, n_layer=1, d_state=32, n_track_state=8,
                                  mimo_p=2))
    x1, x9 = torch.zeros(1, 512), torch.zeros(9, 512)
    with torch.no_grad():
        assert blk.small_step_ok(x1)
        assert blk.small_step_ok(torch.zeros(8, 512))
        assert not blk.small_step_ok(x9)                       # more rows than the kernels take
        assert not blk.small_step_ok(x1.double())              # fp32 only
    assert not blk.small_step_ok(x1)                           # autograd on: the training path
    wide = Mamba3Block(MambaConfig(d_model=2048, n_layer=1, d_state=32, n_track_state=8,
                                   mimo_p=2))
    with torch.no_grad():
        assert not wide.small_step_ok(torch.zeros(1, 2048))    # dt_rank 128 > 64
    old = Mamba3Block.small_step_max_batch
    Mamba3Block.small_step_max_batch = 0
    try:
        with torch.no_grad():
            assert not blk.small_step_ok(x1)                   # switched off
    finally:
        Mamba3Block.small_step_max_batch = old
