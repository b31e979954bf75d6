"""m3_scan_bwd_noalloc: the backward for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc at the moment they run the
backward (their device memory was carved up at start-up by an allocator they
have no handle to, or they run in a loop that must not allocate).  For them the
library exposes one entry point whose scratch lives in a device buffer built
into the library.  This test calls it through the C ABI three times in a row --
bidirectional, causal, then bidirectional again with another batch, length and
seed, so that the shared buffer still holds the earlier calls' partial sums
when it is reused -- and checks every output against the regular m3_scan_bwd
(which is handed a caller-allocated workspace).  Both run the same
deterministic kernels on the same data, so the results must be equal bit for
bit.  It also checks that a problem too large for the built-in buffer is
refused with M3_ERR_SCRATCH_LIMIT.

The file name makes pytest collect it last; it passes alone in a fresh process
as well as after the other tests.
"""

import ctypes

import pytest
import torch

from redpanda_b200 import _lib
from redpanda_b200.scan import M3_DIR_BIDIR, M3_DIR_FWD, ScanPlan, pad_params
from redpanda_b200.synthetic import ScanShape, make_scan_inputs

pytestmark = pytest.mark.gpu

M3_ERR_SCRATCH_LIMIT = 10


def _case(shape, seed, direction, dtype):
    inp = make_scan_inputs(shape, seed=seed, dtype=dtype)
    dev = torch.device("cuda")
    g = {k: (None if v is None else v.to(dev)) for k, v in inp.items()}
    D, N = shape.d_inner, shape.d_state
    Ar, Ai, Tk = (t.contiguous() for t in pad_params(g["A_real"], g["A_imag"], g["track"],
                                                     shape.n_rot, N, D, dev))
    plan = ScanPlan(shape.batch, shape.seqlen, D, N, shape.n_rot, dtype, dtype, direction)
    y = torch.empty(shape.batch, shape.seqlen, D, device=dev)
    ckpt = torch.empty(max(plan.ckpt_floats(), 1), device=dev)
    plan.forward(g["delta"], g["u"], g["Bc"], g["Cc"], Ar, Ai, Tk, y,
                 ckpt if plan.ckpt_floats() else None)
    dy = g["dy"].contiguous()
    return plan, g, (Ar, Ai, Tk), dy, (ckpt if plan.ckpt_floats() else None)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _run(lib, plan, g, params, dy, ckpt, noalloc):
    D, N = plan.shape[2], plan.shape[3]
    outs = [torch.empty_like(g["delta"]), torch.empty_like(g["u"]), torch.empty_like(g["Bc"]),
            torch.empty_like(g["Cc"])] + [torch.empty(D, N, device="cuda") for _ in range(3)]
    Ar, Ai, Tk = params
    stream = torch.cuda.current_stream().cuda_stream
    args = [ctypes.byref(plan.desc), g["delta"].data_ptr(), g["u"].data_ptr(),
            g["Bc"].data_ptr(), g["Cc"].data_ptr(), Ar.data_ptr(), Ai.data_ptr(), Tk.data_ptr(),
            dy.data_ptr(), 0, _ptr(ckpt)] + [o.data_ptr() for o in outs]
    assert dy.dtype == torch.float32   # dtype_dy = M3_F32 above
    if noalloc:
        rc = lib.m3_scan_bwd_noalloc(*args, stream)
    else:
        nws = lib.m3_scan_bwd_workspace_bytes(ctypes.byref(plan.desc))
        ws = torch.empty(nws, device="cuda", dtype=torch.uint8)
        rc = lib.m3_scan_bwd(*args, ws.data_ptr(), nws, stream)
    torch.cuda.synchronize()
    assert rc == 0, _lib.strerror(rc)
    return outs


def test_noalloc_backward_matches_regular_backward_calls_in_a_row():
    lib = _lib.load()
    cases = [
        (ScanShape(4, 40, 256, 32, 16, 4), 21, M3_DIR_BIDIR, torch.float32),
        (ScanShape(3, 64, 192, 16, 4, 4), 22, M3_DIR_FWD, torch.float32),
        # bidirectional again, with a different batch, length and seed: its
        # partial sums and first-direction rows land on stale buffer contents
        (ScanShape(2, 29, 256, 32, 16, 4), 23, M3_DIR_BIDIR, torch.bfloat16),
    ]
    prepared = [_case(*c) for c in cases]
    refs = []
    for plan, g, params, dy, ckpt in prepared:
        assert lib.m3_scan_bwd_workspace_bytes(ctypes.byref(plan.desc)) <= _noalloc_bytes()
        refs.append(_run(lib, plan, g, params, dy, ckpt, noalloc=False))
    # no-allocation calls in a row: each finds the previous one's data in the
    # shared buffer
    gots = [_run(lib, *prep, noalloc=True) for prep in prepared]
    for got, ref in zip(gots, refs):
        for a, b in zip(got, ref):
            assert torch.isfinite(a.float()).all()
            assert torch.equal(a, b)


def _noalloc_bytes():
    # M3_NOALLOC_SCRATCH_BYTES in include/m3scan.h
    return 64 * 1024 * 1024


def test_noalloc_refuses_problems_beyond_its_buffer():
    lib = _lib.load()
    # config-2 rows: the workspace of 1024 rows is far above the built-in 64 MiB
    shape = ScanShape(1024, 64, 1536, 32, 16, 4)
    plan = ScanPlan(shape.batch, shape.seqlen, shape.d_inner, shape.d_state, shape.n_rot,
                    torch.bfloat16, torch.bfloat16, M3_DIR_BIDIR)
    assert lib.m3_scan_bwd_workspace_bytes(ctypes.byref(plan.desc)) > _noalloc_bytes()
    fake = ctypes.c_void_p(256)   # never dereferenced: the size check comes first
    args = [ctypes.byref(plan.desc)] + [fake] * 8 + [0, fake] + [fake] * 7
    rc = lib.m3_scan_bwd_noalloc(*args, None)
    assert rc == M3_ERR_SCRATCH_LIMIT
    assert "no-allocation buffer" in _lib.strerror(rc)
