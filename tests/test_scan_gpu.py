"""GPU parity of the sm_100a scan kernels against the CPU oracle.

Bars (norm-wise relative error max|a-b| / max|ref|):
  * forward y: 1e-5 against the reference's own fp32 numerics (the oracle run
    in float32)
  * fp32 gradients: 1e-6 against the same fp32 reference.  A (case, key) pair
    that misses it passes only when it is listed in GRAD_ALLOW below, with
    its measured value and a bound, AND is at least as close to the float64
    recurrence as the fp32 reference itself is (there the fp32 reference, not
    the kernel, carries the larger error)
  * bf16 outputs (grads cast to the bf16 input dtype, as triton_scan.py:313-315
    does): within one bf16 ulp of the fp32 reference value
Every measured error is recorded in helpers.PARITY_TABLE and printed as a
table at the end of the pytest run (tests/conftest.py), so the figures behind
these bars are part of the test output.

The wide gate-argument cases (test_scan_parity_wide_gate_arguments) drive
|delta*A_imag| far past the benchmark range (see helpers.wide_gate_inputs).
There the reference's fp32 path evaluates cos at the fp32-ROUNDED product
delta*A_imag and is itself 6e-6..6e-4 from the exact recurrence, so those
cases are held to the same bars against the float64 recurrence, and the fp32
reference's own distance is recorded beside them.
"""

import pytest
import torch

from helpers import (GRAD_KEYS, PARITY_TABLE, WIDE_REGIMES, gate_arg_stats, oracle_scan,
                     rel_err, to_cuda, wide_gate_inputs)
from redpanda_b200 import scan as S
from redpanda_b200.synthetic import ScanShape, make_scan_inputs

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-5
GRAD_TOL = 1e-6

CASES = [
    # name, shape, input dtype, direction (0 causal, 1 reverse, 2 bidirectional)
    ("c0_causal", ScanShape(8, 64, 256, 16, 4, 4), torch.float32, 0),
    ("c0_reverse", ScanShape(8, 64, 256, 16, 4, 4), torch.float32, 1),
    ("c0_bidir", ScanShape(8, 64, 256, 16, 4, 4), torch.float32, 2),
    ("c1_rows_bidir_f32", ScanShape(2, 64, 1536, 32, 16, 4), torch.float32, 2),
    ("c1_rows_bidir_bf16", ScanShape(2, 64, 1536, 32, 16, 4), torch.bfloat16, 2),
    ("c2_rows_causal_bf16", ScanShape(2, 64, 1536, 32, 16, 4), torch.bfloat16, 0),
    ("c3_rows_causal", ScanShape(2, 64, 1024, 32, 8, 2), torch.float32, 0),
    ("ragged_L70_no_track", ScanShape(2, 70, 64, 16, 0, 2), torch.float32, 0),
    ("L1", ScanShape(3, 1, 32, 12, 8, 2), torch.float32, 0),
    ("L33_N12_bidir", ScanShape(3, 33, 96, 12, 4, 2), torch.float32, 2),
    ("D200_virtual_lanes", ScanShape(2, 40, 200, 8, 2, 2), torch.float32, 0),
    ("N64_bidir", ScanShape(2, 50, 128, 64, 16, 4), torch.float32, 2),
    ("bf16_odd_D", ScanShape(2, 20, 33, 16, 4, 2), torch.bfloat16, 0),
    ("all_tracking", ScanShape(2, 24, 64, 8, 8, 2), torch.float32, 0),
    ("no_rotation_verify_cfg", ScanShape(3, 70, 96, 16, 0, 2), torch.float32, 2),
    # config-1 lane layout (gates kept in Tensor Memory, 8-step chunks): ragged
    # last chunk, a single chunk, and a one-step last chunk
    ("c1_layout_L37_bidir", ScanShape(3, 37, 96, 32, 16, 4), torch.float32, 2),
    ("c1_layout_L8_causal", ScanShape(2, 8, 64, 32, 16, 4), torch.float32, 0),
    ("c1_layout_L9_reverse_bf16", ScanShape(2, 9, 64, 32, 16, 4), torch.bfloat16, 1),
    ("N8_no_track_bidir", ScanShape(2, 20, 256, 8, 0, 2), torch.float32, 2),
]

_FN = {0: S.m3_trapezoidal_scan, 1: S.m3_reverse_scan, 2: S.m3_bidir_scan}


def run_m3(inp, direction, dtype):
    g = to_cuda(inp)
    lv = {}
    for k in ("delta", "u", "Bc", "Cc"):
        lv[k] = g[k].to(dtype).clone().requires_grad_(True)
    for k in ("A_real", "A_imag", "track"):
        lv[k] = None if g[k] is None else g[k].clone().requires_grad_(True)
    nr = 0 if inp["A_real"] is None else inp["A_real"].shape[-1]
    y = _FN[direction](lv["delta"], lv["u"], lv["Bc"], lv["Cc"], lv["A_real"], lv["A_imag"],
                       lv["track"], nr, inp["Bc"].shape[-1])
    (y * g["dy"]).sum().backward()
    torch.cuda.synchronize()
    return y.detach(), {k: (None if v is None else v.grad) for k, v in lv.items()}


def _bf16_ok(a, ref):
    a = a.float().cpu()
    ref = ref.float().cpu()
    ulp = torch.pow(2.0, torch.floor(torch.log2(ref.abs().clamp(min=1e-30))) - 7)
    return bool(((a - ref).abs() <= ulp + 1e-6 * ref.abs().max()).all())


# (case, gradient key) -> (error vs the fp32 reference measured on a B200, bound).
# Each entry is a gradient whose fp32 rounding differs from the reference's
# fp32 rounding by a little more than 1e-6 of its largest element while being
# at least as close to the float64 recurrence as the reference is.
GRAD_ALLOW = {}


def _check_grads(name, g, g32, g64, failures):
    """Record every gradient's errors and collect the ones that miss their bar."""
    for k in GRAD_KEYS:
        if g[k] is None:
            continue
        e32 = rel_err(g[k], g32[k])
        e64 = rel_err(g[k], g64[k])
        r64 = rel_err(g32[k], g64[k])
        if g[k].dtype == torch.bfloat16:
            ok = _bf16_ok(g[k], g32[k])
            PARITY_TABLE.append((name, "d" + k, "bf16", e32, e64, r64,
                                 "ok (1 bf16 ulp)" if ok else "FAIL"))
            if not ok:
                failures.append((k, "bf16 ulp"))
            continue
        if e32 <= GRAD_TOL:
            verdict = "ok"
        elif (name, k) in GRAD_ALLOW and e32 <= GRAD_ALLOW[(name, k)][1] and e64 <= max(r64, GRAD_TOL):
            verdict = "allow-listed"
        else:
            verdict = "FAIL"
            failures.append((k, e32))
        PARITY_TABLE.append((name, "d" + k, "fp32", e32, e64, r64, verdict))


@pytest.mark.parametrize("name,shape,dtype,direction", CASES, ids=[c[0] for c in CASES])
def test_scan_parity(name, shape, dtype, direction):
    inp = make_scan_inputs(shape, seed=11, dtype=dtype)
    inp32 = {k: (None if v is None else v.float()) for k, v in inp.items()}
    y, g = run_m3(inp, direction, dtype)
    y32, g32 = oracle_scan(inp32, direction, torch.float32)
    y64, g64 = oracle_scan(inp32, direction, torch.float64)
    assert y.dtype == torch.float32
    ey = rel_err(y, y32)
    PARITY_TABLE.append((name, "y", "fp32", ey, rel_err(y, y64), rel_err(y32, y64),
                         "ok" if ey <= FWD_TOL else "FAIL"))
    failures = []
    _check_grads(name, g, g32, g64, failures)
    assert ey <= FWD_TOL
    assert not failures, failures


# Wide-regime (case, gradient key) -> (error vs float64 measured on a B200, bound).
# dA_real of the config-1 lane layout at D=128, bf16 inputs, causal: the
# kernel's fp32 value misses 1e-6 of float64 while the reference's own fp32
# path is further from float64 still (2.4e-6 and 1.1e-4 in the two regimes);
# folding the chunk sums into float64 totals left it unchanged, so it is the
# fp32 rounding of the per-cell terms, not the summation order.  The test
# also requires the kernel to stay at least as close to float64 as the
# fp32 reference.
WIDE_GRAD_ALLOW = {
    ("wide_k_mid_N32T16_dir0_bf16", "A_real"): (1.67e-6, 3e-6),
    ("wide_mixed_N32T16_dir0_bf16", "A_real"): (2.20e-6, 4e-6),
}

WIDE_CASES = [
    # regime, shape, input dtype, direction
    (r, sh, dt, d)
    for r in WIDE_REGIMES
    for (sh, dt, d) in (
        (ScanShape(2, 64, 256, 32, 16, 4), torch.float32, 2),    # config-1 lane layout
        (ScanShape(2, 64, 256, 32, 16, 4), torch.bfloat16, 2),
        (ScanShape(2, 50, 256, 32, 8, 2), torch.float32, 0),     # config-3 lane layout
        (ScanShape(2, 40, 256, 16, 4, 4), torch.float32, 1),     # config-0 lane layout
        (ScanShape(2, 64, 128, 32, 16, 4), torch.bfloat16, 0),
    )
]


@pytest.mark.parametrize("regime,shape,dtype,direction", WIDE_CASES,
                         ids=[f"{c[0]}-N{c[1].d_state}T{c[1].n_track}-"
                              f"{'bf16' if c[2] == torch.bfloat16 else 'f32'}-"
                              f"{('causal', 'reverse', 'bidir')[c[3]]}" for c in WIDE_CASES])
def test_scan_parity_wide_gate_arguments(regime, shape, dtype, direction):
    """Forward and every gradient over the whole range of the gate's argument
    reduction (2 <= |k| <= 2048 on the packed path, the checked per-step path,
    and the double-precision slow path for |k| > 2048), against the float64
    recurrence (mamba.py:396-401 evaluated exactly)."""
    inp = wide_gate_inputs(shape, 41, regime, dtype=dtype)
    xmax, kmax, frac_slow = gate_arg_stats(inp)
    if regime == "k_mid":
        assert 2 <= kmax <= 2048 and frac_slow == 0.0
    elif regime == "mixed":
        assert kmax > 2048 and 0.0 < frac_slow < 0.05
    else:
        assert frac_slow > 0.9
    inp32 = {k: (None if v is None else v.float()) for k, v in inp.items()}
    y, g = run_m3(inp, direction, dtype)
    y32, g32 = oracle_scan(inp32, direction, torch.float32)
    y64, g64 = oracle_scan(inp32, direction, torch.float64)
    name = f"wide_{regime}_N{shape.d_state}T{shape.n_track}_dir{direction}_" + \
        ("bf16" if dtype == torch.bfloat16 else "f32")
    ey = rel_err(y, y64)
    PARITY_TABLE.append((name, "y", "fp32", rel_err(y, y32), ey, rel_err(y32, y64),
                         "ok" if ey <= FWD_TOL else "FAIL"))
    failures = [("y", ey)] if ey > FWD_TOL else []
    for k in GRAD_KEYS:
        if g[k] is None:
            continue
        e64 = rel_err(g[k], g64[k])
        r64 = rel_err(g32[k], g64[k])
        if g[k].dtype == torch.bfloat16:
            ok = _bf16_ok(g[k], g64[k])
            PARITY_TABLE.append((name, "d" + k, "bf16", rel_err(g[k], g32[k]), e64, r64,
                                 "ok (1 bf16 ulp of fp64)" if ok else "FAIL"))
            if not ok:
                failures.append((k, "bf16 ulp"))
            continue
        if e64 <= GRAD_TOL:
            verdict = "ok"
        elif ((name, k) in WIDE_GRAD_ALLOW and e64 <= WIDE_GRAD_ALLOW[(name, k)][1]
              and e64 <= r64):
            verdict = "allow-listed"
        else:
            verdict = "FAIL"
            failures.append((k, e64))
        PARITY_TABLE.append((name, "d" + k, "fp32", rel_err(g[k], g32[k]), e64, r64, verdict))
    assert not failures, (failures, xmax, kmax, frac_slow)
    assert S.device_error() == 0


def test_grad_dtypes_follow_inputs():
    inp = make_scan_inputs(ScanShape(2, 20, 64, 16, 4, 2), seed=2, dtype=torch.bfloat16)
    _, g = run_m3(inp, 2, torch.bfloat16)
    for k in ("delta", "u", "Bc", "Cc"):
        assert g[k].dtype == torch.bfloat16
    for k in ("A_real", "A_imag", "track"):
        assert g[k].dtype == torch.float32


def test_return_state_matches_oracle():
    import oracle as O
    sh = ScanShape(3, 50, 256, 32, 8, 2)
    inp = make_scan_inputs(sh, seed=4)
    g = to_cuda(inp)
    y, (h, dbu) = S.m3_scan_with_state(g["delta"], g["u"], g["Bc"], g["Cc"], g["A_real"],
                                       g["A_imag"], g["track"], sh.n_rot, sh.d_state)
    yr, (hr, dr) = O.scan_chunked(inp["delta"], inp["u"], inp["Bc"], inp["Cc"], inp["A_real"],
                                  inp["A_imag"], inp["track"], return_state=True)
    assert rel_err(y, yr) <= FWD_TOL
    assert rel_err(h, hr) <= FWD_TOL
    assert rel_err(dbu, dr) <= FWD_TOL


def test_bidir_equals_forward_plus_reverse_bitwise_full_c1():
    """Size-independent property at the full config-1 shape."""
    sh = ScanShape(1024, 64, 1536, 32, 16, 4)
    gen = torch.Generator("cuda").manual_seed(0)
    B, L, D, N = sh.batch, sh.seqlen, sh.d_inner, sh.d_state
    dl = torch.nn.functional.softplus(torch.randn(B, L, D, device="cuda", generator=gen) * 0.5 - 2)
    dl = dl.bfloat16()
    u = torch.randn(B, L, D, device="cuda", generator=gen).bfloat16()
    Bc = torch.randn(B, L, N, device="cuda", generator=gen).bfloat16()
    Cc = torch.randn(B, L, N, device="cuda", generator=gen).bfloat16()
    Ar = -torch.exp(torch.randn(D, 16, device="cuda", generator=gen) * 0.5)
    Ai = (torch.rand(D, 16, device="cuda", generator=gen) * 2 - 1) * 3.14159
    tk = torch.tanh(torch.randn(D, 16, device="cuda", generator=gen))
    yb = S.m3_bidir_scan(dl, u, Bc, Cc, Ar, Ai, tk, 16, 32)
    yf = S.m3_trapezoidal_scan(dl, u, Bc, Cc, Ar, Ai, tk, 16, 32)
    yr = S.m3_reverse_scan(dl, u, Bc, Cc, Ar, Ai, tk, 16, 32)
    assert torch.equal(yb, yf + yr)
    # reverse == flip(forward(flip)) bit for bit
    yff = S.m3_trapezoidal_scan(dl.flip(1), u.flip(1), Bc.flip(1), Cc.flip(1), Ar, Ai, tk, 16, 32)
    assert torch.equal(yr, yff.flip(1))
    # rows are independent: a slice of the batch reproduces its rows exactly
    idx = torch.tensor([0, 517, 1023], device="cuda")
    ys = S.m3_bidir_scan(dl[idx], u[idx], Bc[idx], Cc[idx], Ar, Ai, tk, 16, 32)
    assert torch.equal(ys, yb[idx])
    assert torch.isfinite(yb).all()


def test_backward_is_deterministic():
    sh = ScanShape(16, 64, 1536, 32, 16, 4)
    inp = make_scan_inputs(sh, seed=1, dtype=torch.bfloat16)
    ya, ga = run_m3(inp, 2, torch.bfloat16)
    yb, gb = run_m3(inp, 2, torch.bfloat16)
    assert torch.equal(ya, yb)
    for k in GRAD_KEYS:
        assert torch.equal(ga[k], gb[k]), k


def test_no_device_error_recorded():
    assert S.device_error(clear=True) == 0


BULK_CASES = [
    ("c1_layout_bidir_f32", ScanShape(3, 37, 256, 32, 16, 4), torch.float32, 2),
    ("c1_layout_bidir_bf16", ScanShape(2, 64, 256, 32, 16, 4), torch.bfloat16, 2),
    ("c3_layout_causal", ScanShape(2, 50, 256, 32, 8, 2), torch.float32, 0),
    ("c0_layout_reverse", ScanShape(2, 20, 256, 16, 4, 4), torch.float32, 1),
    # TMA boxes of the last, ragged chunk reach past the end of the tensor
    ("c1_layout_bidir_bf16_ragged", ScanShape(3, 37, 256, 32, 16, 4), torch.bfloat16, 2),
    ("c3_layout_reverse_bf16_ragged", ScanShape(3, 29, 256, 32, 8, 2), torch.bfloat16, 1),
]


@pytest.mark.parametrize("name,shape,dtype,direction", BULK_CASES, ids=[c[0] for c in BULK_CASES])
def test_bulk_staging_equals_cp_async_staging(name, shape, dtype, direction, monkeypatch):
    """Whole channel tiles with 16-byte aligned rows are staged with bulk
    asynchronous copies; the element-wise cp.async path (M3_NO_BULK) must give
    the same bits for the output and every gradient."""
    inp = make_scan_inputs(shape, seed=19, dtype=dtype)
    runs = []
    for no_bulk in (False, True):
        if no_bulk:
            monkeypatch.setenv("M3_NO_BULK", "1")
        else:
            monkeypatch.delenv("M3_NO_BULK", raising=False)
        runs.append(run_m3(inp, direction, dtype))
    (y0, g0), (y1, g1) = runs
    assert torch.equal(y0, y1)
    for k in GRAD_KEYS:
        if g0[k] is not None:
            assert torch.equal(g0[k], g1[k]), k
    assert S.device_error() == 0


def test_verify_gate_passes():
    """The drop-in module's gate (triton_scan.verify's counterpart), thorough
    configuration list: forward and all gradients vs the float64 recurrence."""
    assert S.verify(device="cuda", thorough=True, verbose=False) is True


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_backward_grad_outputs_off_16_byte_boundary(dtype):
    """d_delta/d_u that start off a 16-byte boundary (views into a larger
    buffer) are written by the element-wise flush; the results equal those of
    aligned outputs, which take the vector-store flush, bit for bit."""
    from redpanda_b200.scan import ScanPlan, pad_params
    B, L, D, N, NR = 2, 64, 256, 32, 16
    sh = ScanShape(B, L, D, N, N - NR, 4)
    inp = to_cuda(make_scan_inputs(sh, seed=23, dtype=dtype))
    dev = inp["u"].device
    Ar, Ai, Tk = (t.contiguous() for t in pad_params(inp["A_real"], inp["A_imag"],
                                                     inp["track"], NR, N, D, dev))
    plan = ScanPlan(B, L, D, N, NR, dtype, dtype, S.M3_DIR_BIDIR)
    y = torch.empty(B, L, D, device=dev)
    ckpt = torch.empty(plan.ckpt_floats(), device=dev)
    args = (inp["delta"], inp["u"], inp["Bc"], inp["Cc"], Ar, Ai, Tk)
    plan.forward(*args, y, ckpt)
    dy = torch.randn(B, L, D, device=dev).to(dtype)
    outs = []
    for shift in (0, 1):   # elements: 2 or 4 bytes off the allocation's alignment
        flat = torch.empty(2, B * L * D + 8, device=dev, dtype=dtype)
        gd = flat[0, shift:shift + B * L * D].view(B, L, D)
        gu = flat[1, shift:shift + B * L * D].view(B, L, D)
        gB, gC = torch.empty_like(inp["Bc"]), torch.empty_like(inp["Cc"])
        gA = torch.empty(3, D, N, device=dev)
        ws = torch.empty(plan.workspace_bytes(), device=dev, dtype=torch.uint8)
        plan.backward(*args, dy, ckpt, gd, gu, gB, gC, gA[0], gA[1], gA[2], ws)
        outs.append((gd.clone(), gu.clone(), gB, gC, gA))
    torch.cuda.synchronize()
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
    assert S.device_error() == 0


BF16_Y_CASES = [
    ("bulk_bidir", ScanShape(2, 37, 256, 32, 16, 4), torch.bfloat16, 2),
    ("bulk_causal", ScanShape(2, 40, 256, 32, 8, 2), torch.bfloat16, 0),
    ("bulk_reverse_f32_inputs", ScanShape(2, 29, 256, 32, 16, 4), torch.float32, 1),
    ("elementwise_bidir_odd_D", ScanShape(2, 20, 40, 16, 4, 2), torch.float32, 2),
]


@pytest.mark.parametrize("name,shape,dtype,direction", BF16_Y_CASES,
                         ids=[c[0] for c in BF16_Y_CASES])
def test_bf16_y_output(name, shape, dtype, direction, monkeypatch):
    """y stored in bf16 (m3_scan_fwd_typed): one direction rounds the same fp32
    value the fp32 output holds; the bidirectional pair rounds the first
    direction's partial and then the sum (at most one bf16 ulp more); the
    gradients are those of the fp32-y scan fed the same (bf16) dy."""
    inp = make_scan_inputs(shape, seed=29, dtype=dtype)
    g = to_cuda(inp)
    nr = shape.n_rot
    fn = _FN[direction]
    args = (g["delta"], g["u"], g["Bc"], g["Cc"], g["A_real"], g["A_imag"], g["track"], nr,
            shape.d_state)
    with torch.no_grad():
        y32 = fn(*args)
        y16 = fn(*args, y_dtype=torch.bfloat16)
    assert y16.dtype == torch.bfloat16
    if direction != 2:
        assert torch.equal(y16, y32.to(torch.bfloat16))
    else:
        # the first pass (the reverse direction) is rounded to bf16, then the
        # sum: |err| <= half a bf16 ulp of each (ulp(x) = 2^(floor(log2|x|) - 7))
        with torch.no_grad():
            yrev = S.m3_reverse_scan(*args)
        def half_ulp(x):
            return torch.pow(2.0, torch.floor(torch.log2(x.abs().clamp(min=1e-30))) - 8)
        bound = half_ulp(yrev) + half_ulp(y32) + 1e-6 * y32.abs().max()
        assert bool(((y16.float() - y32).abs() <= bound).all())
    # gradients with a bf16 y equal the fp32-y scan's for the same dy
    dy = g["dy"].to(torch.bfloat16)
    grads = []
    for yd in (torch.float32, torch.bfloat16):
        lv = {k: g[k].clone().requires_grad_(True) for k in ("delta", "u", "Bc", "Cc")}
        y = fn(lv["delta"], lv["u"], lv["Bc"], lv["Cc"], g["A_real"], g["A_imag"], g["track"],
               nr, shape.d_state, y_dtype=yd)
        y.backward(dy.to(yd))
        grads.append([lv[k].grad for k in ("delta", "u", "Bc", "Cc")])
    for a, b in zip(*grads):
        assert torch.equal(a, b)
    assert S.device_error() == 0


@pytest.mark.parametrize("types", [("f32", "bf16", "bf16", "bf16"), ("bf16", "bf16", "bf16", "bf16"),
                                   ("f32", "f32", "bf16", "f32"), ("bf16", "f32", "f32", "f32")])
def test_gate_typed_matches_torch(types):
    """(y + c*u*D) * silu(z) with an element type per operand, against the
    same formula in fp32 torch on the widened operands (out rounded once)."""
    dt = {"f32": torch.float32, "bf16": torch.bfloat16}
    ty, tu, tz, to = (dt[t] for t in types)
    rows, D = 300, 136
    gen = torch.Generator("cuda").manual_seed(3)
    y = torch.randn(rows, D, device="cuda", generator=gen).to(ty)
    u = torch.randn(rows, D, device="cuda", generator=gen).to(tu)
    zf = torch.randn(rows, 2 * D, device="cuda", generator=gen).to(tz)
    z = zf[:, D:]                                   # row-strided view, as in the layer
    ds = torch.randn(D, device="cuda", generator=gen)
    out = S.m3_gate(y, u, z, ds, 2.0, out_dtype=to)
    ref = (y.float() + 2.0 * (u.float() * ds)) * (z.float() / (1 + torch.exp(-z.float())))
    assert out.dtype == to
    if to == torch.float32:
        assert rel_err(out, ref) <= 1e-6
    else:
        assert _bf16_ok(out, ref)


@pytest.mark.parametrize("shape,dtype,direction", [
    (ScanShape(8, 64, 256, 16, 4, 4), torch.float32, 0),      # config 0
    (ScanShape(2, 48, 256, 32, 16, 4), torch.bfloat16, 2),    # config-1 lane layout
    (ScanShape(1, 40, 512, 32, 8, 2), torch.float32, 0),      # config 3, one board
], ids=["c0_causal", "c1_layout_bidir", "c3_layout_one_row"])
def test_small_batch_tiling_matches_regular_tiling(shape, dtype, direction):
    """A batch too small to fill the GPU runs the small-batch tiling (2
    channels per thread); the same rows inside a large batch run the regular
    one.  y, dΔ and du must be the same bits; dB/dC and dA, whose sums follow
    the tiling's partition, within the gradient bar."""
    big = ScanShape(512, shape.seqlen, shape.d_inner, shape.d_state, shape.n_track,
                    shape.mimo_p)
    inp = make_scan_inputs(big, seed=31, dtype=dtype)
    rows = shape.batch
    small = {k: (v[:rows] if v is not None and v.dim() == 3 else v) for k, v in inp.items()}
    ys, gs_ = run_m3(small, direction, dtype)
    yb, gb = run_m3(inp, direction, dtype)
    assert torch.equal(ys, yb[:rows])
    for k in ("delta", "u"):
        assert torch.equal(gs_[k], gb[k][:rows]), k
    for k in ("Bc", "Cc"):
        assert rel_err(gs_[k].float(), gb[k][:rows].float()) <= (1e-2 if dtype == torch.bfloat16
                                                                 else GRAD_TOL), k
    # dA of the small batch equals the large batch's restricted to those rows
    # only as a sum; compare it with the oracle instead
    inp32 = {k: (None if v is None else v.float()) for k, v in small.items()}
    _, g32 = oracle_scan(inp32, direction, torch.float32)
    for k in ("A_real", "A_imag", "track"):
        if gs_[k] is not None:
            assert rel_err(gs_[k], g32[k]) <= 2e-6, k
    assert S.device_error() == 0


def test_param_grads_at_large_batch_vs_float64():
    """dA_real, dA_imag and dtrack are sums over every (row, step) of the batch.
    At B=2048 (config-2 lane layout, bidirectional, bf16 inputs) each backward
    CTA accumulates ~170 rows x 128 steps in fp32; the float64 reference is the
    oracle run on the GPU in float64 over blocks of 128 rows and summed."""
    sh = ScanShape(2048, 64, 256, 32, 16, 4)
    inp = make_scan_inputs(sh, seed=37, dtype=torch.bfloat16)
    _, g = run_m3(inp, 2, torch.bfloat16)
    acc = {k: None for k in ("A_real", "A_imag", "track")}
    dev = torch.device("cuda")
    for r0 in range(0, sh.batch, 128):
        blk = {k: (None if v is None else
                   (v[r0:r0 + 128] if v.dim() == 3 else v).to(dev, torch.float64))
               for k, v in inp.items()}
        _, gb = oracle_scan(blk, 2, torch.float64)
        for k in acc:
            acc[k] = gb[k] if acc[k] is None else acc[k] + gb[k]
    worst = 0.0
    for k in acc:
        e = rel_err(g[k], acc[k])
        PARITY_TABLE.append(("B2048_bidir_bf16", "d" + k, "fp32", float("nan"), e, float("nan"),
                             "ok" if e <= GRAD_TOL else "FAIL"))
        worst = max(worst, e)
    assert worst <= GRAD_TOL, worst
