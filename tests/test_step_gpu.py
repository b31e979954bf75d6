"""The O(1) step kernel: bit-exact against the scan kernel at every position,
within tolerance of the reference step, and row-independent (the batched-step
gate of redpanda/engine/mars_diagnostics.py:94-164)."""

import pytest
import torch

import oracle as O
from helpers import WIDE_REGIMES, gate_arg_stats, rel_err, to_cuda, wide_gate_inputs
from redpanda_b200 import scan as S
from redpanda_b200.synthetic import ScanShape, make_scan_inputs

pytestmark = pytest.mark.gpu

SHAPES = [
    ScanShape(4, 40, 1024, 32, 8, 2),    # config-3 state layout
    ScanShape(3, 20, 256, 16, 4, 4),     # config-0 layout
    ScanShape(2, 9, 64, 8, 2, 2),        # virtual lanes (6 rot + 2 track)
    ScanShape(2, 35, 96, 32, 16, 4),     # config-1 layout, L past two checkpoints
    ScanShape(2, 17, 40, 64, 16, 4),     # N=64, D not a multiple of 32
]


def _step_all(g, sh, h=None, dbu=None, start=0):
    B, D, N = sh.batch, sh.d_inner, sh.d_state
    h = torch.zeros(B, D, N, device="cuda") if h is None else h
    dbu = torch.zeros_like(h) if dbu is None else dbu
    ys = []
    for t in range(start, sh.seqlen):
        ys.append(S.m3_step_(h, dbu, g["delta"][:, t], g["u"][:, t], g["Bc"][:, t], g["Cc"][:, t],
                             g["A_real"], g["A_imag"], g["track"], sh.n_rot, N))
    return torch.stack(ys, 1), h, dbu


@pytest.mark.parametrize("sh", SHAPES, ids=lambda s: f"B{s.batch}L{s.seqlen}D{s.d_inner}N{s.d_state}")
def test_step_bit_exact_vs_scan_every_position(sh):
    g = to_cuda(make_scan_inputs(sh, seed=3))
    y, (h, dbu) = S.m3_scan_with_state(g["delta"], g["u"], g["Bc"], g["Cc"], g["A_real"],
                                       g["A_imag"], g["track"], sh.n_rot, sh.d_state)
    ys, hs, ds = _step_all(g, sh)
    assert torch.equal(ys, y)
    assert torch.equal(hs, h)
    assert torch.equal(ds, dbu)


WIDE_STEP_SHAPES = [
    ScanShape(3, 40, 256, 32, 8, 2),     # config-3 state layout
    ScanShape(2, 24, 128, 32, 16, 4),    # config-1 layout
    ScanShape(2, 20, 96, 16, 4, 4),      # config-0 layout, D not a multiple of 64
]


@pytest.mark.parametrize("regime", WIDE_REGIMES)
@pytest.mark.parametrize("sh", WIDE_STEP_SHAPES,
                         ids=lambda s: f"B{s.batch}L{s.seqlen}D{s.d_inner}N{s.d_state}")
def test_step_bit_exact_vs_scan_wide_gate_arguments(sh, regime):
    """Step == scan at every position, bit for bit, when the gate arguments
    |delta*A_imag| cover the packed path with |k| >= 2, the checked path and the
    double-precision slow path (helpers.wide_gate_inputs); the factored step
    too."""
    inp = wide_gate_inputs(sh, 43, regime)
    _, kmax, _ = gate_arg_stats(inp)
    assert kmax >= 2
    g = to_cuda(inp)
    y, (h, dbu) = S.m3_scan_with_state(g["delta"], g["u"], g["Bc"], g["Cc"], g["A_real"],
                                       g["A_imag"], g["track"], sh.n_rot, sh.d_state)
    ys, hs, ds = _step_all(g, sh)
    assert torch.equal(ys, y)
    assert torch.equal(hs, h)
    assert torch.equal(ds, dbu)
    hf = torch.zeros_like(hs)
    fa = torch.zeros(sh.batch, sh.d_inner + sh.d_state, device="cuda")
    fb = torch.empty_like(fa)
    for t in range(sh.seqlen):
        yt = S.m3_step_factored_(hf, fa, fb, g["delta"][:, t], g["u"][:, t], g["Bc"][:, t],
                                 g["Cc"][:, t], g["A_real"], g["A_imag"], g["track"], sh.n_rot,
                                 sh.d_state)
        assert torch.equal(yt, y[:, t]), t
        fa, fb = fb, fa
    assert torch.equal(hf, h)
    assert torch.isfinite(y).all()
    assert S.device_error() == 0


def test_step_continues_a_primed_prefix_bit_exactly():
    """prime (scan with state over a prefix) then step == scan of the whole line."""
    sh = ScanShape(4, 48, 1024, 32, 8, 2)
    g = to_cuda(make_scan_inputs(sh, seed=8))
    y = S.m3_trapezoidal_scan(g["delta"], g["u"], g["Bc"], g["Cc"], g["A_real"], g["A_imag"],
                              g["track"], sh.n_rot, sh.d_state)
    for k in (1, 16, 17, 33):
        pre = {key: (v[:, :k] if v is not None and v.dim() == 3 and v.shape[1] == sh.seqlen else v)
               for key, v in g.items()}
        _, (h, dbu) = S.m3_scan_with_state(pre["delta"], pre["u"], pre["Bc"], pre["Cc"],
                                           g["A_real"], g["A_imag"], g["track"], sh.n_rot,
                                           sh.d_state)
        ys, _, _ = _step_all(g, sh, h.clone(), dbu.clone(), start=k)
        assert torch.equal(ys, y[:, k:]), k


def test_step_matches_reference_step():
    sh = ScanShape(3, 6, 128, 32, 8, 2)
    inp = make_scan_inputs(sh, seed=9)
    g = to_cuda(inp)
    ys, hs, ds = _step_all(g, sh)
    h = torch.zeros(3, 128, 32)
    dbu = torch.zeros_like(h)
    for t in range(sh.seqlen):
        yr, h, dbu = O.step_cells(h, dbu, inp["delta"][:, t], inp["u"][:, t], inp["Bc"][:, t],
                                  inp["Cc"][:, t], inp["A_real"], inp["A_imag"], inp["track"])
        assert rel_err(ys[:, t], yr) <= 1e-5
    assert rel_err(hs, h) <= 1e-5 and rel_err(ds, dbu) <= 1e-5


def test_batched_step_equals_single_row_steps():
    """Gate (a)/(b) of mars_diagnostics.py:110-143: batched == per-row, over a chain of 8."""
    sh = ScanShape(6, 8, 256, 32, 8, 2)
    g = to_cuda(make_scan_inputs(sh, seed=12))
    h0 = torch.randn(6, 256, 32, device="cuda") * 0.1
    d0 = torch.randn(6, 256, 32, device="cuda") * 0.1
    yb, hb, db = _step_all(g, sh, h0.clone(), d0.clone())
    for r in range(6):
        gr = {k: (v[r:r + 1] if v is not None and v.shape[0] == 6 else v) for k, v in g.items()}
        shr = ScanShape(1, 8, 256, 32, 8, 2)
        yr, hr, dr = _step_all(gr, shr, h0[r:r + 1].clone(), d0[r:r + 1].clone())
        assert torch.equal(yr, yb[r:r + 1])
        assert torch.equal(hr, hb[r:r + 1]) and torch.equal(dr, db[r:r + 1])
    assert torch.isfinite(yb).all()


def test_functional_step_does_not_mutate_input_state():
    sh = ScanShape(2, 1, 64, 16, 4, 2)
    g = to_cuda(make_scan_inputs(sh, seed=1))
    h = torch.randn(2, 64, 16, device="cuda")
    d = torch.randn(2, 64, 16, device="cuda")
    hc, dc = h.clone(), d.clone()
    _, (h2, d2) = S.m3_step((h, d), g["delta"][:, 0], g["u"][:, 0], g["Bc"][:, 0], g["Cc"][:, 0],
                            g["A_real"], g["A_imag"], g["track"], sh.n_rot, 16)
    assert torch.equal(h, hc) and torch.equal(d, dc)
    assert not torch.equal(h2, h)


@pytest.mark.parametrize("sh", SHAPES, ids=lambda s: f"B{s.batch}L{s.seqlen}D{s.d_inner}N{s.d_state}")
def test_factored_step_equals_full_step_and_scan(sh):
    """The factored state (h, [delta*u | B]) reproduces the full-state step and
    the scan bit for bit."""
    g = to_cuda(make_scan_inputs(sh, seed=5))
    k = max(1, sh.seqlen // 2)
    pre = {key: (v[:, :k] if v is not None and v.dim() == 3 and v.shape[1] == sh.seqlen else v)
           for key, v in g.items()}
    y, (h, dbu) = S.m3_scan_with_state(g["delta"], g["u"], g["Bc"], g["Cc"], g["A_real"],
                                       g["A_imag"], g["track"], sh.n_rot, sh.d_state)
    _, (hk, dk) = S.m3_scan_with_state(pre["delta"], pre["u"], pre["Bc"], pre["Cc"],
                                       g["A_real"], g["A_imag"], g["track"], sh.n_rot,
                                       sh.d_state)
    hf = hk.clone()
    fa = S.factored_state(pre["delta"], pre["u"], pre["Bc"])
    fb = torch.empty_like(fa)
    hfull, dfull = hk.clone(), dk.clone()
    for t in range(k, sh.seqlen):
        args = (g["delta"][:, t], g["u"][:, t], g["Bc"][:, t], g["Cc"][:, t], g["A_real"],
                g["A_imag"], g["track"], sh.n_rot, sh.d_state)
        yf = S.m3_step_factored_(hf, fa, fb, *args)
        ys = S.m3_step_(hfull, dfull, *args)
        assert torch.equal(yf, ys)
        assert torch.equal(yf, y[:, t])
        fa, fb = fb, fa
    assert torch.equal(hf, h) and torch.equal(hfull, h)
    # the final factors rebuild the scan's dBu exactly
    D = sh.d_inner
    rebuilt = fa[:, :D, None] * fa[:, None, D:]
    assert torch.equal(rebuilt, dbu)


def test_factored_step_rejects_aliased_factors():
    sh = ScanShape(2, 1, 64, 16, 4, 2)
    g = to_cuda(make_scan_inputs(sh, seed=1))
    h = torch.zeros(2, 64, 16, device="cuda")
    fac = torch.zeros(2, 64 + 16, device="cuda")
    with pytest.raises(RuntimeError, match="distinct"):
        S.m3_step_factored_(h, fac, fac, g["delta"][:, 0], g["u"][:, 0], g["Bc"][:, 0],
                            g["Cc"][:, 0], g["A_real"], g["A_imag"], g["track"], sh.n_rot, 16)


@pytest.mark.parametrize("sh", SHAPES[:3], ids=lambda s: f"B{s.batch}D{s.d_inner}N{s.d_state}")
def test_bf16_inputs_step_bit_exact_vs_scan(sh):
    g = to_cuda(make_scan_inputs(sh, seed=13, dtype=torch.bfloat16))
    y, (h, dbu) = S.m3_scan_with_state(g["delta"], g["u"], g["Bc"], g["Cc"], g["A_real"],
                                       g["A_imag"], g["track"], sh.n_rot, sh.d_state)
    ys, hs, ds = _step_all(g, sh)
    assert torch.equal(ys, y) and torch.equal(hs, h) and torch.equal(ds, dbu)


def _offset_copy(t, dtype=None):
    """A copy of ``t`` whose data starts one element past a 16-byte boundary."""
    t = t if dtype is None else t.to(dtype)
    flat = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
    out = flat[1:].view(t.shape)
    out.copy_(t)
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_unaligned_rows_take_the_scalar_path_with_equal_results(dtype):
    """B/C rows and factors that are only element-aligned give the same bits."""
    sh = ScanShape(4, 6, 256, 32, 8, 2)
    g = to_cuda(make_scan_inputs(sh, seed=21, dtype=dtype))
    B, D, N = sh.batch, sh.d_inner, sh.d_state
    h0 = torch.randn(B, D, N, device="cuda") * 0.1
    fa0 = torch.randn(B, D + N, device="cuda")
    d0 = fa0[:, :D, None] * fa0[:, None, D:]
    outs = []
    for shift in (False, True):
        h, dbu = h0.clone(), d0.clone()
        hf, fa = h0.clone(), fa0.clone()
        fb = torch.empty_like(fa)
        if shift:
            fa, fb = _offset_copy(fa), _offset_copy(fb)
        ys = []
        for t in range(sh.seqlen):
            bc, cc = g["Bc"][:, t].contiguous(), g["Cc"][:, t].contiguous()
            if shift:
                bc, cc = _offset_copy(bc), _offset_copy(cc)
                assert bc.data_ptr() % 16 != 0
            args = (g["delta"][:, t], g["u"][:, t], bc, cc, g["A_real"], g["A_imag"],
                    g["track"], sh.n_rot, N)
            y1 = S.m3_step_(h, dbu, *args)
            y2 = S.m3_step_factored_(hf, fa, fb, *args)
            assert torch.equal(y1, y2)
            ys.append(y1)
            fa, fb = fb, fa
        outs.append((torch.stack(ys, 1), h, dbu, hf))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("n_track", [8, 16])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_pipelined_step_equals_register_path(n_track, dtype, monkeypatch):
    """Aligned dense tiles go through the bulk-copy pipeline (several row pairs
    per CTA, so every stage is reused, and an odd last row), 32-lane tiles with
    swizzled 2D TMA state tiles; the 1D bulk rows (M3_NO_SWIZZLE) and the
    per-row register path (M3_NO_BULK) must give the same bits, for the full
    and the factored state, over several consecutive steps."""
    B, D, N, steps = 301, 1024, 32, 5
    gen = torch.Generator().manual_seed(31)
    sh = ScanShape(B, steps, D, N, n_track, 2)
    g = to_cuda(make_scan_inputs(sh, seed=17, dtype=dtype))
    h0 = (torch.randn(B, D, N, generator=gen) * 0.1).cuda()
    fa0 = torch.randn(B, D + N, generator=gen).cuda()
    d0 = fa0[:, :D, None] * fa0[:, None, D:]
    runs = []
    # TMA 2D with the 128-byte swizzle (32-lane tiles), 1D bulk rows, register path
    for mode in ("swizzle", "bulk", "register"):
        monkeypatch.delenv("M3_NO_BULK", raising=False)
        monkeypatch.delenv("M3_NO_SWIZZLE", raising=False)
        if mode != "swizzle":
            monkeypatch.setenv("M3_NO_SWIZZLE", "1")
        if mode == "register":
            monkeypatch.setenv("M3_NO_BULK", "1")
        h, dbu, hf, fa = h0.clone(), d0.clone(), h0.clone(), fa0.clone()
        fb = torch.empty_like(fa)
        ys, yfs = [], []
        for t in range(steps):
            args = (g["delta"][:, t], g["u"][:, t], g["Bc"][:, t], g["Cc"][:, t], g["A_real"],
                    g["A_imag"], g["track"], sh.n_rot, N)
            ys.append(S.m3_step_(h, dbu, *args))
            yfs.append(S.m3_step_factored_(hf, fa, fb, *args))
            fa, fb = fb, fa
        torch.cuda.synchronize()
        runs.append((torch.stack(ys), torch.stack(yfs), h, dbu, hf, fa))
    for other in runs[1:]:
        for a, b in zip(runs[0], other):
            assert torch.equal(a, b)
    assert torch.equal(runs[0][0], runs[0][1])
    assert S.device_error() == 0
