"""The O(1) step kernel: bit-exact against the scan kernel at every position,
within tolerance of the reference step, and row-independent (the batched-step
gate of redpanda/engine/mars_diagnostics.py:94-164)."""

import pytest
import torch

import oracle as O
from helpers import rel_err, to_cuda
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
