"""The scan with the layer's prologue fused into its staging (m3_scan_fwd_fused).

The fused forward reads the raw projections -- dt (before softplus) and the
x_proj rows holding B_raw and C_raw -- and applies softplus, BCNorm and the MIMO
fold (redpanda/engine/mamba.py:284-301, 336-337) as each chunk lands.  Its
results must equal, bit for bit, the unfused bf16 layer: the standalone
prologue (m3_step_inputs, fp32), a cast of delta/Bc/Cc to bf16, and the scan.
"""

import ctypes

import pytest
import torch

from redpanda_b200 import _lib
from redpanda_b200 import scan as S
from redpanda_b200.scan import ScanPlan, pad_params

pytestmark = pytest.mark.gpu

BF = torch.bfloat16

CASES = [
    # name, B, L, D, N, n_track, p, dt_rank, direction, y dtype, BCNorm weights
    ("c1_layout_bidir", 3, 37, 256, 32, 16, 4, 48, S.M3_DIR_BIDIR, torch.float32, True),
    ("c1_layout_causal_y_bf16", 2, 64, 256, 32, 16, 4, 48, S.M3_DIR_FWD, BF, True),
    ("c3_layout_reverse", 2, 29, 256, 32, 8, 2, 32, S.M3_DIR_REV, torch.float32, True),
    ("no_bcnorm_bidir_y_bf16", 2, 40, 128, 32, 16, 4, 16, S.M3_DIR_BIDIR, BF, False),
]


def make(B, L, D, N, nt, p, dt_rank, seed, weights):
    g = torch.Generator("cuda").manual_seed(seed)
    ld_x = dt_rank + 2 * N * p
    dt = (torch.randn(B, L, D, device="cuda", generator=g) * 1.5 - 2.5).to(BF)
    x_dbl = torch.randn(B, L, ld_x, device="cuda", generator=g).to(BF)
    u = torch.randn(B, L, D, device="cuda", generator=g).to(BF)
    nr = N - nt
    ar = -torch.exp(torch.randn(D, nr, device="cuda", generator=g) * 0.5)
    ai = (torch.rand(D, nr, device="cuda", generator=g) * 2 - 1) * 3.14159
    tk = torch.tanh(torch.randn(D, nt, device="cuda", generator=g))
    wb = wc = None
    if weights:
        wb = 1 + 0.3 * torch.randn(N * p, device="cuda", generator=g)
        wc = 1 + 0.3 * torch.randn(N * p, device="cuda", generator=g)
    return dt, x_dbl, u, (ar, ai, tk), wb, wc


def unfused_inputs(dt, x_dbl, wb, wc, N, p, dt_rank):
    B, L, D = dt.shape
    rows = B * L
    delta, bc, cc = S.m3_step_inputs(dt.float().reshape(rows, D),
                                     x_dbl.float().reshape(rows, -1), dt_rank,
                                     dt_rank + N * p, wb, wc, 1e-5, N, p)
    return (delta.view(B, L, D).to(BF), bc.view(B, L, N).to(BF), cc.view(B, L, N).to(BF))


def fused_forward(plan, dt, x_dbl, u, P, wb, wc, N, p, dt_rank, y, ckpt):
    lib = _lib.load()
    rc = lib.m3_scan_fwd_fused(
        ctypes.byref(plan.desc), p, dt.data_ptr(), x_dbl.data_ptr(), x_dbl.shape[-1], dt_rank,
        dt_rank + N * p, None if wb is None else wb.data_ptr(),
        None if wc is None else wc.data_ptr(), 1e-5, u.data_ptr(), P[0].data_ptr(),
        P[1].data_ptr(), P[2].data_ptr(), y.data_ptr(), S._dt_code(y.dtype),
        None if ckpt is None else ckpt.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.strerror(rc)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_fused_forward_equals_unfused(case):
    name, B, L, D, N, nt, p, dt_rank, direction, ydt, weights = case
    dt, x_dbl, u, (ar, ai, tk), wb, wc = make(B, L, D, N, nt, p, dt_rank, 5, weights)
    nr = N - nt
    P = [t.contiguous() for t in pad_params(ar, ai, tk, nr, N, D, dt.device)]
    plan = ScanPlan(B, L, D, N, nr, BF, BF, direction)
    delta, bc, cc = unfused_inputs(dt, x_dbl, wb, wc, N, p, dt_rank)
    nck = plan.ckpt_floats()
    y0 = torch.empty(B, L, D, device="cuda", dtype=ydt)
    c0 = torch.empty(max(nck, 1), device="cuda")
    plan.forward(delta, u, bc, cc, *P, y0, c0 if nck else None)
    y1 = torch.empty_like(y0)
    c1 = torch.empty_like(c0)
    fused_forward(plan, dt, x_dbl, u, P, wb, wc, N, p, dt_rank, y1, c1 if nck else None)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
    if nck:
        assert torch.equal(c0, c1)
    assert torch.isfinite(y1.float()).all()
    assert S.device_error() == 0


def test_fused_forward_refuses_unaligned_columns():
    B, L, D, N, nt, p = 2, 16, 128, 32, 16, 4
    dt, x_dbl, u, (ar, ai, tk), wb, wc = make(B, L, D, N, nt, p, 12, 6, True)
    P = [t.contiguous() for t in pad_params(ar, ai, tk, N - nt, N, D, dt.device)]
    plan = ScanPlan(B, L, D, N, N - nt, BF, BF, S.M3_DIR_FWD)
    y = torch.empty(B, L, D, device="cuda")
    lib = _lib.load()
    rc = lib.m3_scan_fwd_fused(ctypes.byref(plan.desc), p, dt.data_ptr(), x_dbl.data_ptr(),
                               x_dbl.shape[-1], 12, 12 + N * p, wb.data_ptr(), wc.data_ptr(),
                               1e-5, u.data_ptr(), P[0].data_ptr(), P[1].data_ptr(),
                               P[2].data_ptr(), y.data_ptr(), 0, None,
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 4   # M3_ERR_UNSUPPORTED: column offset 12 is off an 8-element boundary


_SCAN = {S.M3_DIR_FWD: S.m3_trapezoidal_scan, S.M3_DIR_REV: S.m3_reverse_scan,
         S.M3_DIR_BIDIR: S.m3_bidir_scan}


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_fused_backward_equals_unfused(case):
    """Every gradient of the fused pair (dt, x_dbl, BCNorm weights, u, the
    eigenvalues) equals the unfused autograd chain's bit for bit: softplus,
    BCNorm and fold in fp32 (m3_step_inputs and its backward), the casts to
    bf16, the scan and its backward."""
    name, B, L, D, N, nt, p, dt_rank, direction, ydt, weights = case
    dt0, x0, u0, (ar0, ai0, tk0), wb0, wc0 = make(B, L, D, N, nt, p, dt_rank, 7, weights)
    dy = torch.randn(B, L, D, device="cuda", generator=torch.Generator("cuda").manual_seed(8))
    nr = N - nt
    runs = []
    for fused in (False, True):
        leaf = lambda t: None if t is None else t.clone().requires_grad_(True)  # noqa: E731
        dt, x, u, ar, ai, tk, wb, wc = (leaf(t) for t in (dt0, x0, u0, ar0, ai0, tk0, wb0, wc0))
        if fused:
            y = S.m3_fused_scan(dt, x, wb, wc, 1e-5, u, ar, ai, tk, nr, N, p, dt_rank,
                                dt_rank + N * p, direction, y_dtype=ydt)
        else:
            rows = B * L
            delta, bc, cc = S.step_inputs(dt.float().reshape(rows, D), x.float().reshape(rows, -1),
                                          dt_rank, dt_rank + N * p, wb, wc, 1e-5, N, p)
            y = _SCAN[direction](delta.view(B, L, D).to(BF), u, bc.view(B, L, N).to(BF),
                                 cc.view(B, L, N).to(BF), ar, ai, tk, nr, N, y_dtype=ydt)
        (y.float() * dy).sum().backward()
        runs.append((y.detach(), [None if t is None else t.grad
                                  for t in (dt, x, u, ar, ai, tk, wb, wc)]))
    (ya, ga), (yb, gb) = runs
    assert torch.equal(ya, yb)
    for k, (a, b) in enumerate(zip(ga, gb)):
        if a is None:
            assert b is None
            continue
        assert torch.equal(a, b), ("dt", "x_dbl", "u", "A_real", "A_imag", "track", "wb", "wc")[k]
    assert S.device_error() == 0


@pytest.mark.parametrize("bidir,n_track,p", [(True, 16, 4), (False, 8, 2)])
def test_model_bf16_fused_prologue_equals_unfused(bidir, n_track, p, monkeypatch):
    """A bf16 (autocast) Mamba trains and infers identically with the prologue
    fused into the scan kernels or run as its own launch before them."""
    from redpanda_b200.mamba import Mamba, Mamba3Block, MambaConfig
    torch.manual_seed(4)
    cfg = MambaConfig(d_model=128, n_layer=2, d_state=32, n_track_state=n_track, mimo_p=p,
                      vocab_size=64, bidirectional=bidir)
    model = Mamba(cfg).cuda()
    with torch.no_grad():   # non-zero rotation phases
        for layer in model.layers:
            layer["mixer"].A_phase.uniform_(-1.4, 1.4)
    ids = torch.randint(0, 64, (3, 40), device="cuda")
    taken = []
    orig = Mamba3Block._fused_scan

    def spy(self, *a, **k):
        r = orig(self, *a, **k)
        taken.append(r is not None)
        return r
    monkeypatch.setattr(Mamba3Block, "_fused_scan", spy)
    runs = []
    for fused in (False, True):
        monkeypatch.setattr(Mamba3Block, "fuse_prologue", fused)
        model.zero_grad(set_to_none=True)
        model.train()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = model(ids)
        y.float().pow(2).mean().backward()
        model.eval()
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            yi = model(ids)
        runs.append((y.detach(), yi, {k: q.grad.clone() for k, q in model.named_parameters()}))
    assert taken and all(taken[len(taken) // 2:])   # the fused kernels ran in the second pass
    (ya, ia, ga), (yb, ib, gb) = runs
    assert torch.equal(ya, yb) and torch.equal(ia, ib)
    for k in ga:
        assert torch.equal(ga[k], gb[k]), k
