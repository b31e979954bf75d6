"""The fused step layer: m3_step_inputs (softplus, BCNorm, MIMO fold in one
launch) and m3_step_gated (the step with the gated output (y + u*D) * silu(z)),
against the torch formulation of Mamba3Block.step (redpanda/engine/mamba.py:427-498)."""

import pytest
import torch
import torch.nn.functional as F

from redpanda_b200 import scan as S
from redpanda_b200.mamba import Mamba, MambaConfig

pytestmark = pytest.mark.gpu

TOL = 1e-6


def _rel(a, b):
    a, b = a.detach().double(), b.detach().double()
    den = b.abs().max().item()
    return (a - b).abs().max().item() / (den if den > 0 else 1.0)


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


@pytest.mark.parametrize("bcnorm", [True, False])
@pytest.mark.parametrize("n,p", [(32, 2), (16, 4), (12, 2)])
def test_step_inputs_match_torch(bcnorm, n, p):
    g = torch.Generator(device="cuda").manual_seed(3)
    B, D, R = 37, 96, 8
    dt = torch.randn(B, D, device="cuda", generator=g) * 8     # both softplus branches
    x_dbl = torch.randn(B, R + 2 * n * p, device="cuda", generator=g)
    wb = torch.rand(n * p, device="cuda", generator=g) + 0.5 if bcnorm else None
    wc = torch.rand(n * p, device="cuda", generator=g) + 0.5 if bcnorm else None
    eps = 1e-5
    delta, bc, cc = S.m3_step_inputs(dt, x_dbl, R, R + n * p, wb, wc, eps, n, p)
    ref_d = F.softplus(dt)
    braw, craw = x_dbl[:, R:R + n * p], x_dbl[:, R + n * p:]
    if bcnorm:
        braw = braw * torch.rsqrt(braw.pow(2).mean(-1, keepdim=True) + eps) * wb
        craw = craw * torch.rsqrt(craw.pow(2).mean(-1, keepdim=True) + eps) * wc
    assert _rel(delta, ref_d) <= TOL
    assert _rel(bc, braw.reshape(B, n, p).sum(-1)) <= TOL
    assert _rel(cc, craw.reshape(B, n, p).sum(-1)) <= TOL


@pytest.mark.parametrize("D,pad", [(1024, 0), (96, 4), (90, 3)])
def test_step_inputs_bias_and_silu(D, pad):
    """m3_step_inputs with the dt_proj bias passed apart equals it on dt + bias
    (torch's matmul-then-add), on the float4 and the scalar path; m3_silu on a
    row-strided view equals torch's silu bit for bit."""
    g = torch.Generator(device="cuda").manual_seed(11)
    B, n, p, R = 19, 32, 2, 8
    base = torch.randn(B, D + pad, device="cuda", generator=g) * 6
    dt = base[:, :D]                                   # row stride D + pad
    bias = torch.randn(D, device="cuda", generator=g)
    x_dbl = torch.randn(B, R + 2 * n * p, device="cuda", generator=g)
    wb = torch.rand(n * p, device="cuda", generator=g) + 0.5
    wc = torch.rand(n * p, device="cuda", generator=g) + 0.5
    ref = S.m3_step_inputs((dt + bias).contiguous(), x_dbl, R, R + n * p, wb, wc, 1e-5, n, p)
    got = S.m3_step_inputs(dt, x_dbl, R, R + n * p, wb, wc, 1e-5, n, p, dt_bias=bias)
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    xz = torch.randn(B, 2 * D + pad, device="cuda", generator=g) * 5
    u = S.m3_silu(xz[:, :D])
    assert u.is_contiguous() and torch.equal(u, F.silu(xz[:, :D]))


@pytest.mark.parametrize("B,D,N,n_track", [(37, 256, 32, 8), (6, 40, 64, 16), (9, 128, 32, 16)])
def test_gated_step_equals_step_and_torch_epilogue(B, D, N, n_track):
    """Same state bits as m3_step_ / m3_step_factored_; output (y + u*D)*silu(z)."""
    g = torch.Generator(device="cuda").manual_seed(5)
    n_rot = N - n_track
    A_real = -torch.exp(torch.randn(D, n_rot, device="cuda", generator=g) * 0.5)
    A_imag = (torch.rand(D, n_rot, device="cuda", generator=g) * 2 - 1) * 3.14159
    track = torch.tanh(torch.randn(D, n_track, device="cuda", generator=g))
    params = tuple(t.contiguous() for t in S.pad_params(A_real, A_imag, track, n_rot, N, D,
                                                        torch.device("cuda")))
    h0 = torch.randn(B, D, N, device="cuda", generator=g) * 0.1
    fa0 = torch.randn(B, D + N, device="cuda", generator=g)
    d0 = fa0[:, :D, None] * fa0[:, None, D:]
    d_skip = torch.randn(D, device="cuda", generator=g)
    hr, dr = h0.clone(), d0.clone()
    hg, dg = h0.clone(), d0.clone()
    hf, fa = h0.clone(), fa0.clone()
    fb = torch.empty_like(fa)
    for _ in range(3):
        delta = F.softplus(torch.randn(B, D, device="cuda", generator=g) * 0.5 - 2)
        u = torch.randn(B, D, device="cuda", generator=g)
        bc = torch.randn(B, N, device="cuda", generator=g)
        cc = torch.randn(B, N, device="cuda", generator=g)
        xz = torch.randn(B, 2 * D, device="cuda", generator=g)
        z = xz[:, D:]                                          # row stride 2D
        y = S.m3_step_(hr, dr, delta, u, bc, cc, A_real, A_imag, track, n_rot, N)
        ref = (y + u * d_skip) * F.silu(z)
        out = S.m3_step_gated_((hg, dg), delta, u, bc, cc, params, n_rot, z, d_skip)
        outf = S.m3_step_gated_((hf, fa, fb), delta, u, bc, cc, params, n_rot, z, d_skip)
        fa, fb = fb, fa
        assert torch.equal(hg, hr) and torch.equal(dg, dr) and torch.equal(hf, hr)
        assert torch.equal(out, outf)
        assert _rel(out, ref) <= TOL
    assert S.device_error() == 0


@pytest.mark.parametrize("B,D,n_track,p,bcnorm", [(37, 256, 8, 2, True), (8, 1024, 16, 2, True),
                                                  (5, 64, 8, 2, False), (1, 128, 8, 1, True)])
def test_step_gated_fused_equals_inputs_then_gated(B, D, n_track, p, bcnorm):
    """m3_step_gated_fused (softplus, BCNorm, MIMO fold, recurrence and gated
    output in one launch) gives the bits of m3_step_inputs + m3_step_gated, for
    both state forms, odd batches (the last row pair half empty) and dt values
    on both sides of softplus' threshold."""
    g = torch.Generator(device="cuda").manual_seed(9)
    N, R = 32, 16
    n_rot = N - n_track
    A_real = -torch.exp(torch.randn(D, n_rot, device="cuda", generator=g) * 0.5)
    A_imag = (torch.rand(D, n_rot, device="cuda", generator=g) * 2 - 1) * 3.14159
    track = torch.tanh(torch.randn(D, n_track, device="cuda", generator=g))
    params = tuple(t.contiguous() for t in S.pad_params(A_real, A_imag, track, n_rot, N, D,
                                                        torch.device("cuda")))
    wb = torch.rand(N * p, device="cuda", generator=g) + 0.5 if bcnorm else None
    wc = torch.rand(N * p, device="cuda", generator=g) + 0.5 if bcnorm else None
    d_skip = torch.randn(D, device="cuda", generator=g)
    h0 = torch.randn(B, D, N, device="cuda", generator=g) * 0.1
    fa0 = torch.randn(B, D + N, device="cuda", generator=g)
    d0 = fa0[:, :D, None] * fa0[:, None, D:]
    hu, du_ = h0.clone(), d0.clone()
    hf, df = h0.clone(), d0.clone()
    hfa, fa, fb = h0.clone(), fa0.clone(), torch.empty_like(fa0)
    hua, ua, ub = h0.clone(), fa0.clone(), torch.empty_like(fa0)
    bias = torch.randn(D, device="cuda", generator=g)
    for it in range(3):
        dt = torch.randn(B, D, device="cuda", generator=g) * 2 - 3
        dt[:, ::17] += 24.0                                     # above the threshold
        x_dbl = torch.randn(B, R + 2 * N * p, device="cuda", generator=g)
        u = torch.randn(B, D, device="cuda", generator=g)
        z = torch.randn(B, 2 * D, device="cuda", generator=g)[:, D:]
        db = bias if it == 1 else None                          # dt_proj bias passed apart
        delta, bc, cc = S.m3_step_inputs(dt, x_dbl, R, R + N * p, wb, wc, 1e-5, N, p,
                                         dt_bias=db)
        ref = S.m3_step_gated_((hu, du_), delta, u, bc, cc, params, n_rot, z, d_skip)
        out = S.m3_step_gated_fused_((hf, df), dt, x_dbl, R, R + N * p, wb, wc, 1e-5, p, u,
                                     params, n_rot, z, d_skip, dt_bias=db)
        assert out is not None, "the fused step kernel should serve this shape"
        assert torch.equal(out, ref) and torch.equal(hf, hu) and torch.equal(df, du_)
        ref_f = S.m3_step_gated_((hua, ua, ub), delta, u, bc, cc, params, n_rot, z, d_skip)
        out_f = S.m3_step_gated_fused_((hfa, fa, fb), dt, x_dbl, R, R + N * p, wb, wc, 1e-5, p,
                                       u, params, n_rot, z, d_skip, dt_bias=db)
        assert torch.equal(out_f, ref_f) and torch.equal(hfa, hua) and torch.equal(fb, ub)
        fa, fb = fb, fa
        ua, ub = ub, ua
    assert S.device_error() == 0


def test_step_gated_fused_declines_unserved_shapes():
    """Shapes outside the fused kernel (a 16-lane state, a misaligned B_raw
    column, mimo_p 4) return None with nothing launched; the model then runs
    the two launches."""
    g = torch.Generator(device="cuda").manual_seed(1)
    B, D, N = 4, 64, 16
    params = tuple(t.contiguous() for t in S.pad_params(
        -torch.ones(D, 12, device="cuda"), torch.zeros(D, 12, device="cuda"),
        torch.zeros(D, 4, device="cuda"), 12, N, D, torch.device("cuda")))
    st = (torch.zeros(B, D, N, device="cuda"), torch.zeros(B, D, N, device="cuda"))
    dt = torch.randn(B, D, device="cuda", generator=g)
    x = torch.randn(B, 8 + 2 * N * 2, device="cuda", generator=g)
    u, z = torch.randn(B, D, device="cuda"), torch.randn(B, D, device="cuda")
    ds = torch.zeros(D, device="cuda")
    assert S.m3_step_gated_fused_(st, dt, x, 8, 8 + 2 * N, None, None, 0.0, 2, u, params, 12,
                                  z, ds) is None
    st32 = (torch.zeros(B, D, 32, device="cuda"), torch.zeros(B, D, 32, device="cuda"))
    p32 = tuple(t.contiguous() for t in S.pad_params(
        -torch.ones(D, 24, device="cuda"), torch.zeros(D, 24, device="cuda"),
        torch.zeros(D, 8, device="cuda"), 24, 32, D, torch.device("cuda")))
    x32 = torch.randn(B, 7 + 2 * 64, device="cuda", generator=g)
    assert S.m3_step_gated_fused_(st32, dt, x32, 7, 7 + 64, None, None, 0.0, 2, u, p32, 24,
                                  z, ds) is None
    x4 = torch.randn(B, 8 + 2 * 128, device="cuda", generator=g)
    assert S.m3_step_gated_fused_(st32, dt, x4, 8, 8 + 128, None, None, 0.0, 4, u, p32, 24,
                                  z, ds) is None
    assert S.device_error() == 0


def test_model_step_prologue_in_kernel_equals_two_launches():
    """Mamba.step_fused_ with the prologue inside the step kernel and with it as
    its own launch (Mamba3Block.fuse_step) give the same bits, state and output
    (projections on cuBLAS in both: the small-batch layer is switched off)."""
    from redpanda_b200.mamba import Mamba3Block
    old_small = Mamba3Block.small_step_max_batch
    Mamba3Block.small_step_max_batch = 0
    torch.manual_seed(7)
    cfg = MambaConfig(d_model=64, n_layer=2, d_state=32, n_track_state=8, mimo_p=2,
                      vocab_size=256)
    m = Mamba(cfg).cuda().eval()
    ids = torch.randint(0, 256, (7, 9), device="cuda")
    with torch.no_grad():
        _, cache = m.prime_cache(ids[:, :5])
        ca = [(h.clone(), d.clone()) for h, d in cache]
        cb = [(h.clone(), d.clone()) for h, d in cache]
        try:
            for t in range(5, 9):
                Mamba3Block.fuse_step = True
                ha, ca = m.step_fused_(token_id=ids[:, t], cache=ca)
                Mamba3Block.fuse_step = False
                hb, cb = m.step_fused_(token_id=ids[:, t], cache=cb)
                assert torch.equal(ha, hb)
        finally:
            Mamba3Block.fuse_step = True
            Mamba3Block.small_step_max_batch = old_small
        for (h1, d1), (h2, d2) in zip(ca, cb):
            assert torch.equal(h1, h2) and torch.equal(d1, d2)


def test_model_fused_step_matches_unfused_step_and_forward():
    """Config-3-like layers: the fused step layer reproduces Mamba.step_ (torch
    projections + m3_step_) and, from a primed cache, the full forward."""
    torch.manual_seed(2)
    cfg = MambaConfig(d_model=64, n_layer=2, d_state=32, n_track_state=8, mimo_p=2,
                      vocab_size=256)
    m = Mamba(cfg).cuda().eval()
    ids = torch.randint(0, 256, (5, 12), device="cuda")
    with torch.no_grad():
        full = m(ids)
        _, cache = m.prime_cache(ids[:, :8])
        cache_u = [(h.clone(), d.clone()) for h, d in cache]
        cache_f = [(h.clone(), d.clone()) for h, d in cache]
        for t in range(8, 12):
            hu, cache_u = m.step_(token_id=ids[:, t], cache=cache_u)
            hf, cache_f = m.step_fused_(token_id=ids[:, t], cache=cache_f)
            assert _rel(hf, hu) <= 1e-5
            assert torch.allclose(hf, full[:, t], atol=1e-5)
        for (h1, d1), (h2, d2) in zip(cache_u, cache_f):
            assert _rel(h2, h1) <= 1e-5 and _rel(d2, d1) <= 1e-5


def test_model_fused_step_factored_state_equals_full_state():
    torch.manual_seed(4)
    cfg = MambaConfig(d_model=64, n_layer=3, d_state=32, n_track_state=8, mimo_p=2,
                      vocab_size=256)
    m = Mamba(cfg).cuda().eval()
    B, D, N = 6, cfg.d_inner, cfg.d_state
    ids = torch.randint(0, 256, (B, 7), device="cuda")
    full = [(torch.zeros(B, D, N, device="cuda"), torch.zeros(B, D, N, device="cuda"))
            for _ in range(cfg.n_layer)]
    fac = [[torch.zeros(B, D, N, device="cuda"), torch.zeros(B, D + N, device="cuda"),
            torch.zeros(B, D + N, device="cuda")] for _ in range(cfg.n_layer)]
    with torch.no_grad():
        for t in range(7):
            a, _ = m.step_fused_(token_id=ids[:, t], cache=full)
            b, _ = m.step_fused_(token_id=ids[:, t], cache=fac)
            for st in fac:
                st[1], st[2] = st[2], st[1]
            assert torch.equal(a, b)
        for (h1, _), (h2, _, _) in zip(full, fac):
            assert torch.equal(h1, h2)


@pytest.mark.parametrize("coef", [1.0, 2.0])
@pytest.mark.parametrize("udtype", [torch.float32, torch.bfloat16])
def test_gate_matches_torch(coef, udtype):
    g = torch.Generator(device="cuda").manual_seed(9)
    B, L, D = 3, 17, 96
    y = torch.randn(B, L, D, device="cuda", generator=g)
    u = torch.randn(B, L, D, device="cuda", generator=g).to(udtype)
    xz = torch.randn(B, L, 2 * D, device="cuda", generator=g)
    d_skip = torch.randn(D, device="cuda", generator=g)
    out = S.m3_gate(y, u, xz[..., D:], d_skip, coef)
    ref = (y + coef * (u.float() * d_skip)) * F.silu(xz[..., D:])
    assert _rel(out, ref) <= TOL


@pytest.mark.parametrize("bidir", [False, True])
def test_inference_forward_equals_autograd_forward(bidir):
    """The no-grad layer forward (m3_step_inputs over B*L rows, scan, m3_gate)
    reproduces the training-path forward; prime_cache likewise."""
    torch.manual_seed(6)
    cfg = MambaConfig(d_model=64, n_layer=2, d_state=32, n_track_state=8, mimo_p=2,
                      vocab_size=256, bidirectional=bidir)
    m = Mamba(cfg).cuda().eval()
    ids = torch.randint(0, 256, (4, 21), device="cuda")
    with torch.enable_grad():
        ref = m(ids)
    with torch.no_grad():
        out = m(ids)
    assert _rel(out, ref) <= 1e-5
    if not bidir:
        with torch.enable_grad():
            fr, cr = m.prime_cache(ids)
        with torch.no_grad():
            fi, ci = m.prime_cache(ids)
        assert _rel(fi, fr) <= 1e-5
        for (h1, d1), (h2, d2) in zip(ci, cr):
            assert _rel(h1, h2) <= 1e-5 and _rel(d1, d2) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("coef", [1.0, 2.0])
def test_gated_output_fn_matches_torch_autograd(dtype, coef):
    """S.gated_output (m3_gate forward, m3_gate_bwd backward) against torch's
    autograd of (y + coef*u*D) * silu(z) with z a view of in_proj's output:
    the forward bit for bit; the gradients within fp32 rounding (fp32) or
    bf16 rounding (bf16: torch rounds some intermediates to bf16, the kernel
    rounds each gradient once)."""
    g = torch.Generator(device="cuda").manual_seed(21)
    B, L, D = 3, 37, 96
    xz0 = (torch.randn(B, L, 2 * D, device="cuda", generator=g) * 3).to(dtype)
    y0 = torch.randn(B, L, D, device="cuda", generator=g).to(dtype)
    u0 = torch.randn(B, L, D, device="cuda", generator=g).to(dtype)
    d0 = torch.randn(D, device="cuda", generator=g)
    go = torch.randn(B, L, D, device="cuda", generator=g)
    leaves = []
    for _ in range(2):
        leaves.append([t.clone().requires_grad_() for t in (xz0, y0, u0, d0)])
    (xa, ya, ua, da), (xb, yb, ub, db) = leaves
    ref = (ya + coef * ua * da) * F.silu(xa[..., D:])
    ref.backward(go)
    out = S.gated_output(yb, ub, xb[..., D:], db, coef)
    out.backward(go)
    assert out.dtype == ref.dtype and torch.equal(out, ref)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    for a, b in ((xa, xb), (ya, yb), (ua, ub), (da, db)):
        assert a.grad.dtype == b.grad.dtype
        assert _rel(b.grad.float(), a.grad.float()) <= tol, (a.shape, _rel(b.grad, a.grad))
    assert xb.grad[..., :D].abs().max().item() == 0.0
    # deterministic: the d_skip reduction has a fixed order
    first = db.grad.clone()
    for t in leaves[1]:
        t.grad = None
    S.gated_output(yb, ub, xb[..., D:], db, coef).backward(go)
    assert torch.equal(db.grad, first)


@pytest.mark.parametrize("bcnorm", [True, False])
def test_step_inputs_backward_matches_torch_autograd(bcnorm):
    """m3_step_inputs_bwd: the gradients torch's softplus / RMSNorm / sum give."""
    g = torch.Generator(device="cuda").manual_seed(21)
    rows, D, R, n, p = 300, 96, 8, 32, 4
    dt = (torch.randn(rows, D, device="cuda", generator=g) * 8).requires_grad_(True)
    x_dbl = torch.randn(rows, R + 2 * n * p, device="cuda", generator=g).requires_grad_(True)
    wb = (torch.rand(n * p, device="cuda", generator=g) + 0.5).requires_grad_(bcnorm)
    wc = (torch.rand(n * p, device="cuda", generator=g) + 0.5).requires_grad_(bcnorm)
    gd = torch.randn(rows, D, device="cuda", generator=g)
    gb = torch.randn(rows, n, device="cuda", generator=g)
    gc = torch.randn(rows, n, device="cuda", generator=g)
    eps = 1e-5

    def torch_path():
        delta = F.softplus(dt)
        braw, craw = x_dbl[:, R:R + n * p], x_dbl[:, R + n * p:]
        if bcnorm:
            braw = braw * torch.rsqrt(braw.pow(2).mean(-1, keepdim=True) + eps) * wb
            craw = craw * torch.rsqrt(craw.pow(2).mean(-1, keepdim=True) + eps) * wc
        return delta, braw.reshape(rows, n, p).sum(-1), craw.reshape(rows, n, p).sum(-1)

    outs = []
    for fn in (torch_path, lambda: S.step_inputs(dt, x_dbl, R, R + n * p, wb if bcnorm else None,
                                                 wc if bcnorm else None, eps, n, p)):
        for t in (dt, x_dbl, wb, wc):
            t.grad = None
        d, b, c = fn()
        ((d * gd).sum() + (b * gb).sum() + (c * gc).sum()).backward()
        outs.append([t.grad.clone() if t.grad is not None else None for t in (dt, x_dbl, wb, wc)])
    for a, r in zip(outs[1], outs[0]):
        if r is None:
            assert a is None
        else:
            assert _rel(a, r) <= 2e-6
    # bitwise reproducible
    for t in (dt, x_dbl, wb, wc):
        t.grad = None
    d, b, c = S.step_inputs(dt, x_dbl, R, R + n * p, wb if bcnorm else None,
                            wc if bcnorm else None, eps, n, p)
    ((d * gd).sum() + (b * gb).sum() + (c * gc).sum()).backward()
    for t, prev in zip((dt, x_dbl, wb, wc), outs[1]):
        if prev is not None:
            assert torch.equal(t.grad, prev)
