"""The small-batch step layer: m3_rows_linear / m3_xdt_proj against float64
products, and Mamba.step_fused_ on those kernels against the same step on
cuBLAS GEMMs (the reference's projections, TF32 off).

The kernels change only the summation order of the projections, so the
bars are a few float32 roundings of the products' magnitude."""

import pytest
import torch

from redpanda_b200 import scan as S
from redpanda_b200.graphs import StepGraph
from redpanda_b200.mamba import Mamba, Mamba3Block, MambaConfig

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("rows", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("norm,bias,resid,split", [(True, False, False, 0.5),
                                                   (False, True, True, 1.0),
                                                   (True, True, False, 1.0)])
def test_rows_linear_matches_float64(rows, norm, bias, resid, split):
    g = torch.Generator("cuda").manual_seed(rows)
    d_in, d_out = 512, 768
    x = torch.randn(rows, d_in, device="cuda", generator=g)
    W = torch.randn(d_out, d_in, device="cuda", generator=g) / d_in ** 0.5
    nw = torch.rand(d_in, device="cuda", generator=g) + 0.5 if norm else None
    b = torch.randn(d_out, device="cuda", generator=g) if bias else None
    r = torch.randn(rows, d_out, device="cuda", generator=g) if resid else None
    sp = int(d_out * split)
    xd = x.double()
    if norm:
        xd = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-5) * nw.double()
    ref = xd @ W.double().t()
    if bias:
        ref = ref + b.double()
    if resid:
        ref = ref + r.double()
    ref = torch.cat([torch.nn.functional.silu(ref[:, :sp]), ref[:, sp:]], 1) if sp < d_out \
        else ref
    out0, out1 = S.m3_rows_linear(x, W, b, nw, 1e-5, residual=r, split=sp, silu=sp < d_out)
    got = out0 if out1 is None else torch.cat([out0, out1], 1)
    assert _rel(got, ref) <= 2e-6
    again = S.m3_rows_linear(x, W, b, nw, 1e-5, residual=r, split=sp, silu=sp < d_out)
    assert torch.equal(out0, again[0])                    # deterministic


@pytest.mark.parametrize("rows", [1, 5])
def test_rows_linear_unaligned_rows_match_aligned(rows):
    """Input rows that are not 16-byte aligned take the element-wise staging;
    same bits as the vector staging of the same values."""
    g = torch.Generator("cuda").manual_seed(11)
    buf = torch.randn(rows, 513, device="cuda", generator=g)
    x_un = buf[:, 1:]                                  # 4-byte offset, row stride 513
    x_al = x_un.contiguous()
    W = torch.randn(256, 512, device="cuda", generator=g) / 512 ** 0.5
    nw = torch.rand(512, device="cuda", generator=g) + 0.5
    a = S.m3_rows_linear(x_un, W, None, nw, 1e-5, split=128, silu=True)
    b = S.m3_rows_linear(x_al, W, None, nw, 1e-5, split=128, silu=True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_rows_linear_residual_in_place():
    g = torch.Generator("cuda").manual_seed(9)
    x = torch.randn(3, 256, device="cuda", generator=g)
    W = torch.randn(128, 256, device="cuda", generator=g) / 16
    res = torch.randn(3, 128, device="cuda", generator=g)
    want = S.m3_rows_linear(x, W, residual=res)[0]
    out = S.m3_rows_linear(x, W, residual=res, out0=res)[0]
    assert out.data_ptr() == res.data_ptr() and torch.equal(res, want)


@pytest.mark.parametrize("rows", [1, 4, 8])
def test_xdt_proj_matches_float64(rows):
    g = torch.Generator("cuda").manual_seed(rows)
    d, r, n_x = 1024, 32, 160
    u = torch.randn(rows, d, device="cuda", generator=g)
    wx = torch.randn(n_x, d, device="cuda", generator=g) / d ** 0.5
    bx = torch.randn(n_x, device="cuda", generator=g)
    wdt = torch.randn(d, r, device="cuda", generator=g) / r ** 0.5
    x_dbl, dt = S.m3_xdt_proj(u, wx, bx, wdt)
    ref_x = u.double() @ wx.double().t() + bx.double()
    assert _rel(x_dbl, ref_x) <= 2e-6
    # dt from the kernel's own dt_raw columns (the step's contract), in float64
    assert _rel(dt, x_dbl[:, :r].double() @ wdt.double().t()) <= 2e-6
    assert _rel(dt, ref_x[:, :r] @ wdt.double().t()) <= 5e-6


def test_small_batch_limits_decline():
    u = torch.randn(9, 64, device="cuda")
    assert S.m3_rows_linear(u, torch.randn(32, 64, device="cuda")) is None      # 9 rows
    x = torch.randn(8, 2048, device="cuda")
    assert S.m3_rows_linear(x, torch.randn(16, 2048, device="cuda")) is None    # 64 KB staged


def _model(d_state, n_track, mimo_p, seed=0):
    torch.manual_seed(seed)
    cfg = MambaConfig(d_model=128, n_layer=3, d_state=d_state, n_track_state=n_track,
                      mimo_p=mimo_p, vocab_size=256)
    m = Mamba(cfg).cuda().eval()
    with torch.no_grad():   # rotation phases off zero, as a trained model has
        for layer in m.layers:
            layer["mixer"].A_phase.uniform_(-1.4, 1.4)
    return m


def _rollout(m, ids, small):
    old = Mamba3Block.small_step_max_batch
    Mamba3Block.small_step_max_batch = 8 if small else 0
    try:
        with torch.no_grad():
            B = ids.shape[0]
            cfg = m.config
            cache = [(torch.zeros(B, cfg.d_inner, cfg.d_state, device="cuda"),
                      torch.zeros(B, cfg.d_inner, cfg.d_state, device="cuda"))
                     for _ in m.layers]
            hs = []
            for t in range(ids.shape[1]):
                h, cache = m.step_fused_(token_id=ids[:, t], cache=cache)
                hs.append(h.clone())
        return torch.stack(hs, 1), cache
    finally:
        Mamba3Block.small_step_max_batch = old


@pytest.mark.parametrize("B", [1, 3, 8])
@pytest.mark.parametrize("shape", [(32, 8, 2),     # the fused step kernel (32 lanes)
                                   (16, 4, 2)])    # the two-launch step (16 lanes)
def test_small_step_matches_gemm_step(B, shape):
    m = _model(*shape)
    ids = torch.randint(0, 256, (B, 12), device="cuda", generator=torch.Generator("cuda").manual_seed(B))
    hs_small, c_small = _rollout(m, ids, True)
    hs_ref, c_ref = _rollout(m, ids, False)
    assert _rel(hs_small, hs_ref) <= 1e-5
    for (h1, d1), (h2, d2) in zip(c_small, c_ref):
        assert _rel(h1, h2) <= 1e-5 and _rel(d1, d2) <= 1e-5
    again, _ = _rollout(m, ids, True)
    assert torch.equal(again, hs_small)


def test_small_step_leaves_input_embed_alone():
    m = _model(32, 8, 2)
    emb = torch.randn(2, 128, device="cuda")
    keep = emb.clone()
    cfg = m.config
    cache = [(torch.zeros(2, cfg.d_inner, cfg.d_state, device="cuda"),
              torch.zeros(2, cfg.d_inner, cfg.d_state, device="cuda")) for _ in m.layers]
    with torch.no_grad():
        m.step_fused_(input_embed=emb, cache=cache)
    assert torch.equal(emb, keep)


def test_small_step_graph_equals_eager():
    m = _model(32, 8, 2, seed=4)
    ids = torch.randint(0, 256, (1, 6), device="cuda")
    hs_eager, c_eager = _rollout(m, ids, True)
    g = StepGraph(m, 1)
    hs = []
    for t in range(ids.shape[1]):
        hs.append(g.step(ids[:, t])[0].clone())
    assert torch.equal(torch.stack(hs, 1), hs_eager)
    for (h1, d1), (h2, d2) in zip(g.cache, c_eager):
        assert torch.equal(h1, h2) and torch.equal(d1, d2)


@pytest.mark.parametrize("B", [1, 2, 5])
def test_step_fused_proj_matches_fused_with_dt(B):
    """dt_proj's product inside the step kernel equals the fused step given
    dt = x_dbl[:, :r] @ W_dt.T (float64, rounded once) to a few float32 ulps;
    state and output."""
    g = torch.Generator("cuda").manual_seed(B)
    D, N, nr, p, r = 256, 32, 24, 2, 32
    ld = r + 2 * N * p
    x_dbl = torch.randn(B, ld, device="cuda", generator=g)
    w_dt = torch.randn(D, r, device="cuda", generator=g) * 0.1
    bias = torch.randn(D, device="cuda", generator=g) * 0.5 - 2
    u = torch.randn(B, D, device="cuda", generator=g)
    z = torch.randn(B, D, device="cuda", generator=g)
    d_skip = torch.randn(D, device="cuda", generator=g)
    bw = torch.rand(N * p, device="cuda", generator=g) + 0.5
    cw = torch.rand(N * p, device="cuda", generator=g) + 0.5
    A_real = -torch.exp(torch.randn(D, nr, device="cuda", generator=g) * 0.5)
    A_imag = (torch.rand(D, nr, device="cuda", generator=g) * 2 - 1) * 3.0
    track = torch.tanh(torch.randn(D, N - nr, device="cuda", generator=g))
    params = tuple(t.contiguous() for t in S.pad_params(A_real, A_imag, track, nr, N, D,
                                                        torch.device("cuda")))
    h0 = torch.randn(B, D, N, device="cuda", generator=g)
    d0 = torch.randn(B, D, N, device="cuda", generator=g)
    sa = (h0.clone(), d0.clone())
    sb = (h0.clone(), d0.clone())
    dt = (x_dbl[:, :r].double() @ w_dt.double().t()).float()
    ya = S.m3_step_gated_fused_proj_(sa, w_dt, x_dbl, r, r + N * p, bw, cw, 1e-5, p, u, params,
                                     nr, z, d_skip, dt_bias=bias)
    yb = S.m3_step_gated_fused_(sb, dt, x_dbl, r, r + N * p, bw, cw, 1e-5, p, u, params, nr, z,
                                d_skip, dt_bias=bias)
    assert ya is not None and yb is not None
    assert _rel(ya, yb) <= 1e-5
    assert _rel(sa[0], sb[0]) <= 1e-5 and _rel(sa[1], sb[1]) <= 1e-5
