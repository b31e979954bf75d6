"""The whole-stack step captured as one CUDA graph (redpanda_b200.graphs).

Replaying the graph runs the same kernels as the eager fused step on the same
addresses, so its outputs and state must equal the eager ones; priming into a
given cache must equal priming into new tensors; the graphed node evaluation
must keep eval_step's contract (search_mamba.py:275-291).
"""

import pytest
import torch

from redpanda_b200.graphs import StepGraph
from redpanda_b200.mamba import Mamba, MambaConfig
from redpanda_b200.search_mamba import SearchMamba, SearchMambaConfig

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _model(seed=5):
    torch.manual_seed(seed)
    cfg = MambaConfig(d_model=64, n_layer=3, d_state=32, n_track_state=8, mimo_p=2,
                      vocab_size=256)
    m = Mamba(cfg).cuda().eval()
    with torch.no_grad():   # learned-looking rotation phases (A_imag != 0)
        for layer in m.layers:
            layer["mixer"].A_phase.uniform_(-1.2, 1.2)
    return m


def test_prime_into_given_cache_equals_prime():
    m = _model()
    ids = torch.randint(0, 256, (4, 24), device="cuda")
    with torch.no_grad():
        h_ref, cache_ref = m.prime_cache(ids)
        out = [(torch.full_like(h, 7.0), torch.full_like(d, -3.0)) for h, d in cache_ref]
        h_out, cache_out = m.prime_cache(ids, out=out)
    assert torch.equal(h_ref, h_out)
    for (a, b), (c, d), (e, f) in zip(cache_ref, cache_out, out):
        assert c is e and d is f
        assert torch.equal(a, c) and torch.equal(b, d)


def test_step_graph_equals_eager_fused_step():
    m = _model()
    B = 6
    ids = torch.randint(0, 256, (B, 16), device="cuda")
    moves = torch.randint(0, 256, (5, B), device="cuda")
    with torch.no_grad():
        _, cache = m.prime_cache(ids)
        g = StepGraph(m, B)
        m.prime_cache(ids, out=g.cache)
        eager = [(h.clone(), d.clone()) for h, d in cache]
        for t in range(5):
            he, eager = m.step_fused_(token_id=moves[t], cache=eager)
            hg = g.step(moves[t])[0]
            assert torch.equal(he, hg), t
        for (h1, d1), (h2, d2) in zip(eager, g.cache):
            assert torch.equal(h1, h2) and torch.equal(d1, d2)


def test_step_graph_load_snapshot_reset():
    m = _model()
    B = 3
    ids = torch.randint(0, 256, (B, 10), device="cuda")
    with torch.no_grad():
        _, cache = m.prime_cache(ids)
        g = StepGraph(m, B)
        g.load_(cache)                       # per-tensor copy
        for (a, b), (c, d) in zip(cache, g.cache):
            assert torch.equal(a, c) and torch.equal(b, d)
        snap = g.snapshot()
        h1 = g.step(torch.tensor([1, 2, 3]))[0].clone()
        g.load_(snap)                        # one flat copy back to the snapshot
        h2 = g.step(torch.tensor([1, 2, 3]))[0]
        assert torch.equal(h1, h2)
        g.reset_()
        assert float(g.flat.abs().max()) == 0.0
        # the zero state is the reference's empty cache: the graph equals the
        # eager step from no cache
        h0, _ = m.step_fused_(token_id=torch.tensor([9, 9, 9], device="cuda"),
                              cache=[(torch.zeros_like(a), torch.zeros_like(b))
                                     for a, b in cache])
        assert torch.equal(g.step(torch.tensor([9, 9, 9]))[0], h0)
        # the token forms: one Python int for every row (a fill kernel), a CUDA
        # tensor, a host list (through the pinned buffer) give the same step
        outs = []
        for tok in (9, torch.full((3,), 9, device="cuda"), [9, 9, 9]):
            g.reset_()
            outs.append(g.step(tok)[0].clone())
        assert all(torch.equal(o, h0) for o in outs)


@pytest.mark.parametrize("shape", [dict(d_model=48, d_state=16, n_track_state=4),
                                   dict(d_model=64, d_state=32, n_track_state=8)])
def test_search_eval_step_graphed_matches_eval_step(shape):
    """Two state layouts: 16 lanes (the step kernel's element-wise path) and 32
    (the pipelined kernel with the prologue fused in, batch 1)."""
    torch.manual_seed(3)
    scfg = SearchMambaConfig(n_layer=3, mimo_p=2, vocab_size=300, **shape)
    sm = SearchMamba(scfg, vocab_size=300).cuda().eval()
    board = torch.randint(1, 300, (30,), device="cuda")
    moves = [5, 17, 250, 3]
    with torch.no_grad():
        _, cache = sm.prime_board(board)
        keep = [(h.clone(), d.clone()) for h, d in cache]
        ce, cg = cache, cache
        for mv in moves:
            ve, le, ce = sm.eval_step(ce, mv)
            vg, lg, cg = sm.eval_step_graphed(cg, mv)
            # the graph runs the fused step layer (one kernel for the recurrence
            # and its gated output); eager eval_step runs the step kernel and
            # the gate in torch: equal up to rounding
            assert abs(ve - vg) < 1e-5
            assert (le - lg).abs().max().item() <= 1e-5 * max(1.0, le.abs().max().item())
            for (h1, d1), (h2, d2) in zip(ce, cg):
                assert (h1 - h2).abs().max().item() <= 1e-5 * max(1.0, h1.abs().max().item())
    # the caller's cache is untouched
    for (a, b), (c, d) in zip(keep, cache):
        assert torch.equal(a, c) and torch.equal(b, d)


def test_search_evaluate_lines_fast_graphed_matches_eager():
    torch.manual_seed(4)
    scfg = SearchMambaConfig(d_model=48, n_layer=3, d_state=32, n_track_state=8, mimo_p=2,
                             vocab_size=300)
    sm = SearchMamba(scfg, vocab_size=300).cuda().eval()
    board = torch.randint(1, 300, (24,), device="cuda")
    lines = torch.randint(1, 300, (5, 6), device="cuda")
    lengths = torch.tensor([6, 1, 3, 6, 2], device="cuda")
    with torch.no_grad():
        eager = sm.evaluate_lines_fast(board, lines, lengths)
        graphed = sm.evaluate_lines_fast(board, lines, lengths, graphed=True)
        again = sm.evaluate_lines_fast(board, lines, lengths, graphed=True)   # reused graph
        slow = sm.evaluate_lines(board, lines)
    assert torch.allclose(eager, graphed, atol=1e-5)
    assert torch.equal(graphed, again)
    full = lengths == lines.shape[1]
    assert torch.allclose(slow[full], graphed[full], atol=1e-4)
    sm.release_graphs()
