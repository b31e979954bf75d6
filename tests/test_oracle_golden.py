"""Pin the CPU oracle to golden vectors produced by the reference itself.

The fixtures under tests/golden were written by tests/golden/make_golden.py,
which imports the reference ``redpanda/engine/mamba.py`` and runs its scan
(``_selective_scan_trapezoidal``), its autograd gradients, and the reference
``Mamba`` model's forward / ``step`` / ``prime_cache``.  These tests need no GPU.
"""

import glob
import os

import pytest
import torch

import oracle as O
from oracle import model_oracle as MO

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# The oracle repeats the reference's torch CPU ops in the same order; the
# tolerance only absorbs CPU SIMD-path differences between machines.
TOL = 2e-6


def _rel(a, b):
    den = b.abs().max().item()
    return (a - b).abs().max().item() / (den if den > 0 else 1.0)


SCAN_CASES = sorted(os.path.basename(p)[:-3] for p in glob.glob(os.path.join(GOLDEN, "scan_*.pt")))
MODEL_CASES = sorted(os.path.basename(p)[:-3] for p in glob.glob(os.path.join(GOLDEN, "model_*.pt")))


def test_fixtures_present():
    assert len(SCAN_CASES) >= 6 and len(MODEL_CASES) >= 3


@pytest.mark.parametrize("name", SCAN_CASES)
def test_scan_oracle_matches_reference(name):
    c = torch.load(os.path.join(GOLDEN, name + ".pt"))
    i = c["inputs"]
    y, g = O.scan_with_grads(i["delta"], i["u"], i["Bc"], i["Cc"], i["A_real"], i["A_imag"],
                             i["track"], i["dy"], bidir=c["bidir"])
    assert _rel(y, c["y"]) <= TOL
    for k in ("delta", "u", "Bc", "Cc", "A_real", "A_imag"):
        if k in c["grads"]:
            assert _rel(g[k], c["grads"][k]) <= TOL, k
    if "theta" in c["grads"]:
        # the reference differentiates w.r.t. theta; chain rule through tanh
        dth = g["track"] * (1 - i["track"] ** 2)
        assert _rel(dth, c["grads"]["theta"]) <= 5e-6
    if "h_last" in c:
        _, (h, dbu) = O.scan_chunked(i["delta"], i["u"], i["Bc"], i["Cc"], i["A_real"],
                                     i["A_imag"], i["track"], return_state=True)
        assert _rel(h, c["h_last"]) <= TOL
        assert _rel(dbu, c["dbu_last"]) <= TOL


@pytest.mark.parametrize("name", SCAN_CASES)
def test_sequential_fp64_agrees_with_reference(name):
    """The fp64 time loop (math spec) and the reference fp32 scan agree to fp32 noise."""
    c = torch.load(os.path.join(GOLDEN, name + ".pt"))
    if c["bidir"]:
        pytest.skip("sequential spec is per direction")
    i = {k: (None if v is None else v.double()) for k, v in c["inputs"].items()}
    y, _, _ = O.scan_sequential(i["delta"], i["u"], i["Bc"], i["Cc"], i["A_real"], i["A_imag"],
                                i["track"])
    assert _rel(c["y"].double(), y) <= 1e-6


@pytest.mark.parametrize("name", MODEL_CASES)
def test_model_oracle_matches_reference(name):
    c = torch.load(os.path.join(GOLDEN, name + ".pt"))
    cfg = MO.OracleConfig(vocab_size=64, bidirectional=c["bidir"], **c["kw"])
    p = {k: v.clone().requires_grad_(v.is_floating_point()) for k, v in c["state_dict"].items()}
    y = MO.model_forward(p, cfg, c["ids"])
    y.pow(2).mean().backward()
    assert _rel(y.detach(), c["forward"]) <= TOL
    for k, g in c["param_grads"].items():
        assert _rel(p[k].grad, g) <= 1e-5, k
    if c["bidir"]:
        return
    pp = {k: v.detach() for k, v in p.items()}
    with torch.no_grad():
        cache, hs = None, []
        for t in range(c["ids"].shape[1]):
            h, cache = MO.model_step(pp, cfg, c["ids"][:, t], cache)
            hs.append(h)
        assert _rel(torch.stack(hs, 1), c["step_hidden"]) <= TOL
        for (h1, d1), (h2, d2) in zip(cache, c["step_cache_last"]):
            assert _rel(h1, h2) <= TOL and _rel(d1, d2) <= TOL
        fin, pc = MO.model_prime_cache(pp, cfg, c["ids"][:, :c["prime_k"]])
        assert _rel(fin, c["prime_final"]) <= TOL
        nxt, _ = MO.model_step(pp, cfg, c["ids"][:, c["prime_k"]], pc)
        assert _rel(nxt, c["prime_next"]) <= TOL


def test_oracle_step_matches_scan_within_reference_tolerance():
    """The reference's own claim (test_v3.py:55, test_v4.py:257): step == forward, atol 1e-4."""
    from redpanda_b200.synthetic import ScanShape, make_scan_inputs
    sh = ScanShape(2, 12, 32, 12, 4, 2)
    i = make_scan_inputs(sh, seed=5)
    y = O.scan_chunked(i["delta"], i["u"], i["Bc"], i["Cc"], i["A_real"], i["A_imag"], i["track"])
    h = torch.zeros(2, 32, 12)
    dbu = torch.zeros_like(h)
    for t in range(sh.seqlen):
        yt, h, dbu = O.step_cells(h, dbu, i["delta"][:, t], i["u"][:, t], i["Bc"][:, t],
                                  i["Cc"][:, t], i["A_real"], i["A_imag"], i["track"])
        assert torch.allclose(yt, y[:, t], atol=1e-4)


def test_verify_gate_recurrence_matches_oracle():
    """The float64 recurrence the verify gate compares the kernels with is the
    oracle's scan (CPU, float64)."""
    from redpanda_b200 import verify as V
    from redpanda_b200.synthetic import ScanShape, make_scan_inputs
    for sh in (ScanShape(2, 9, 16, 8, 2, 2), ScanShape(1, 33, 24, 12, 0, 2),
               ScanShape(2, 5, 8, 4, 4, 2)):
        inp = make_scan_inputs(sh, seed=1)
        d = {k: (None if v is None else v.double()) for k, v in inp.items()}
        y = V._torch_scan(d["delta"], d["u"], d["Bc"], d["Cc"], d["A_real"], d["A_imag"],
                          d["track"])
        yr, _ = O.scan_with_grads(d["delta"], d["u"], d["Bc"], d["Cc"], d["A_real"],
                                  d["A_imag"], d["track"], d["dy"])
        assert (y - yr).abs().max().item() <= 1e-12 * max(1.0, yr.abs().max().item())
