"""The drop-in boundary: the reference's own call into its fused-scan module,
made against ``redpanda_b200.scan``.

The reference reaches the fused scan from ``Mamba3Block._selective_scan_trapezoidal``
(redpanda/engine/mamba.py:343-350) with

    from triton_scan import HAS_TRITON, triton_trapezoidal_scan
    y = triton_trapezoidal_scan(u=u, delta=delta, B_contracted=..., ...)

tests/golden/make_golden.py reads that call site out of the reference source
into tests/golden/dropin_callsite.json (module, imported names, keyword names),
so these tests check the drop-in module against the reference's real call
without the reference checkout:

* (CPU) every name the reference imports exists, and the reference's keyword
  call binds to the drop-in signature;
* (GPU) the call made with exactly the reference's keyword names reproduces
  the reference's own scan outputs and gradients (the golden scan fixtures);
* (GPU, only where a reference checkout is importable: REDPANDA_REFERENCE
  names it) the UNMODIFIED reference ``Mamba`` with ``use_triton_scan=True``
  and ``sys.modules["triton_scan"] = redpanda_b200.scan`` reproduces the
  reference model's forward output and parameter gradients.
"""

import importlib.util
import inspect
import json
import os
import sys

import pytest
import torch

from helpers import PARITY_TABLE, rel_err

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FWD_TOL = 1e-5
GRAD_TOL = 1e-6
MODEL_GRAD_TOL = 1e-4


def _callsite():
    with open(os.path.join(GOLDEN, "dropin_callsite.json")) as f:
        return json.load(f)


def test_dropin_module_exports_what_the_reference_imports():
    from redpanda_b200 import scan as S
    cs = _callsite()
    assert cs["module"] == "triton_scan"
    for name in cs["imports"]:
        assert hasattr(S, name), name
    sig = inspect.signature(S.triton_trapezoidal_scan)
    for call in cs["calls"]:
        args = [object()] * call["n_positional"]
        sig.bind(*args, **{k: object() for k in call["keywords"]})   # raises on a mismatch


def _reference_kwargs(names, tensors):
    """Arguments named as at the reference call site (mamba.py:346-349)."""
    return {k: tensors[k] for k in names}


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["scan_c0_causal", "scan_c3_slice", "scan_l70_notrack", "scan_l1"])
def test_reference_call_reproduces_reference_scan(name):
    from redpanda_b200 import scan as S
    cs = _callsite()
    c = torch.load(os.path.join(GOLDEN, name + ".pt"))
    i = c["inputs"]
    shape = c["shape"]
    n_state, n_track = shape[3], shape[4]
    leaves = {k: i[k].cuda().clone().requires_grad_(True)
              for k in ("delta", "u", "Bc", "Cc", "A_real", "A_imag") if i[k] is not None}
    track = None if i["track"] is None else i["track"].cuda().clone().requires_grad_(True)
    t = {"u": leaves["u"], "delta": leaves["delta"], "B_contracted": leaves["Bc"],
         "C_contracted": leaves["Cc"], "A_real": leaves.get("A_real"),
         "A_imag": leaves.get("A_imag"), "track": track, "n_rot": n_state - n_track,
         "n_state": n_state}
    assert S.HAS_TRITON
    y = S.triton_trapezoidal_scan(**_reference_kwargs(cs["calls"][0]["keywords"], t))
    (y * i["dy"].cuda()).sum().backward()
    ey = rel_err(y, c["y"])
    PARITY_TABLE.append(("dropin_" + name, "y", "fp32", ey, float("nan"), float("nan"),
                         "ok" if ey <= FWD_TOL else "FAIL"))
    assert ey <= FWD_TOL
    for k, g in c["grads"].items():
        if k == "theta":
            got = track.grad * (1 - i["track"].cuda() ** 2)
        else:
            got = leaves[k].grad
        e = rel_err(got, g)
        # the theta gradient adds the chain rule through tanh, evaluated here
        # and in the reference in different fp32 orders
        bar = 5e-6 if k == "theta" else GRAD_TOL
        PARITY_TABLE.append(("dropin_" + name, "d" + k, "fp32", e, float("nan"), float("nan"),
                             "ok" if e <= bar else "FAIL"))
        assert e <= bar, k


def _import_reference_mamba():
    ref = os.environ.get("REDPANDA_REFERENCE")
    if not ref:
        pytest.skip("no reference checkout (set REDPANDA_REFERENCE); it does not travel to "
                    "the GPU box, where the recorded call site above stands in for it")
    path = os.path.join(ref, "redpanda", "engine", "mamba.py")
    if not os.path.exists(path):
        pytest.skip("REDPANDA_REFERENCE does not hold redpanda/engine/mamba.py")
    spec = importlib.util.spec_from_file_location("redpanda_reference_mamba", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["model_verify_trk", "model_phase_bidir"])
def test_unmodified_reference_model_through_dropin(name, monkeypatch):
    from redpanda_b200 import scan as S
    M = _import_reference_mamba()
    monkeypatch.setitem(sys.modules, "triton_scan", S)
    c = torch.load(os.path.join(GOLDEN, name + ".pt"))
    cfg = M.MambaConfig(vocab_size=64, bidirectional=c["bidir"], use_triton_scan=True,
                        **c["kw"])
    m = M.Mamba(cfg).cuda()
    m.load_state_dict(c["state_dict"])
    m.train()
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        y = m(c["ids"].cuda())
        y.pow(2).mean().backward()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    assert rel_err(y, c["forward"]) <= FWD_TOL
    grads = dict(m.named_parameters())
    for k, g in c["param_grads"].items():
        assert rel_err(grads[k].grad, g) <= MODEL_GRAD_TOL, k
