"""Generate the golden fixtures that pin the CPU oracle to the reference itself.

Run in a container where the read-only reference checkout is present:

    python tests/golden/make_golden.py [--ref /path/to/RedPanda]

It imports ``redpanda/engine/mamba.py`` from that checkout, drives the
reference's own ``Mamba3Block._selective_scan_trapezoidal`` (the PyTorch scan
path, training mode with its default ``scan_checkpoint=True``) and the
reference ``Mamba`` model (forward, ``step``, ``prime_cache``, parameter
gradients), and stores inputs and outputs as small ``.pt`` files next to this
script.  Nothing on the GPU box reads the reference; the fixtures travel
instead.
"""

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from redpanda_b200.synthetic import ScanShape, make_scan_inputs  # noqa: E402


def _ref_block(M, shape, theta):
    cfg = M.MambaConfig(d_model=shape.d_inner // 2, n_layer=1, vocab_size=64,
                        d_state=shape.d_state, n_track_state=shape.n_track,
                        mimo_p=1, scan_checkpoint=True, use_triton_scan=False)
    blk = M.Mamba3Block(cfg).train()
    if shape.n_track > 0:
        with torch.no_grad():
            blk.track_theta.copy_(theta)
    return blk


def scan_case(M, shape, seed, bidir):
    """Reference scan (no skip term) + autograd grads for one seeded input set."""
    inp = make_scan_inputs(shape, seed=seed)
    blk = _ref_block(M, shape, inp["theta"])
    leaves = {k: inp[k].clone().requires_grad_(True)
              for k in ("delta", "u", "Bc", "Cc", "A_real", "A_imag") if inp[k] is not None}
    D0 = torch.zeros(shape.d_inner)

    def run(delta, u, Bc, Cc, Ar, Ai, return_state=False):
        # p = 1 view so that the block's B.sum(-1) is the identity.
        return blk._selective_scan_trapezoidal(u, delta, Ar, Ai, Bc.unsqueeze(-1),
                                               Cc.unsqueeze(-1), D0,
                                               return_state=return_state)

    lv = leaves
    y = run(lv["delta"], lv["u"], lv["Bc"], lv["Cc"], lv.get("A_real"), lv.get("A_imag"))
    if bidir:
        y = y + run(lv["delta"].flip(1), lv["u"].flip(1), lv["Bc"].flip(1),
                    lv["Cc"].flip(1), lv.get("A_real"), lv.get("A_imag")).flip(1)
    (y * inp["dy"]).sum().backward()
    out = {"shape": tuple(shape.__dict__.values()), "seed": seed, "bidir": bidir,
           "inputs": {k: (v if v is None else v.clone()) for k, v in inp.items()},
           "y": y.detach().clone(),
           "grads": {k: v.grad.clone() for k, v in leaves.items()}}
    if shape.n_track > 0:
        out["grads"]["theta"] = blk.track_theta.grad.clone()
    if not bidir:
        with torch.no_grad():
            blk.eval()
            _, (h, dbu) = run(inp["delta"], inp["u"], inp["Bc"], inp["Cc"],
                              inp["A_real"], inp["A_imag"], return_state=True)
        out["h_last"], out["dbu_last"] = h.clone(), dbu.clone()
    return out


def _set_phases(layers, seed, bound=1.4):
    """Draw every layer's A_phase from U(-bound, bound).  The reference
    initialises it to zero (mamba.py:188), which leaves A_imag = 0 and the
    rotation unused.  |phase| < pi/2 keeps A_real = -exp(A_log_mag)*cos(phase)
    negative (decaying gates); a phase past pi/2 makes A_real positive, the
    gates exceed 1 and the reference's own outputs overflow within a few dozen
    tokens."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for layer in layers:
            mixer = layer["mixer"]
            if hasattr(mixer, "A_phase"):
                mixer.A_phase.copy_((torch.rand(mixer.A_phase.shape, generator=g) * 2 - 1) * bound)


def model_case(M, kw, seed, L, bidir, phases=False):
    """Reference Mamba: forward, step chain, prime_cache and parameter grads."""
    torch.manual_seed(seed)
    cfg = M.MambaConfig(vocab_size=64, bidirectional=bidir, scan_checkpoint=True,
                        use_triton_scan=False, **kw)
    m = M.Mamba(cfg)
    if phases:
        _set_phases(m.layers, seed + 100)
    ids = torch.randint(0, 64, (3, L))
    out = {"kw": dict(kw), "bidir": bidir, "seed": seed, "ids": ids,
           "state_dict": {k: v.clone() for k, v in m.state_dict().items()}}
    m.train()
    y = m(ids)
    y.pow(2).mean().backward()
    out["forward"] = y.detach().clone()
    out["param_grads"] = {k: p.grad.clone() for k, p in m.named_parameters()
                          if p.grad is not None}
    m.zero_grad(set_to_none=True)
    if not bidir:
        m.eval()
        with torch.no_grad():
            cache = None
            hs = []
            for t in range(L):
                h, cache = m.step(token_id=ids[:, t], cache=cache)
                hs.append(h)
            out["step_hidden"] = torch.stack(hs, 1)
            out["step_cache_last"] = [(a.clone(), b.clone()) for a, b in cache]
            k = max(1, L // 2)
            fin, pc = m.prime_cache(ids[:, :k])
            out["prime_k"] = k
            out["prime_final"] = fin.clone()
            out["prime_cache"] = [(a.clone(), b.clone()) for a, b in pc]
            nxt, _ = m.step(token_id=ids[:, k], cache=pc)
            out["prime_next"] = nxt.clone()
    return out


def search_case(SM, kw, seed, eval_dim=16, vocab=64):
    """Reference SearchMamba: dynamics_rollout (values, continuation logits,
    consistency features, parameter gradients), prime_board + eval_step chain,
    evaluate_lines_fast with lengths, evaluate_lines and score_branch
    (search_mamba.py:103-291), with non-zero rotation phases (see _set_phases)."""
    torch.manual_seed(seed)
    cfg = SM.SearchMambaConfig(vocab_size=vocab, scan_checkpoint=True, use_triton_scan=False,
                               **kw)
    sm = SM.SearchMamba(cfg, vocab_size=vocab, eval_dim=eval_dim)
    _set_phases(sm.backbone.layers, seed + 100)
    board = torch.randint(1, vocab, (2, 24))
    moves = torch.randint(1, vocab, (2, 6))
    lines = torch.randint(1, vocab, (5, 6))
    lengths = torch.tensor([6, 3, 1, 5, 2])
    out = {"kw": dict(kw), "seed": seed, "eval_dim": eval_dim, "vocab": vocab,
           "board": board, "moves": moves, "lines": lines, "lengths": lengths,
           "state_dict": {k: v.clone() for k, v in sm.state_dict().items()}}
    sm.train()
    v, c, f = sm.dynamics_rollout(board, moves)
    (v.pow(2).mean() + 0.1 * c.pow(2).mean() + f.pow(2).mean()).backward()
    out["rollout"] = (v.detach().clone(), c.detach().clone(), f.detach().clone())
    out["rollout_param_grads"] = {k: p.grad.clone() for k, p in sm.named_parameters()
                                  if p.grad is not None}
    sm.zero_grad(set_to_none=True)
    # the reference's own agreement between two equivalent formulations of the
    # rollout: prime_cache + step loop (above) and one causal forward over the
    # board and the moves.  Some head gradients (the continuation head's first
    # layer, behind a LayerNorm of small variance) amplify fp32 rounding of the
    # hidden states by orders of magnitude; this figure is the floor of any
    # comparison against the fixture.
    Lb = board.shape[1]
    hid = sm.backbone(torch.cat([board, moves], 1))[:, Lb:]
    v2 = torch.tanh(sm.value_head(hid)).squeeze(-1)
    (v2.pow(2).mean() + 0.1 * sm.continuation_head(hid).pow(2).mean()
     + sm.consistency_proj(hid).pow(2).mean()).backward()
    out["rollout_self_consistency"] = {
        k: ((p.grad - out["rollout_param_grads"][k]).abs().max()
            / out["rollout_param_grads"][k].abs().max()).item()
        for k, p in sm.named_parameters() if p.grad is not None}
    sm.zero_grad(set_to_none=True)
    sm.eval()
    with torch.no_grad():
        _, cache = sm.prime_board(board[0])
        vals, conts = [], []
        for t in range(moves.shape[1]):
            val, cont, cache = sm.eval_step(cache, int(moves[0, t]))
            vals.append(val)
            conts.append(cont.clone())
        out["eval_values"] = torch.tensor(vals, dtype=torch.float64)
        out["eval_cont"] = torch.stack(conts)
        out["lines_fast"] = sm.evaluate_lines_fast(board[0], lines, lengths=lengths).clone()
        out["lines_slow"] = sm.evaluate_lines(board[0], lines).clone()
        _, bcache = sm.prime_board(board[1])
        q, logits = sm.score_branch(bcache, moves[1])
        out["branch"] = (float(q), logits.clone())
    return out


def dropin_callsite(ref):
    """The reference's call into the fused-scan module, read from its source
    (mamba.py:343-350): the module name, the names it imports from it, and the
    keyword names of the scan call.  Stored as JSON so that the tests can check
    the drop-in module against it without the reference checkout."""
    import ast
    src_path = os.path.join(ref, "redpanda", "engine", "mamba.py")
    tree = ast.parse(open(src_path).read())
    out = {"file": "redpanda/engine/mamba.py", "imports": [], "calls": []}
    for node in ast.walk(tree):
        if isinstance(node, ast.ImportFrom) and node.module == "triton_scan":
            out["module"] = node.module
            out["imports"] += [a.name for a in node.names]
            out["import_line"] = node.lineno
        if isinstance(node, ast.Call) and getattr(node.func, "id", None) == "triton_trapezoidal_scan":
            out["calls"].append({"line": node.lineno, "n_positional": len(node.args),
                                 "keywords": [k.arg for k in node.keywords]})
    assert out["imports"] and out["calls"], "call site not found"
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("REDPANDA_REFERENCE"),
                    help="checkout of PranavPrasannaV/RedPanda (or set REDPANDA_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("--ref (or REDPANDA_REFERENCE) must name a reference checkout")
    sys.path.insert(0, os.path.join(args.ref, "redpanda", "engine"))
    import mamba as M  # the reference module, read-only
    import search_mamba as SM  # the reference module, read-only

    torch.set_num_threads(1)
    cases = {
        # config-0 shapes with the batch cut to 2 (rows are independent)
        "scan_c0_causal": scan_case(M, ScanShape(2, 64, 256, 16, 4, 4), 0, False),
        "scan_c0_bidir": scan_case(M, ScanShape(2, 64, 256, 16, 4, 4), 1, True),
        # ragged length (not a multiple of the 32-token chunk), no tracking lanes
        "scan_l70_notrack": scan_case(M, ScanShape(2, 70, 64, 16, 0, 2), 2, False),
        # length 1, mostly tracking lanes
        "scan_l1": scan_case(M, ScanShape(3, 1, 32, 12, 8, 2), 3, False),
        # config-1 state layout (16 rot + 16 track) at a tiny batch
        "scan_c1_slice": scan_case(M, ScanShape(1, 33, 128, 32, 16, 4), 4, True),
        # config-3 state layout (24 rot + 8 track)
        "scan_c3_slice": scan_case(M, ScanShape(2, 40, 64, 32, 8, 2), 5, False),
    }
    for name, c in cases.items():
        torch.save(c, os.path.join(HERE, name + ".pt"))
    models = {
        # the reference's own verify() configs (triton_scan.py:353-354)
        "model_verify_trk": model_case(M, dict(d_model=32, n_layer=2, d_state=12,
                                               n_track_state=4, mimo_p=2), 10, 33, False),
        "model_verify_trk_bidir": model_case(M, dict(d_model=32, n_layer=2, d_state=12,
                                                     n_track_state=4, mimo_p=2), 11, 33, True),
        "model_verify_notrk": model_case(M, dict(d_model=48, n_layer=2, d_state=16,
                                                 n_track_state=0, mimo_p=2), 12, 70, False),
        # rotation phases drawn from U(-1.4, 1.4): A_imag != 0 in every rotational lane
        "model_phase_trk": model_case(M, dict(d_model=32, n_layer=2, d_state=12,
                                              n_track_state=4, mimo_p=2), 13, 33, False,
                                      phases=True),
        "model_phase_bidir": model_case(M, dict(d_model=32, n_layer=2, d_state=16,
                                                n_track_state=4, mimo_p=2), 14, 40, True,
                                        phases=True),
    }
    for name, c in models.items():
        torch.save(c, os.path.join(HERE, name + ".pt"))
    searches = {
        "search_phase": search_case(SM, dict(d_model=32, n_layer=2, d_state=12,
                                             n_track_state=4, mimo_p=2), 20),
    }
    for name, c in searches.items():
        torch.save(c, os.path.join(HERE, name + ".pt"))
    import json
    with open(os.path.join(HERE, "dropin_callsite.json"), "w") as f:
        json.dump(dropin_callsite(args.ref), f, indent=1)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
