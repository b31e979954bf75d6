"""Correctness gate of the scan kernels: the counterpart of the reference's
``triton_scan.verify`` (redpanda/engine/triton_scan.py:340-398).

The reference gate compares its fused Triton scan against its own PyTorch
scan, forward and every gradient, over several layer shapes, both directions
and a range of sequence lengths, and raises AssertionError on a mismatch
(tolerances: 2e-3 absolute on the forward, 2e-3 on gradients relative to
max(|grad|, 1)).  Here the fused path is the sm_100a kernels behind
:mod:`redpanda_b200.scan` and the comparison path is a direct float64 torch
restatement of the recurrence (sequential in t, differentiated by autograd),
used by this gate only.
"""

import torch

from . import scan as S

# the reference gate's layer configurations (triton_scan.py:351-354), as scan
# shapes: d_inner = 2 * d_model, d_state, tracking lanes
_CFGS = [dict(d_model=32, d_state=12, n_track_state=4),
         dict(d_model=48, d_state=16, n_track_state=0)]
_THOROUGH_CFG = dict(d_model=512, d_state=64, n_track_state=16)


def _torch_scan(delta, u, Bc, Cc, A_real, A_imag, track):
    """y of the causal trapezoidal scan (redpanda/engine/mamba.py:382-423), by
    the sequential recurrence h[t] = g*h[t-1] + 0.5*dBu[t] + 0.5*g*dBu[t-1]."""
    B, L, D = u.shape
    gates = []
    if A_real is not None:
        dA = delta.unsqueeze(-1) * A_real
        g = torch.exp(dA)
        if A_imag is not None:
            g = g * torch.cos(delta.unsqueeze(-1) * A_imag)
        gates.append(g)
    if track is not None:
        gates.append(track.expand(B, L, *track.shape))
    gate = torch.cat(gates, -1) if len(gates) > 1 else gates[0]
    dbu = (delta * u).unsqueeze(-1) * Bc.unsqueeze(2)
    h = torch.zeros(B, D, gate.shape[-1], dtype=u.dtype, device=u.device)
    prev = torch.zeros_like(h)
    ys = []
    for t in range(L):
        g = gate[:, t]
        h = g * h + 0.5 * dbu[:, t] + 0.5 * g * prev
        prev = dbu[:, t]
        ys.append(torch.einsum("bdn,bn->bd", h, Cc[:, t]))
    return torch.stack(ys, 1)


def _inputs(d_inner, n_state, n_track, L, device, gen):
    n_rot = n_state - n_track
    rnd = lambda *s: torch.randn(*s, device=device, generator=gen)  # noqa: E731
    x = {
        "delta": torch.nn.functional.softplus(rnd(3, L, d_inner) * 0.5 - 2),
        "u": rnd(3, L, d_inner),
        "Bc": rnd(3, L, n_state),
        "Cc": rnd(3, L, n_state),
        "A_real": -torch.exp(rnd(d_inner, n_rot) * 0.5) if n_rot else None,
        "A_imag": (torch.rand(d_inner, n_rot, device=device, generator=gen) * 2 - 1) * 3.14159
        if n_rot else None,
        "track": torch.tanh(rnd(d_inner, n_track)) if n_track else None,
        "dy": rnd(3, L, d_inner),
    }
    return x, n_rot


def verify(device="cuda", thorough=True, verbose=True):
    """Gate: the kernels against the float64 torch recurrence, forward and all
    gradients, causal and bidirectional, across shapes and lengths.  Raises
    AssertionError on any mismatch; returns True (triton_scan.py:340-398)."""
    assert S.HAS_M3, "the m3 scan library or an sm_100 device is not available"
    keys = ("delta", "u", "Bc", "Cc", "A_real", "A_imag", "track")
    gen = torch.Generator(device=device).manual_seed(0)
    cfgs = list(_CFGS) + ([_THOROUGH_CFG] if thorough else [])
    lens = (1, 31, 32, 33, 70, 107, 160) if thorough else (33, 70)
    for kw in cfgs:
        d_inner, n, trk = 2 * kw["d_model"], kw["d_state"], kw["n_track_state"]
        for bidir in (False, True):
            for L in lens:
                x, n_rot = _inputs(d_inner, n, trk, L, device, gen)
                mine = {k: (None if x[k] is None else x[k].clone().requires_grad_(True))
                        for k in keys}
                ref = {k: (None if x[k] is None else x[k].double().requires_grad_(True))
                       for k in keys}
                args = [mine[k] for k in keys]
                if bidir:
                    y = S.m3_bidir_scan(*args, n_rot, n)
                else:
                    y = S.m3_trapezoidal_scan(*args, n_rot, n)
                rargs = [ref[k] for k in keys]
                yr = _torch_scan(*rargs)
                if bidir:
                    flip = lambda t: None if t is None else t.flip(1)  # noqa: E731
                    yr = yr + _torch_scan(flip(ref["delta"]), flip(ref["u"]), flip(ref["Bc"]),
                                          flip(ref["Cc"]), ref["A_real"], ref["A_imag"],
                                          ref["track"]).flip(1)
                fd = (y.double() - yr).abs().max().item()
                assert fd < 2e-3, f"forward mismatch {fd:.2e} cfg={kw} L={L} bidir={bidir}"
                (y * x["dy"]).sum().backward()
                (yr * x["dy"].double()).sum().backward()
                gd = 0.0
                for k in keys:
                    if mine[k] is None:
                        continue
                    gm, gr = mine[k].grad.double(), ref[k].grad
                    denom = gr.abs().max().clamp(min=1.0)
                    gd = max(gd, ((gm - gr).abs().max() / denom).item())
                assert gd < 2e-3, f"grad mismatch {gd:.2e} cfg={kw} L={L} bidir={bidir}"
                if verbose:
                    print(f"  ok cfg(d={kw['d_model']},N={n},trk={trk}) L={L} "
                          f"bidir={int(bidir)} | fwd {fd:.1e} grad {gd:.1e}")
    if verbose:
        print("M3 SCAN VERIFIED: forward + gradients match the reference recurrence.")
    return True
