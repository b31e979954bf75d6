"""Scan-level CPU oracle (test infrastructure; see ``oracle/__init__.py``).

Restates the reference recurrence of ``redpanda/engine/mamba.py`` at the
boundary of ``triton_trapezoidal_scan`` (``redpanda/engine/triton_scan.py:318``):
inputs are the post-softplus ``delta`` (B, L, D), the SSM input ``u`` (B, L, D),
the MIMO-contracted ``Bc``/``Cc`` (B, L, N), the rotational eigenvalues
``A_real``/``A_imag`` (D, n_rot) and the tracking gate ``track`` (D, n_track);
the output ``y`` (B, L, D) excludes the ``u * D`` skip term.

All functions are dtype-generic: run them on float32 tensors to reproduce the
reference's own fp32 numerics, or on float64 tensors for a tie-breaker.
"""

import math

import torch

# Chunk length of the reference's streaming scan (mamba.py:101).
SCAN_CHUNK = 32


def compute_A(A_log_mag, A_phase):
    """Rotational eigenvalues (A_real, A_imag), shape (D, n_rot).

    Follows ``Mamba3Block._compute_A`` (mamba.py:211-224), complex branch:
    magnitude ``-exp(A_log_mag)``, rotated by ``A_phase``.
    """
    mag = -torch.exp(A_log_mag)
    return mag * torch.cos(A_phase), mag * torch.sin(A_phase)


def track_gate(theta):
    """Tracking-channel eigenvalue tanh(theta) (mamba.py:227-229)."""
    return torch.tanh(theta)


def pad_params(A_real, A_imag, track, n_rot, n_state, d_inner, dtype=torch.float32):
    """Pad the per-group eigenvalues to (D, N) the way triton_scan.py:325-335 does.

    Rotational lanes occupy state columns [0, n_rot) of ``Ar_p``/``Ai_p``;
    tracking lanes occupy columns [n_rot, N) of ``Tk_p``; the rest is zero.
    """
    z = torch.zeros(d_inner, n_state, dtype=dtype)
    Ar_p, Ai_p, Tk_p = z.clone(), z.clone(), z.clone()
    if A_real is not None:
        Ar_p[:, :n_rot] = A_real.to(dtype)
        if A_imag is not None:
            Ai_p[:, :n_rot] = A_imag.to(dtype)
    if track is not None:
        Tk_p[:, n_rot:] = track.to(dtype)
    return Ar_p, Ai_p, Tk_p


def parallel_scan(gates, tokens):
    """Inclusive Hillis-Steele scan of h[t] = gates[t]*h[t-1] + tokens[t], h[-1]=0.

    Same doubling schedule as mamba.py:104-136 (stride 1, 2, 4, ... over dim 1),
    so the fp32 rounding matches the reference's.
    """
    a, b = gates, tokens
    n = a.shape[1]
    s = 1
    while s < n:
        b = torch.cat([b[:, :s], a[:, s:] * b[:, :-s] + b[:, s:]], dim=1)
        a = torch.cat([a[:, :s], a[:, s:] * a[:, :-s]], dim=1)
        s <<= 1
    return b


def _gates(delta_c, A_real, A_imag, track):
    """Per-token gate tensor (B, c, D, N) (mamba.py:396-405)."""
    nb, c, d = delta_c.shape
    parts = []
    if A_real is not None:
        g = torch.exp(torch.einsum("bld,dn->bldn", delta_c, A_real))
        if A_imag is not None:
            g = g * torch.cos(torch.einsum("bld,dn->bldn", delta_c, A_imag))
        parts.append(g)
    if track is not None:
        parts.append(track.view(1, 1, d, -1).expand(nb, c, d, -1))
    return parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)


def _chunk(delta_c, u_c, B_c, C_c, h, dbu_carry, A_real, A_imag, track):
    """One chunk of the streaming scan; returns (y_c, h_last, dBu_last).

    Follows ``Mamba3Block._scan_chunk`` (mamba.py:382-423): trapezoidal tokens
    0.5*dBu[t] + 0.5*g[t]*dBu[t-1], the carried state folded into token 0, then
    the Hillis-Steele scan and the contraction with C.
    """
    g = _gates(delta_c, A_real, A_imag, track)
    dbu = torch.einsum("bld,bln->bldn", delta_c, B_c) * u_c.unsqueeze(-1)
    if dbu_carry is None:
        dbu_carry = torch.zeros_like(dbu[:, 0])
    dbu_shift = torch.cat([dbu_carry.unsqueeze(1), dbu[:, :-1]], dim=1)
    tok = 0.5 * dbu + 0.5 * g * dbu_shift
    first = tok[:, 0] + g[:, 0] * h.to(g.dtype)
    tok = torch.cat([first.unsqueeze(1), tok[:, 1:]], dim=1)
    hs = parallel_scan(g, tok)
    y_c = torch.einsum("bldn,bln->bld", hs, C_c)
    return y_c, hs[:, -1], dbu[:, -1]


def scan_chunked(delta, u, Bc, Cc, A_real, A_imag, track, return_state=False,
                 chunk=SCAN_CHUNK):
    """The reference's PyTorch scan path without the skip term.

    Follows ``Mamba3Block._selective_scan_trapezoidal`` (mamba.py:352-380):
    chunks of ``SCAN_CHUNK`` tokens, fp32 carry state (the carry uses the input
    dtype here so that a float64 run stays float64).  Activation checkpointing
    (mamba.py:358-371) recomputes the same values, so it is not modelled.
    Returns ``y`` or ``(y, (h_last, dBu_last))`` as mamba.py:377-380 does.
    """
    nb, L, d = u.shape
    n = Bc.shape[-1]
    h = torch.zeros(nb, d, n, dtype=delta.dtype, device=delta.device)
    carry = None
    ys = []
    for s in range(0, L, chunk):
        e = min(s + chunk, L)
        y_c, h, carry = _chunk(delta[:, s:e], u[:, s:e], Bc[:, s:e], Cc[:, s:e],
                               h, carry, A_real, A_imag, track)
        ys.append(y_c)
    y = torch.cat(ys, dim=1)
    if return_state:
        return y, (h, carry)
    return y


def scan_bidir(delta, u, Bc, Cc, A_real, A_imag, track):
    """Bidirectional scan without skip terms: scan(x) + flip(scan(flip(x))).

    Mirrors the bidirectional branch of ``Mamba3Block.forward``
    (mamba.py:254-260).  The reference adds ``u*D`` once per direction; the
    caller of this function adds ``2*u*D`` when it needs the block output.
    """
    y = scan_chunked(delta, u, Bc, Cc, A_real, A_imag, track)
    yb = scan_chunked(delta.flip(1), u.flip(1), Bc.flip(1), Cc.flip(1),
                      A_real, A_imag, track)
    return y + yb.flip(1)


def scan_sequential(delta, u, Bc, Cc, A_real, A_imag, track, reverse=False):
    """Plain time loop of the same recurrence (math spec; use with float64).

    gate = exp(delta*A_real)*cos(delta*A_imag) (rotational lanes) or
    tanh(theta) (tracking lanes); dBu = delta*B*u;
    h[t] = gate*h[t-1] + 0.5*dBu[t] + 0.5*gate*dBu[t-1]; y[t] = sum_n h*C
    (the recurrence stated at triton_scan.py:7-12 and mamba.py:307-308).
    Returns (y, h_last, dbu_last).
    """
    nb, L, d = u.shape
    n = Bc.shape[-1]
    h = torch.zeros(nb, d, n, dtype=delta.dtype, device=delta.device)
    dbu_prev = torch.zeros(nb, d, n, dtype=delta.dtype, device=delta.device)
    y = torch.zeros(nb, L, d, dtype=delta.dtype, device=delta.device)
    order = range(L - 1, -1, -1) if reverse else range(L)
    for t in order:
        g = _gates(delta[:, t:t + 1], A_real, A_imag, track)[:, 0]
        dbu = delta[:, t, :, None] * Bc[:, t, None, :] * u[:, t, :, None]
        h = g * h + 0.5 * dbu + 0.5 * g * dbu_prev
        dbu_prev = dbu
        y[:, t] = (h * Cc[:, t, None, :]).sum(-1)
    return y, h, dbu_prev


def scan_with_grads(delta, u, Bc, Cc, A_real, A_imag, track, dy, bidir=False):
    """Forward + reference autograd gradients of sum(y * dy).

    The reference's backward for the PyTorch path is plain autograd through
    the ops above (mamba.py:358-375).  Returns (y, grads) where grads has keys
    delta, u, Bc, Cc, A_real, A_imag, track (None where the input is None).
    """
    leaves = {}
    def leaf(name, t):
        if t is None:
            leaves[name] = None
            return None
        x = t.detach().clone().requires_grad_(True)
        leaves[name] = x
        return x
    dl, uu, bb, cc = (leaf("delta", delta), leaf("u", u), leaf("Bc", Bc), leaf("Cc", Cc))
    ar, ai, tk = leaf("A_real", A_real), leaf("A_imag", A_imag), leaf("track", track)
    if bidir:
        y = scan_bidir(dl, uu, bb, cc, ar, ai, tk)
    else:
        y = scan_chunked(dl, uu, bb, cc, ar, ai, tk)
    (y * dy.to(y.dtype)).sum().backward()
    grads = {k: (None if v is None else v.grad.detach()) for k, v in leaves.items()}
    return y.detach(), grads


def step_cells(h, dbu_prev, delta_t, u_t, Bc_t, Cc_t, A_real, A_imag, track):
    """One O(1) recurrent step at the recurrence boundary (no skip term).

    Follows ``Mamba3Block.step`` (mamba.py:466-493): gate as in the scan,
    dBu_t formed as (delta*u)*B (mamba.py:481, a different product order from
    the scan's (delta*B)*u), tokens and state update, y = sum_n h*C.
    Shapes: h, dbu_prev (B, D, N); delta_t, u_t (B, D); Bc_t, Cc_t (B, N).
    Returns (y (B, D), h_new, dbu_t).
    """
    g = _gates(delta_t.unsqueeze(1), A_real, A_imag, track)[:, 0]
    dbu = (delta_t * u_t).unsqueeze(-1) * Bc_t.unsqueeze(1)
    tok = 0.5 * dbu + 0.5 * g * dbu_prev
    h = g * h + tok
    y = torch.einsum("bdn,bn->bd", h, Cc_t)
    return y, h, dbu


def default_chunks(L):
    """Number of reference scan chunks for a sequence of length L."""
    return int(math.ceil(L / SCAN_CHUNK))
