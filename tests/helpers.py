"""Shared helpers of the parity tests: seeded inputs, oracle runs, error metrics."""

import torch

import oracle as O
from redpanda_b200.synthetic import ScanShape, make_scan_inputs

GRAD_KEYS = ("delta", "u", "Bc", "Cc", "A_real", "A_imag", "track")


def rel_err(a, ref):
    """Norm-wise relative error max|a - ref| / max|ref| (0 when both are 0)."""
    a = a.detach().double().cpu()
    ref = ref.detach().double().cpu()
    den = ref.abs().max().item()
    num = (a - ref).abs().max().item()
    if den == 0.0:
        return num
    return num / den


def inputs(shape: ScanShape, seed=0, dtype=torch.float32):
    """Seeded inputs; floating inputs are rounded to ``dtype`` then held in fp32 for the oracle."""
    inp = make_scan_inputs(shape, seed=seed, dtype=dtype)
    return inp


def oracle_scan(inp, direction, dtype=torch.float64, with_grads=True):
    """Oracle y (and grads) for direction 0 (causal), 1 (reverse) or 2 (bidirectional)."""
    def cvt(x):
        return None if x is None else x.to(dtype)
    d, u, b, c = (cvt(inp[k]) for k in ("delta", "u", "Bc", "Cc"))
    ar, ai, tk = cvt(inp["A_real"]), cvt(inp["A_imag"]), cvt(inp["track"])
    dy = inp["dy"].to(dtype)
    if direction == 1:
        flip = lambda x: None if x is None else x.flip(1)  # noqa: E731
        y, g = O.scan_with_grads(flip(d), flip(u), flip(b), flip(c), ar, ai, tk, flip(dy))
        y = y.flip(1)
        for k in ("delta", "u", "Bc", "Cc"):
            g[k] = g[k].flip(1)
        return y, g
    return O.scan_with_grads(d, u, b, c, ar, ai, tk, dy, bidir=(direction == 2))


def to_cuda(inp, dev="cuda"):
    return {k: (None if v is None else v.to(dev)) for k, v in inp.items()}
