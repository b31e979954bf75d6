"""Seeded synthetic scan inputs with the benchmark's shapes and distributions.

The scan configurations have no dataset behind them: every input is drawn from
a seeded CPU generator in a fixed order (x, dt, A_re, A_im, theta, B, C, dy):

* u = x ~ N(0, 1), shape (B, L, D)
* delta = softplus(N(-2, 0.5)), shape (B, L, D)
* A_real = -exp(N(0, 0.5)), A_imag ~ U(-pi, pi), shape (D, n_rot)
* track = tanh(theta), theta ~ N(0, 1), shape (D, n_track)
* B_raw, C_raw ~ N(0, 1) / sqrt(N) on (B, L, N*p), RMS-normalised over the
  N*p vector with unit weight and eps 1e-5 (BCNorm, reference
  ``redpanda/engine/mamba.py:82-89,295-299``), viewed as (B, L, N, p) and
  summed over p (the MIMO fold, mamba.py:336-337)
* dy ~ N(0, 1), shape (B, L, D)
"""

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class ScanShape:
    batch: int
    seqlen: int
    d_inner: int
    d_state: int
    n_track: int
    mimo_p: int = 4

    @property
    def n_rot(self):
        return self.d_state - self.n_track


# The benchmark configurations (shapes only).
C0 = ScanShape(8, 64, 256, 16, 4, 4)        # CPU-runnable reference case
C1 = ScanShape(1024, 64, 1536, 32, 16, 4)   # Eval-Mamba bidirectional forward
C2 = C1                                      # backward at the same shape
C3 = ScanShape(8192, 64, 1024, 32, 8, 2)    # Search-Mamba prime / step rows


def bcnorm_fold(raw, n_state, p, eps=1e-5):
    """RMSNorm over the N*p vector (unit weight), then the sum over p."""
    normed = raw * torch.rsqrt(raw.pow(2).mean(-1, keepdim=True) + eps)
    return normed.view(*raw.shape[:-1], n_state, p).sum(-1)


def make_scan_inputs(shape: ScanShape, seed: int = 0, dtype=torch.float32):
    """Draw one seeded set of scan inputs on the CPU (float32 draws).

    Returns a dict with delta, u, Bc, Cc (cast to ``dtype``), A_real, A_imag,
    track (float32 or None when the group is empty), theta and dy (float32).
    """
    g = torch.Generator("cpu").manual_seed(seed)
    b, L, d, n, p = shape.batch, shape.seqlen, shape.d_inner, shape.d_state, shape.mimo_p
    x = torch.randn(b, L, d, generator=g)
    dt = torch.randn(b, L, d, generator=g) * 0.5 - 2.0
    a_re = -torch.exp(torch.randn(d, shape.n_rot, generator=g) * 0.5)
    a_im = (torch.rand(d, shape.n_rot, generator=g) * 2.0 - 1.0) * math.pi
    theta = torch.randn(d, shape.n_track, generator=g)
    b_raw = torch.randn(b, L, n * p, generator=g) / math.sqrt(n)
    c_raw = torch.randn(b, L, n * p, generator=g) / math.sqrt(n)
    dy = torch.randn(b, L, d, generator=g)
    out = {
        "delta": F.softplus(dt).to(dtype),
        "u": x.to(dtype),
        "Bc": bcnorm_fold(b_raw, n, p).to(dtype),
        "Cc": bcnorm_fold(c_raw, n, p).to(dtype),
        "A_real": a_re if shape.n_rot > 0 else None,
        "A_imag": a_im if shape.n_rot > 0 else None,
        "track": torch.tanh(theta) if shape.n_track > 0 else None,
        "theta": theta,
        "dy": dy,
    }
    return out
