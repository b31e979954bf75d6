"""Block- and model-level CPU oracle (test infrastructure; see ``oracle/__init__.py``).

A functional restatement of ``Mamba3Block`` and ``Mamba`` from
``redpanda/engine/mamba.py`` operating on a ``state_dict``-style parameter
mapping with the reference's parameter names (``in_proj.weight``,
``x_proj.weight``, ``A_log_mag`` ...).  It covers the calls on the scan/step hot
path: ``forward`` (causal and bidirectional), ``forward_with_state``, ``step``,
``Mamba.step`` and ``Mamba.prime_cache``.
"""

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import scan_oracle as so


@dataclass
class OracleConfig:
    """The hot-path fields of ``MambaConfig`` (mamba.py:24-78)."""
    d_model: int = 512
    n_layer: int = 16
    vocab_size: int = 8192
    d_state: int = 64
    expand: int = 2
    dt_rank: int = 0          # 0 = 'auto' = ceil(d_model / 16) (mamba.py:67-68)
    mimo_p: int = 4
    n_track_state: int = 0
    bidirectional: bool = False
    use_bcnorm: bool = True

    @property
    def d_inner(self):
        return self.expand * self.d_model

    @property
    def rank(self):
        return self.dt_rank if self.dt_rank else math.ceil(self.d_model / 16)

    @property
    def n_rot(self):
        return self.d_state - self.n_track_state


def _rms(x, w, eps=1e-5):
    """RMSNorm.forward (mamba.py:88-89)."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _lin(x, p, name):
    b = p.get(name + ".bias")
    return F.linear(x, p[name + ".weight"], b)


def _A(p, cfg):
    if cfg.n_rot == 0:
        return None, None
    return so.compute_A(p["A_log_mag"].float(), p["A_phase"].float())


def _track(p, cfg):
    return so.track_gate(p["track_theta"].float()) if cfg.n_track_state > 0 else None


def ssm_proj(p, cfg, u):
    """Per-token projections u -> (delta, B, C) (mamba.py:284-301).

    Works for (B, L, D) and (B, D) inputs; B and C are returned with a trailing
    MIMO axis of size ``mimo_p``.
    """
    n, pp = cfg.d_state, cfg.mimo_p
    x_dbl = _lin(u, p, "x_proj")
    dt_raw, B_raw, C_raw = x_dbl.split([cfg.rank, n * pp, n * pp], dim=-1)
    if cfg.use_bcnorm:
        B_raw = _rms(B_raw, p["b_norm.weight"])
        C_raw = _rms(C_raw, p["c_norm.weight"])
    B = B_raw.view(*u.shape[:-1], n, pp)
    C = C_raw.view(*u.shape[:-1], n, pp)
    delta = F.softplus(_lin(dt_raw, p, "dt_proj"))
    return delta, B, C


def block_ssm(p, cfg, u, return_state=False):
    """``Mamba3Block.ssm`` + ``_selective_scan_trapezoidal`` (mamba.py:303-380)."""
    delta, B, C = ssm_proj(p, cfg, u)
    Ar, Ai = _A(p, cfg)
    out = so.scan_chunked(delta, u, B.sum(-1), C.sum(-1), Ar, Ai, _track(p, cfg),
                          return_state=return_state)
    if return_state:
        y, st = out
        return y + u * p["D"], st
    return out + u * p["D"]


def block_forward(p, cfg, x):
    """``Mamba3Block.forward`` (mamba.py:231-267), causal or bidirectional."""
    xb, z = _lin(x, p, "in_proj").chunk(2, dim=-1)
    xb = F.silu(xb)
    if not cfg.bidirectional:
        y = block_ssm(p, cfg, xb)
    else:
        delta, B, C = ssm_proj(p, cfg, xb)
        Ar, Ai = _A(p, cfg)
        tk = _track(p, cfg)
        Bc, Cc = B.sum(-1), C.sum(-1)
        y = so.scan_chunked(delta, xb, Bc, Cc, Ar, Ai, tk) + xb * p["D"]
        yb = so.scan_chunked(delta.flip(1), xb.flip(1), Bc.flip(1),
                             Cc.flip(1), Ar, Ai, tk) + xb.flip(1) * p["D"]
        y = y + yb.flip(1)
    return _lin(y * F.silu(z), p, "out_proj")


def block_forward_with_state(p, cfg, x):
    """``Mamba3Block.forward_with_state`` (mamba.py:269-282)."""
    xb, z = _lin(x, p, "in_proj").chunk(2, dim=-1)
    xb = F.silu(xb)
    y, st = block_ssm(p, cfg, xb, return_state=True)
    return _lin(y * F.silu(z), p, "out_proj"), st


def block_step(p, cfg, x_t, state=None):
    """``Mamba3Block.step`` (mamba.py:427-498): one token, returns (out, (h, dBu))."""
    xb, z = _lin(x_t, p, "in_proj").chunk(2, dim=-1)
    xb = F.silu(xb)
    delta, B, C = ssm_proj(p, cfg, xb)
    Ar, Ai = _A(p, cfg)
    nb = x_t.shape[0]
    if state is None:
        h = torch.zeros(nb, cfg.d_inner, cfg.d_state, dtype=x_t.dtype)
        dbu_prev = torch.zeros_like(h)
    else:
        h, dbu_prev = state
    y, h, dbu = so.step_cells(h, dbu_prev, delta, xb, B.sum(-1), C.sum(-1), Ar, Ai,
                              _track(p, cfg))
    y = y + xb * p["D"]
    return _lin(y * F.silu(z), p, "out_proj"), (h, dbu)


def _layer(p, i):
    pre = f"layers.{i}.mixer."
    return {k[len(pre):]: v for k, v in p.items() if k.startswith(pre)}


def model_forward(p, cfg, ids):
    """``Mamba.forward`` (mamba.py:534-556) without layer checkpointing."""
    x = F.embedding(ids, p["embedding.weight"])
    for i in range(cfg.n_layer):
        x = x + block_forward(_layer(p, i), cfg, _rms(x, p[f"layers.{i}.norm.weight"]))
    return _rms(x, p["norm_f.weight"])


def model_step(p, cfg, token_id, cache=None, apply_final_norm=True):
    """``Mamba.step`` (mamba.py:564-601)."""
    if token_id.dim() == 2:
        token_id = token_id.squeeze(1)
    x = F.embedding(token_id, p["embedding.weight"])
    cache = cache if cache is not None else [None] * cfg.n_layer
    new = []
    for i in range(cfg.n_layer):
        d, st = block_step(_layer(p, i), cfg, _rms(x, p[f"layers.{i}.norm.weight"]), cache[i])
        x = x + d
        new.append(st)
    if apply_final_norm:
        x = _rms(x, p["norm_f.weight"])
    return x, new


def model_prime_cache(p, cfg, ids):
    """``Mamba.prime_cache`` (mamba.py:603-620)."""
    cur = F.embedding(ids, p["embedding.weight"])
    cache = []
    for i in range(cfg.n_layer):
        mixed, st = block_forward_with_state(_layer(p, i), cfg,
                                             _rms(cur, p[f"layers.{i}.norm.weight"]))
        cur = cur + mixed
        cache.append(st)
    return _rms(cur[:, -1, :], p["norm_f.weight"]), cache
