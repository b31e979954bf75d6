"""Mamba-3 backbone whose scan and recurrent step run on the sm_100a kernels.

Host-side mirror of ``redpanda/engine/mamba.py`` (the reference's backbone)
with the same class names, constructor arguments, parameter names and
initialisation, so a reference ``state_dict`` loads unchanged.  The
projections (``in_proj``, ``x_proj``, ``dt_proj``, ``out_proj``) are cuBLAS
GEMMs, as in the reference, except in the small-batch lockstep step, where
the library's matrix-vector kernels run them with the norm, silu and residual
folded in; the recurrences go through :mod:`redpanda_b200.scan`:

* causal scan (``_selective_scan_trapezoidal``, mamba.py:318-380) ->
  ``m3_trapezoidal_scan`` (forward + analytic backward)
* ``return_state`` priming (mamba.py:377-379) -> ``m3_scan_with_state``
* bidirectional pair (mamba.py:254-260) -> one fused ``m3_bidir_scan`` launch
* ``Mamba3Block.step`` recurrence (mamba.py:466-493) -> ``m3_step``

There is no CPU path: the scan ops raise on CPU tensors.
"""

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import scan as S


@dataclass
class MambaConfig:
    """Fields and defaults of the reference ``MambaConfig`` (mamba.py:24-62)."""
    d_model: int = 512
    n_layer: int = 16
    vocab_size: int = 8192
    d_state: int = 64
    expand: int = 2
    dt_rank: int = 'auto'
    pad_vocab_size_multiple: int = 8
    bias: bool = False
    use_complex: bool = True
    mimo_p: int = 4
    use_bcnorm: bool = True
    n_track_state: int = 0
    bidirectional: bool = False
    grad_checkpoint: bool = False
    scan_checkpoint: bool = True     # accepted for compatibility; the kernels checkpoint themselves
    use_triton_scan: bool = False    # accepted for compatibility; the kernels are always used

    def __post_init__(self):
        self.d_inner = int(self.expand * self.d_model)
        if self.dt_rank == 'auto':
            self.dt_rank = math.ceil(self.d_model / 16)
        assert 0 <= self.n_track_state < self.d_state, "n_track_state must be < d_state"
        self.n_rot_state = self.d_state - self.n_track_state
        if self.vocab_size % self.pad_vocab_size_multiple != 0:
            self.vocab_size += (self.pad_vocab_size_multiple
                                - self.vocab_size % self.pad_vocab_size_multiple)


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight (mamba.py:82-89)."""

    def __init__(self, d: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        if not torch.is_grad_enabled():   # inference: torch's fused kernel, same formula
            return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


def _bf16_layer():
    """True under torch.autocast("cuda", dtype=torch.bfloat16), the reference's
    mixed-precision training (train.py:268): the layer then runs the bf16
    configuration of the kernels -- bf16 delta, u, Bc, Cc into the scan (the
    config-1/2 element types), a bf16 y with fp32 state and accumulation, and
    the gated output in bf16 for the bf16 out_proj GEMM."""
    return (torch.is_autocast_enabled("cuda")
            and torch.get_autocast_dtype("cuda") == torch.bfloat16)


class Mamba3Block(nn.Module):
    """One Mamba-3 layer (mamba.py:141-498) with the recurrences on the kernels."""

    # bf16 layers can run the scan with its prologue fused into the kernels
    # (m3_scan_fwd_fused / m3_scan_bwd_fused; identical results).  Off by
    # default: measured on a B200 the fused pair is slower than the separate
    # HBM-bound prologue launch plus the scans, because the scan kernels are
    # issue-bound and the fused staging repeats softplus per direction and the
    # BCNorm per channel tile on their critical path (bench.py, configs line
    # c2_fused_prologue_bidir).
    fuse_prologue = False
    # the fused step layer (step_fused_) computes softplus, BCNorm and the MIMO
    # fold inside the step kernel (m3_step_gated_fused, bit-identical to the
    # two launches) for batches of at most fuse_step_max_batch rows, and runs
    # m3_step_inputs + m3_step_gated_ above that.  Measured on a B200 (the
    # 12-layer config-3 stack replayed as a CUDA graph, per step): 390 vs 474 us
    # at B=1, 872 vs 920 us at B=256, but 1.88 vs 1.79 ms at B=1024, 5.96 vs
    # 5.44 ms at B=4096 and 11.8 vs 10.7 ms at B=8192 -- small batches are
    # launch-latency-bound and gain a launch per layer, large ones are
    # HBM-bound and lose more to the per-row-pair BCNorm and barrier in every
    # channel-tile CTA than the delta/Bc/Cc round trip costs.
    fuse_step = True
    fuse_step_max_batch = 512
    # Lockstep batches of at most this many rows (a search node, a few lines)
    # run the whole step layer on the library's small-batch kernels, four
    # launches per layer (``step_small_``): their projections are
    # matrix-vector products, where launch latency, not arithmetic, sets the
    # time.  0 disables it.
    small_step_max_batch = 8

    def __init__(self, config: MambaConfig):
        super().__init__()
        self.config = config
        d_inner, n = config.d_inner, config.d_state
        n_rot, n_track, p = config.n_rot_state, config.n_track_state, config.mimo_p
        self.in_proj = nn.Linear(config.d_model, d_inner * 2, bias=config.bias)
        self.x_proj = nn.Linear(d_inner, config.dt_rank + n * p * 2, bias=True)
        self.dt_proj = nn.Linear(config.dt_rank, d_inner, bias=True)
        with torch.no_grad():
            # dt bias: softplus^-1 of log-uniform timescales in [1e-3, 1e-1]
            dt0 = torch.exp(torch.rand(d_inner) * (math.log(0.1) - math.log(0.001))
                            + math.log(0.001))
            self.dt_proj.bias.copy_(dt0 + torch.log(-torch.expm1(-dt0)))
            self.dt_proj.bias._no_reinit = True
        if n_rot > 0:
            mags = torch.arange(1, n_rot + 1, dtype=torch.float32).repeat(d_inner, 1)
            if config.use_complex:
                self.A_log_mag = nn.Parameter(torch.log(mags))
                self.A_phase = nn.Parameter(torch.zeros(d_inner, n_rot))
            else:
                self.A_log = nn.Parameter(torch.log(mags))
        if n_track > 0:
            theta = torch.atanh(torch.linspace(-0.95, 0.95, n_track).clamp(-0.999, 0.999))
            self.track_theta = nn.Parameter(theta.unsqueeze(0).repeat(d_inner, 1))
        if config.use_bcnorm:
            self.b_norm = RMSNorm(n * p)
            self.c_norm = RMSNorm(n * p)
        self.D = nn.Parameter(torch.ones(d_inner))
        self.out_proj = nn.Linear(d_inner, config.d_model, bias=config.bias)

    # -- eigenvalues (mamba.py:211-229)
    def _compute_A(self):
        if self.config.n_rot_state == 0:
            return None, None
        if self.config.use_complex:
            mag = -torch.exp(self.A_log_mag.float())
            phase = self.A_phase.float()
            return mag * torch.cos(phase), mag * torch.sin(phase)
        return -torch.exp(self.A_log.float()), None

    def _track_gate(self):
        return torch.tanh(self.track_theta.float())

    # -- projections (mamba.py:284-301)
    def _ssm_proj(self, u):
        cfg = self.config
        n, p = cfg.d_state, cfg.mimo_p
        x_dbl = self.x_proj(u)
        dt_raw, B_raw, C_raw = x_dbl.split([cfg.dt_rank, n * p, n * p], dim=-1)
        if cfg.use_bcnorm:
            B_raw = self.b_norm(B_raw)
            C_raw = self.c_norm(C_raw)
        B = B_raw.view(*u.shape[:-1], n, p)
        C = C_raw.view(*u.shape[:-1], n, p)
        delta = F.softplus(self.dt_proj(dt_raw))
        return delta, B, C

    def _projections(self, u):
        """x_proj output and dt = dt_proj(dt_raw) (mamba.py:287-300)."""
        x_dbl = self.x_proj(u)
        return x_dbl, self.dt_proj(x_dbl[..., :self.config.dt_rank])

    def _fused_scan(self, u, x_dbl, dt, direction):
        """The bf16 layer's scan with its prologue fused into the kernels
        (m3_scan_fwd_fused / m3_scan_bwd_fused), or None when it does not apply
        (fuse_prologue off, non-bf16 projections, a shape the staging cannot
        take): the caller then runs m3_step_inputs and the scan."""
        cfg = self.config
        if not self.fuse_prologue or not (x_dbl.dtype == dt.dtype == u.dtype == torch.bfloat16):
            return None
        n, p = cfg.d_state, cfg.mimo_p
        bw = self.b_norm.weight if cfg.use_bcnorm else None
        cw = self.c_norm.weight if cfg.use_bcnorm else None
        eps = self.b_norm.eps if cfg.use_bcnorm else 0.0
        track = self._track_gate() if cfg.n_track_state > 0 else None
        A_real, A_imag = self._compute_A()
        try:
            return S.m3_fused_scan(dt, x_dbl, bw, cw, eps, u, A_real, A_imag, track,
                                   cfg.n_rot_state, n, p, cfg.dt_rank, cfg.dt_rank + n * p,
                                   direction, y_dtype=torch.bfloat16)
        except S.FusedUnsupported:
            return None

    def _ssm_inputs(self, u, x_dbl=None, dt=None):
        """(delta, Bc, Cc) of a sequence for the training path: the x_proj and
        dt_proj GEMMs in torch, softplus + BCNorm + MIMO fold (and their
        backward) in one launch each (m3_step_inputs / m3_step_inputs_bwd)."""
        cfg = self.config
        n, p = cfg.d_state, cfg.mimo_p
        lead = u.shape[:-1]
        if x_dbl is None:
            x_dbl, dt = self._projections(u)
        rows = u.numel() // cfg.d_inner
        bw = self.b_norm.weight if cfg.use_bcnorm else None
        cw = self.c_norm.weight if cfg.use_bcnorm else None
        eps = self.b_norm.eps if cfg.use_bcnorm else 0.0
        delta, bc, cc = S.step_inputs(dt.reshape(rows, cfg.d_inner), x_dbl.reshape(rows, -1),
                                      cfg.dt_rank, cfg.dt_rank + n * p, bw, cw, eps, n, p)
        return delta.view(*lead, cfg.d_inner), bc.view(*lead, n), cc.view(*lead, n)

    def _scan_args(self, delta, u, B, C):
        cfg = self.config
        track = self._track_gate() if cfg.n_track_state > 0 else None
        A_real, A_imag = self._compute_A()
        return (delta, u, B.sum(dim=-1), C.sum(dim=-1), A_real, A_imag, track,
                cfg.n_rot_state, cfg.d_state)

    def _selective_scan_trapezoidal(self, u, delta, A_real, A_imag, B, C, D,
                                    return_state=False):
        """Same contract as mamba.py:318-380: returns y + u*D (and the state)."""
        cfg = self.config
        track = self._track_gate() if cfg.n_track_state > 0 else None
        args = (delta, u, B.sum(dim=-1), C.sum(dim=-1), A_real, A_imag, track,
                cfg.n_rot_state, cfg.d_state)
        if return_state:
            y, state = S.m3_scan_with_state(*args)
            return y + u * D, state
        return S.m3_trapezoidal_scan(*args) + u * D

    def ssm(self, u, return_state=False):
        delta, B, C = self._ssm_proj(u)
        A_real, A_imag = self._compute_A()
        return self._selective_scan_trapezoidal(u, delta, A_real, A_imag, B, C, self.D,
                                                return_state=return_state)

    def _silu_x(self, xz):
        """u = silu(x half of in_proj's output) (mamba.py:243, 452): fp32 rows in
        one launch that reads the half in place (m3_silu, torch's rounding);
        a bf16 layer's activations through torch."""
        d_in = self.config.d_inner
        if xz.dtype != torch.float32 or not xz.is_contiguous():
            return F.silu(xz[..., :d_in])
        rows = xz.numel() // (2 * d_in)
        return S.m3_silu(xz.view(rows, 2 * d_in)[:, :d_in]).view(*xz.shape[:-1], d_in)

    def _dt(self, x_dbl):
        """(dt, bias) for the prologue kernels: fp32 layers take dt_proj without
        its bias and add the bias inside m3_step_inputs / m3_step_gated_fused
        (one fp32 add, as torch's matmul-then-add of a strided input); a bf16
        layer's dt_proj output as autocast gives it, bias included."""
        cfg = self.config
        raw = x_dbl[..., :cfg.dt_rank]
        if x_dbl.dtype != torch.float32 or _bf16_layer():
            return self.dt_proj(raw), None
        return F.linear(raw, self.dt_proj.weight), self.dt_proj.bias

    def _forward_inference(self, x, return_state, residual=None, state_out=None):
        """No-grad layer forward on the fused kernels (mamba.py:231-282): after
        the in_proj / x_proj / dt_proj GEMMs, softplus + BCNorm + MIMO fold of
        every token is one launch (m3_step_inputs over B*L rows), the scan (or
        the fused bidirectional pair) another, (y + u*D)*silu(z) a third
        (m3_gate), then out_proj.  ``state_out``: (h, dBu) tensors that receive
        the final state (with ``return_state``)."""
        cfg = self.config
        n, p, d_in = cfg.d_state, cfg.mimo_p, cfg.d_inner
        bf16 = _bf16_layer()
        xz = self.in_proj(x)
        u = self._silu_x(xz)
        x_dbl = self.x_proj(u)
        dt, dt_bias = self._dt(x_dbl)
        lead = u.shape[:-1]
        rows = u.numel() // d_in
        bw = self.b_norm.weight if cfg.use_bcnorm else None
        cw = self.c_norm.weight if cfg.use_bcnorm else None
        eps = self.b_norm.eps if cfg.use_bcnorm else 0.0
        coef = 2.0 if cfg.bidirectional else 1.0
        state = y = None
        if bf16:
            u = u.to(torch.bfloat16)
            if not return_state:   # the prologue fused into the scan
                y = self._fused_scan(u, x_dbl, dt,
                                     S.M3_DIR_BIDIR if cfg.bidirectional else S.M3_DIR_FWD)
        if y is None:
            delta, bc, cc = S.m3_step_inputs(dt.reshape(rows, d_in), x_dbl.reshape(rows, -1),
                                             cfg.dt_rank, cfg.dt_rank + n * p, bw, cw, eps, n, p,
                                             dt_bias=dt_bias)
            delta, bc, cc = delta.view(*lead, d_in), bc.view(*lead, n), cc.view(*lead, n)
            if bf16:
                bf = torch.bfloat16
                delta, bc, cc = delta.to(bf), bc.to(bf), cc.to(bf)
            yd = torch.bfloat16 if bf16 else None
            track = self._track_gate() if cfg.n_track_state > 0 else None
            A_real, A_imag = self._compute_A()
            args = (delta, u, bc, cc, A_real, A_imag, track, cfg.n_rot_state, n)
            if cfg.bidirectional:
                y = S.m3_bidir_scan(*args, y_dtype=yd)
            elif return_state:
                y, state = S.m3_scan_with_state(*args, state_out=state_out)
            else:
                y = S.m3_trapezoidal_scan(*args, y_dtype=yd)
        y = S.m3_gate(y, u, xz[..., d_in:], self.D, coef,
                      out=None if (bf16 and y.dtype != torch.bfloat16) else y,
                      out_dtype=torch.bfloat16 if bf16 else None)
        if residual is None:
            out = self.out_proj(y)
        elif bf16:   # bf16 out_proj; the residual stream stays in its own (fp32) dtype
            out = residual + self.out_proj(y)
        else:   # residual + out_proj(y) as one GEMM
            op = self.out_proj
            r2 = residual.reshape(-1, residual.shape[-1])
            r2 = r2 if op.bias is None else r2 + op.bias
            out = torch.addmm(r2, y.reshape(-1, y.shape[-1]), op.weight.t()).view(residual.shape)
        return (out, state) if return_state else out

    def forward(self, x):
        """mamba.py:231-267; the bidirectional pair is one fused launch; the
        scan's prologue (softplus, BCNorm, MIMO fold) is one launch forward and
        one backward (_ssm_inputs)."""
        if not torch.is_grad_enabled():
            return self._forward_inference(x, False)
        cfg = self.config
        x_branch, z = self.in_proj(x).chunk(2, dim=-1)
        x_branch = F.silu(x_branch)
        coef = 2.0 if cfg.bidirectional else 1.0
        x_dbl, dt = self._projections(x_branch)
        if _bf16_layer():
            x_branch = x_branch.to(torch.bfloat16)
            y = self._fused_scan(x_branch, x_dbl, dt,
                                 S.M3_DIR_BIDIR if cfg.bidirectional else S.M3_DIR_FWD)
            if y is not None:
                return self.out_proj(self._gated(y, x_branch, z, coef))
        delta, bc, cc = self._ssm_inputs(x_branch, x_dbl, dt)
        yd = None
        if _bf16_layer():   # the kernels' bf16 configuration (autograd casts the grads back)
            bf = torch.bfloat16
            delta, bc, cc, yd = delta.to(bf), bc.to(bf), cc.to(bf), bf
        track = self._track_gate() if cfg.n_track_state > 0 else None
        A_real, A_imag = self._compute_A()
        args = (delta, x_branch, bc, cc, A_real, A_imag, track, cfg.n_rot_state, cfg.d_state)
        if not cfg.bidirectional:
            y = S.m3_trapezoidal_scan(*args, y_dtype=yd)
        else:
            y = S.m3_bidir_scan(*args, y_dtype=yd)
        return self.out_proj(self._gated(y, x_branch, z, coef))

    def _gated(self, y, u, z, coef):
        """(y + coef*u*D) * silu(z) (mamba.py:262-265) with autograd, one launch
        each way (S.gated_output); a bf16 layer gets its output in bf16, the
        type autocast's out_proj casts it to anyway."""
        return S.gated_output(y, u, z, self.D, coef,
                              out_dtype=torch.bfloat16 if _bf16_layer() else None)

    def forward_with_state(self, x):
        """mamba.py:269-282: output and the (h_last, dBu_last) state."""
        if not torch.is_grad_enabled():
            return self._forward_inference(x, True)
        x_branch, z = self.in_proj(x).chunk(2, dim=-1)
        x_branch = F.silu(x_branch)
        y, state = self.ssm(x_branch, return_state=True)
        return self.out_proj(y * F.silu(z)), state

    def _step_inputs(self, x_t):
        x_branch, z = self.in_proj(x_t).chunk(2, dim=-1)
        x_branch = F.silu(x_branch)
        delta, B, C = self._ssm_proj(x_branch)
        return x_branch, z, delta, B.sum(dim=-1), C.sum(dim=-1)

    def step_(self, x_t, state):
        """In-place O(1) step: advances ``state = (h, dBu)`` (float32, contiguous)."""
        cfg = self.config
        u, z, delta, Bc, Cc = self._step_inputs(x_t)
        h, dbu = state
        A_real, A_imag = self._compute_A()
        track = self._track_gate() if cfg.n_track_state > 0 else None
        y = S.m3_step_(h, dbu, delta, u, Bc, Cc, A_real, A_imag, track,
                       cfg.n_rot_state, cfg.d_state)
        y = y + u * self.D
        return self.out_proj(y * F.silu(z)), state

    def step_params(self):
        """Padded (A_real, A_imag, track) of the step kernels, cached until a
        parameter changes (tensor version counters)."""
        cfg = self.config
        srcs = [t for t in (getattr(self, "A_log_mag", None), getattr(self, "A_phase", None),
                            getattr(self, "A_log", None), getattr(self, "track_theta", None))
                if t is not None]
        key = tuple((t.data_ptr(), t._version) for t in srcs)
        cached = getattr(self, "_step_params_cache", None)
        if cached is None or cached[0] != key:
            with torch.no_grad():
                A_real, A_imag = self._compute_A()
                track = self._track_gate() if cfg.n_track_state > 0 else None
                dev = self.D.device
                padded = tuple(t.to(torch.float32).contiguous() for t in S.pad_params(
                    A_real, A_imag, track, cfg.n_rot_state, cfg.d_state, cfg.d_inner, dev))
            cached = (key, padded)
            self._step_params_cache = cached
        return cached[1]

    def step_fused_(self, x_t, state):
        """O(1) step of the fused step layer, in place on ``state``.

        ``state``: (h, dBu) (the reference cache pair) or (h, fac_prev, fac_next)
        (the factored state; swap the factor buffers between steps).  The
        projections are cuBLAS GEMMs; softplus, BCNorm, the MIMO fold, the
        recurrence and the gated output (y + u*D) * silu(z) run in one launch
        (``m3_step_gated_fused_``) for batches up to ``fuse_step_max_batch``
        where its kernel serves the shape, else in two (``m3_step_inputs``,
        ``m3_step_gated_``), with identical results.
        Returns the out_proj input (B, d_inner); the caller applies out_proj
        (mamba.py:497).
        """
        cfg = self.config
        n, p = cfg.d_state, cfg.mimo_p
        xz = self.in_proj(x_t)
        u = self._silu_x(xz)
        x_dbl = self.x_proj(u)
        dt, dt_bias = self._dt(x_dbl)
        bw = self.b_norm.weight if cfg.use_bcnorm else None
        cw = self.c_norm.weight if cfg.use_bcnorm else None
        eps = self.b_norm.eps if cfg.use_bcnorm else 0.0
        if self.fuse_step and x_t.shape[0] <= self.fuse_step_max_batch:
            out = S.m3_step_gated_fused_(state, dt, x_dbl, cfg.dt_rank, cfg.dt_rank + n * p,
                                         bw, cw, eps, p, u, self.step_params(),
                                         cfg.n_rot_state, xz[:, cfg.d_inner:], self.D,
                                         dt_bias=dt_bias)
            if out is not None:
                return out
        delta, bc, cc = S.m3_step_inputs(dt, x_dbl, cfg.dt_rank, cfg.dt_rank + n * p, bw, cw,
                                         eps, n, p, dt_bias=dt_bias)
        return S.m3_step_gated_(state, delta, u, bc, cc, self.step_params(), cfg.n_rot_state,
                                xz[:, cfg.d_inner:], self.D)

    def small_step_ok(self, x):
        """True when ``step_small_`` serves a lockstep batch ``x`` (B, d_model):
        no autograd, fp32 outside autocast, B <= small_step_max_batch, and the
        rows fit the kernels' staging (checked here so that a layer never
        stops half way)."""
        cfg = self.config
        B = x.shape[0]
        if not (self.fuse_step and 0 < B <= min(self.small_step_max_batch, S.SMALL_ROWS)):
            return False
        if torch.is_grad_enabled() or _bf16_layer() or x.dtype != torch.float32:
            return False
        pad = S.small_rows_pad(B)
        return (cfg.d_model % 4 == 0 and cfg.d_inner % 4 == 0 and cfg.dt_rank <= S.SMALL_DT_RANK
                and pad * cfg.d_model <= S.SMALL_STAGE
                and pad * (cfg.d_inner + cfg.dt_rank) <= S.SMALL_STAGE
                and all(w.dtype == torch.float32 and w.is_contiguous() for w in (
                    self.in_proj.weight, self.x_proj.weight, self.dt_proj.weight,
                    self.out_proj.weight)))

    def step_small_(self, x, norm, state):
        """One layer of the lockstep step for a small batch (``small_step_ok``),
        in place on the residual stream ``x`` (B, d_model) float32 contiguous
        and on ``state`` (as ``step_fused_``):

        * RMSNorm + in_proj + silu of the x half (``m3_rows_linear``,
          mamba.py:82-89, 450-452),
        * x_proj (``m3_rows_linear``, mamba.py:454),
        * dt_proj's product, softplus, BCNorm, MIMO fold, recurrence and the
          gated output (``m3_step_gated_fused_proj``, mamba.py:455-497; where
          that kernel does not serve the lane split, ``m3_xdt_proj`` then
          ``m3_step_inputs`` + ``m3_step_gated``),
        * out_proj + the residual add, written back into ``x``
          (``m3_rows_linear``, mamba.py:497, 591-595).

        Same arithmetic as ``step_fused_`` except the projections' summation
        order (their products are not cuBLAS GEMMs here)."""
        cfg = self.config
        d_in, n, p = cfg.d_inner, cfg.d_state, cfg.mimo_p
        # each launch may start while the one before it finishes (programmatic
        # dependent launches; no kernel of the step writes a weight)
        u, z = S.m3_rows_linear(x, self.in_proj.weight, self.in_proj.bias, norm.weight,
                                norm.eps, split=d_in, silu=True, overlap=True)
        x_dbl, _ = S.m3_rows_linear(u, self.x_proj.weight, self.x_proj.bias, overlap=True)
        bw = self.b_norm.weight if cfg.use_bcnorm else None
        cw = self.c_norm.weight if cfg.use_bcnorm else None
        eps = self.b_norm.eps if cfg.use_bcnorm else 0.0
        off_b, off_c = cfg.dt_rank, cfg.dt_rank + n * p
        g = S.m3_step_gated_fused_proj_(state, self.dt_proj.weight, x_dbl, off_b, off_c, bw, cw,
                                        eps, p, u, self.step_params(), cfg.n_rot_state, z,
                                        self.D, dt_bias=self.dt_proj.bias, overlap=True)
        if g is None:   # a lane split the fused kernel does not serve: dt, then two launches
            x_dbl, dt = S.m3_xdt_proj(u, self.x_proj.weight, self.x_proj.bias,
                                      self.dt_proj.weight, overlap=True)
            delta, bc, cc = S.m3_step_inputs(dt, x_dbl, cfg.dt_rank, off_c, bw, cw, eps, n, p,
                                             dt_bias=self.dt_proj.bias)
            g = S.m3_step_gated_(state, delta, u, bc, cc, self.step_params(), cfg.n_rot_state,
                                 z, self.D)
        S.m3_rows_linear(g, self.out_proj.weight, self.out_proj.bias, residual=x, out0=x,
                         overlap=True)
        return x

    def step(self, x_t, state=None):
        """Functional O(1) step (mamba.py:427-498): returns (out, (h, dBu_t))."""
        cfg = self.config
        if state is None:
            h = torch.zeros(x_t.shape[0], cfg.d_inner, cfg.d_state, device=x_t.device)
            state = (h, torch.zeros_like(h))
        else:
            state = tuple(s.detach().to(torch.float32).clone(
                memory_format=torch.contiguous_format) for s in state)
        return self.step_(x_t, state)


def _state_pair(entry):
    """An (h, dBu) cache entry as a tuple (the factored state is not primed in place)."""
    if len(entry) != 2:
        raise ValueError("prime_cache(out=...) takes (h, dBu) cache entries")
    return tuple(entry)


class Mamba(nn.Module):
    """Embedding + Mamba3Block layers + final norm (mamba.py:503-620)."""

    def __init__(self, config: MambaConfig):
        super().__init__()
        self.config = config
        self.grad_checkpoint = getattr(config, "grad_checkpoint", False)
        self.embedding = nn.Embedding(config.vocab_size, config.d_model)
        self.layers = nn.ModuleList([
            nn.ModuleDict({"mixer": Mamba3Block(config), "norm": RMSNorm(config.d_model)})
            for _ in range(config.n_layer)
        ])
        self.norm_f = RMSNorm(config.d_model)
        self.apply(self._init_weights)

    def _init_weights(self, module):
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)
            if module.bias is not None and not getattr(module.bias, "_no_reinit", False):
                nn.init.zeros_(module.bias)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)

    def forward(self, input_ids, input_embeds=None):
        x = input_embeds if input_embeds is not None else self.embedding(input_ids)
        for layer in self.layers:
            mixer, norm = layer["mixer"], layer["norm"]
            if self.grad_checkpoint and self.training and x.requires_grad:
                x = x + torch.utils.checkpoint.checkpoint(
                    lambda inp, m=mixer, nm=norm: m(nm(inp)), x, use_reentrant=False)
            elif not torch.is_grad_enabled():   # out_proj and the residual add in one GEMM
                x = mixer._forward_inference(norm(x), False, residual=x)
            else:
                x = x + mixer(norm(x))
        return self.norm_f(x)

    def init_cache(self, batch_size, device):
        return [None] * len(self.layers)

    def _embed_step(self, token_id, input_embed):
        if input_embed is not None:
            return input_embed
        if token_id.dim() == 2:
            token_id = token_id.squeeze(1)
        return self.embedding(token_id)

    def step(self, token_id=None, cache=None, input_embed=None, apply_final_norm=True):
        """mamba.py:564-601; returns (hidden, new_cache) without touching ``cache``."""
        assert not self.config.bidirectional, "step() requires a causal model"
        x = self._embed_step(token_id, input_embed)
        cache = cache if cache is not None else [None] * len(self.layers)
        new_cache = []
        for i, layer in enumerate(self.layers):
            delta, st = layer["mixer"].step(layer["norm"](x), cache[i])
            x = x + delta
            new_cache.append(st)
        return (self.norm_f(x) if apply_final_norm else x), new_cache

    def step_(self, token_id=None, cache=None, input_embed=None, apply_final_norm=True):
        """In-place variant for lockstep rollouts: advances every (h, dBu) in ``cache``."""
        assert not self.config.bidirectional, "step() requires a causal model"
        x = self._embed_step(token_id, input_embed)
        for i, layer in enumerate(self.layers):
            delta, _ = layer["mixer"].step_(layer["norm"](x), cache[i])
            x = x + delta
        return (self.norm_f(x) if apply_final_norm else x), cache

    def step_fused_(self, token_id=None, cache=None, input_embed=None, apply_final_norm=True):
        """Lockstep step of every layer on the fused step layer, in place on
        ``cache`` (entries (h, dBu) or (h, fac_prev, fac_next)); out_proj and
        the residual add are one GEMM (addmm).  Batches of at most
        ``Mamba3Block.small_step_max_batch`` rows run every layer on the
        small-batch kernels instead (``Mamba3Block.step_small_``: norm,
        projections, step and residual in four launches per layer).  Returns
        (hidden, cache)."""
        assert not self.config.bidirectional, "step() requires a causal model"
        x = self._embed_step(token_id, input_embed)
        if self.layers[0]["mixer"].small_step_ok(x):
            # the small-batch layer updates the residual stream in place
            x = x.clone() if input_embed is not None or not x.is_contiguous() else x
            for i, layer in enumerate(self.layers):
                layer["mixer"].step_small_(x, layer["norm"], cache[i])
            return (self.norm_f(x) if apply_final_norm else x), cache
        for i, layer in enumerate(self.layers):
            mixer, norm = layer["mixer"], layer["norm"]
            g = mixer.step_fused_(norm(x), cache[i])
            op = mixer.out_proj
            x = (torch.addmm(x, g, op.weight.t()) if op.bias is None
                 else torch.addmm(x + op.bias, g, op.weight.t()))
        return (self.norm_f(x) if apply_final_norm else x), cache

    def prime_cache(self, input_ids, out=None):
        """mamba.py:603-620: full scan once, then (final_hidden, cache).

        ``out`` (no-grad only): an existing cache, (h, dBu) per layer, that
        receives the primed state in place (a captured step graph's static
        state); it is also the returned cache."""
        assert not self.config.bidirectional, "prime_cache() requires a causal model"
        if out is not None and torch.is_grad_enabled():
            raise ValueError("prime_cache(out=...) is an inference option (autograd disabled)")
        cur = self.embedding(input_ids)
        cache = []
        for i, layer in enumerate(self.layers):
            if not torch.is_grad_enabled():   # out_proj and the residual add in one GEMM
                cur, state = layer["mixer"]._forward_inference(
                    layer["norm"](cur), True, residual=cur,
                    state_out=None if out is None else _state_pair(out[i]))
            else:
                mixed, state = layer["mixer"].forward_with_state(layer["norm"](cur))
                cur = cur + mixed
            cache.append(state)
        return self.norm_f(cur[:, -1, :]), cache
