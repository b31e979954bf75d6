"""PyTorch operator surface of the sm_100a trapezoidal scan.

Mirrors ``redpanda/engine/triton_scan.py`` so that it is a drop-in for the
reference's fused-scan path:

* ``HAS_M3`` (alias ``HAS_TRITON``) -- availability flag (triton_scan.py:30-37)
* ``m3_trapezoidal_scan`` (alias ``triton_trapezoidal_scan``) -- same
  arguments and result as triton_scan.py:318-337: y WITHOUT the ``u*D`` skip
* ``_TrapezoidalScanFn`` -- the autograd Function (triton_scan.py:244-315),
  analytic backward, grads cast to the input dtypes
* ``m3_bidir_scan`` -- y_fwd + flip(scan(flip(x))) in one launch (mamba.py:254-260)
* ``m3_scan_with_state`` -- the ``return_state`` scan (mamba.py:377-379)
* ``m3_step_`` -- the in-place O(1) step recurrence (mamba.py:466-493)
* ``m3_step_factored_`` -- the same step on the factored (h, [delta*u | B])
  state, half the HBM traffic, bit-identical results
* ``verify`` -- the correctness gate (triton_scan.py:340-398): forward and all
  gradients against a float64 torch recurrence, raising on a mismatch
* ``m3_step_inputs`` / ``m3_step_gated_`` -- the fused step layer: softplus,
  BCNorm and MIMO fold in one launch (mamba.py:455-469), the recurrence with
  the gated output (y + u*D) * silu(z) in another (mamba.py:490-497)

Registering this module as ``triton_scan`` in ``sys.modules`` routes the
unmodified reference ``mamba.py`` (with ``use_triton_scan=True``) through
these kernels.  There is
no CPU or PyTorch fallback: every op raises if the CUDA library is missing or a
tensor is not on an sm_100 device.
"""

import torch
import torch.nn.functional as F

from . import _lib
from ._lib import M3_BF16, M3_DIR_BIDIR, M3_DIR_FWD, M3_DIR_REV, M3_F32, ScanDesc, StepDesc

CHUNK = 16  # checkpoint / backward recompute chunk (timesteps)


def _has_m3():
    if not _lib.available() or not torch.cuda.is_available():
        return False
    try:
        return torch.cuda.get_device_capability()[0] == 10
    except Exception:  # pragma: no cover - driver trouble
        return False


HAS_M3 = _has_m3()
HAS_TRITON = HAS_M3   # name the reference's mamba.py:344 imports


def _dt_code(dtype):
    if dtype == torch.float32:
        return M3_F32
    if dtype == torch.bfloat16:
        return M3_BF16
    raise TypeError(f"unsupported dtype {dtype}")


def _prep_pair(a, b):
    """Contiguous copies of a tensor pair in one kernel dtype (f32 or bf16)."""
    if a.dtype == b.dtype and a.dtype in (torch.float32, torch.bfloat16):
        dt = a.dtype
    else:
        dt = torch.float32
    return a.to(dt).contiguous(), b.to(dt).contiguous(), _dt_code(dt)


def ctypes_ptr(t):
    return None if t is None else t.data_ptr()


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("m3 scan ops run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("m3 scan ops need every tensor on one device")
    return dev


def pad_params(A_real, A_imag, track, n_rot, n_state, d_inner, device):
    """(D, N) fp32 parameter tensors in the layout of triton_scan.py:325-335."""
    if A_real is not None:
        Ar_p = F.pad(A_real, (0, n_state - A_real.shape[-1]))
        Ai_p = (F.pad(A_imag, (0, n_state - A_imag.shape[-1]))
                if A_imag is not None else torch.zeros(d_inner, n_state, device=device))
    else:
        Ar_p = torch.zeros(d_inner, n_state, device=device)
        Ai_p = torch.zeros(d_inner, n_state, device=device)
    Tk_p = (F.pad(track, (n_rot, 0))
            if track is not None else torch.zeros(d_inner, n_state, device=device))
    return Ar_p, Ai_p, Tk_p


class ScanPlan:
    """One scan shape bound to the C ABI; calls write into caller-owned buffers.

    The layer below the autograd Function: no allocation per call, no dtype
    conversion.  ``delta``/``u`` share ``dtype_du``, ``Bc``/``Cc`` share
    ``dtype_bc`` (torch.float32 or torch.bfloat16); parameters are the (D, N)
    fp32 padded tensors of :func:`pad_params`.
    """

    def __init__(self, batch, seqlen, d_inner, d_state, n_rot, dtype_du=torch.float32,
                 dtype_bc=torch.float32, direction=M3_DIR_FWD):
        self.shape = (batch, seqlen, d_inner, d_state)
        self.n_rot = int(n_rot)
        self.dtype_du, self.dtype_bc = dtype_du, dtype_bc
        self.direction = int(direction)
        self.desc = ScanDesc(batch, seqlen, d_inner, d_state, self.n_rot, _dt_code(dtype_du),
                             _dt_code(dtype_bc), self.direction)
        self._lib = _lib.load()

    def ckpt_floats(self):
        return int(self._lib.m3_scan_ckpt_floats(self.desc))

    def workspace_bytes(self):
        return int(self._lib.m3_scan_bwd_workspace_bytes(self.desc))

    def forward(self, delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p, y, ckpt=None, h_last=None,
                dbu_last=None, stream=None):
        """y is float32 or bfloat16 (its element type selects the stored y)."""
        dev = delta.device
        s = _stream(dev) if stream is None else stream
        _lib.check(self._lib.m3_scan_fwd_typed(
            self.desc, delta.data_ptr(), u.data_ptr(), Bc.data_ptr(), Cc.data_ptr(),
            Ar_p.data_ptr(), Ai_p.data_ptr(), Tk_p.data_ptr(), y.data_ptr(), _dt_code(y.dtype),
            ctypes_ptr(ckpt), ctypes_ptr(h_last), ctypes_ptr(dbu_last), s))

    def backward(self, delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p, dy, ckpt, d_delta, d_u, d_Bc,
                 d_Cc, d_Ar, d_Ai, d_Tk, workspace, stream=None):
        dev = delta.device
        s = _stream(dev) if stream is None else stream
        _lib.check(self._lib.m3_scan_bwd(
            self.desc, delta.data_ptr(), u.data_ptr(), Bc.data_ptr(), Cc.data_ptr(),
            Ar_p.data_ptr(), Ai_p.data_ptr(), Tk_p.data_ptr(), dy.data_ptr(),
            _dt_code(dy.dtype), ctypes_ptr(ckpt), d_delta.data_ptr(), d_u.data_ptr(),
            d_Bc.data_ptr(), d_Cc.data_ptr(), d_Ar.data_ptr(), d_Ai.data_ptr(),
            d_Tk.data_ptr(), workspace.data_ptr(), workspace.numel(), s))


class _TrapezoidalScanFn(torch.autograd.Function):
    """y = trapezoidal selective scan; analytic, deterministic backward.

    forward(delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p, n_rot, direction, want_state, y_dtype)
    returns (y, h_last, dbu_last); y is float32 (the reference) or bfloat16 (a
    bf16 layer; state and accumulation stay fp32); the state outputs are empty
    unless ``want_state`` and are not differentiable.
    """

    @staticmethod
    def forward(ctx, delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p, n_rot, direction, want_state,
                y_dtype=torch.float32):
        lib = _lib.load()
        dev = _require_cuda(delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p)
        dl, uu, dt_du = _prep_pair(delta, u)
        bb, cc, dt_bc = _prep_pair(Bc, Cc)
        ar, ai, tk = (x.detach().to(torch.float32).contiguous() for x in (Ar_p, Ai_p, Tk_p))
        B, L, D = uu.shape
        N = bb.shape[-1]
        desc = ScanDesc(B, L, D, N, int(n_rot), dt_du, dt_bc, int(direction))
        y = torch.empty(B, L, D, device=dev, dtype=y_dtype)
        need_grad = any(ctx.needs_input_grad[:7])
        nck = lib.m3_scan_ckpt_floats(desc) if need_grad else 0
        ckpt = torch.empty(nck, device=dev, dtype=torch.float32) if nck else None
        if want_state:
            h = torch.empty(B, D, N, device=dev, dtype=torch.float32)
            dbu = torch.empty_like(h)
        else:
            h = dbu = None
        with torch.cuda.device(dev):
            _lib.check(lib.m3_scan_fwd_typed(desc, dl.data_ptr(), uu.data_ptr(), bb.data_ptr(),
                                             cc.data_ptr(), ar.data_ptr(), ai.data_ptr(),
                                             tk.data_ptr(), y.data_ptr(), _dt_code(y_dtype),
                                             ctypes_ptr(ckpt), ctypes_ptr(h), ctypes_ptr(dbu),
                                             _stream(dev)))
        empty = torch.empty(0, device=dev)
        ctx.save_for_backward(dl, uu, bb, cc, ar, ai, tk, ckpt if ckpt is not None else empty)
        ctx.has_ckpt = ckpt is not None
        ctx.desc = (B, L, D, N, int(n_rot), dt_du, dt_bc, int(direction))
        ctx.in_dtypes = (delta.dtype, u.dtype, Bc.dtype, Cc.dtype,
                         Ar_p.dtype, Ai_p.dtype, Tk_p.dtype)
        if want_state:
            ctx.mark_non_differentiable(h, dbu)
            return y, h, dbu
        return y, empty, empty

    @staticmethod
    def backward(ctx, dy, _dh=None, _ddbu=None):
        lib = _lib.load()
        dl, uu, bb, cc, ar, ai, tk, ckpt = ctx.saved_tensors
        dev = dl.device
        desc = ScanDesc(*ctx.desc)
        if dy.dtype not in (torch.float32, torch.bfloat16):
            dy = dy.float()
        dy = dy.contiguous()
        dd = torch.empty_like(dl)
        du = torch.empty_like(uu)
        dB = torch.empty_like(bb)
        dC = torch.empty_like(cc)
        dAr = torch.empty_like(ar)
        dAi = torch.empty_like(ai)
        dTk = torch.empty_like(tk)
        nws = lib.m3_scan_bwd_workspace_bytes(desc)
        ws = torch.empty(max(nws, 1), device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            _lib.check(lib.m3_scan_bwd(
                desc, dl.data_ptr(), uu.data_ptr(), bb.data_ptr(), cc.data_ptr(),
                ar.data_ptr(), ai.data_ptr(), tk.data_ptr(), dy.data_ptr(), _dt_code(dy.dtype),
                ckpt.data_ptr() if ctx.has_ckpt else None,
                dd.data_ptr(), du.data_ptr(), dB.data_ptr(), dC.data_ptr(),
                dAr.data_ptr(), dAi.data_ptr(), dTk.data_ptr(), ws.data_ptr(), nws,
                _stream(dev)))
        td, tu, tb, tc, tar, tai, ttk = ctx.in_dtypes
        return (dd.to(td), du.to(tu), dB.to(tb), dC.to(tc), dAr.to(tar), dAi.to(tai),
                dTk.to(ttk), None, None, None, None)


class FusedUnsupported(RuntimeError):
    """The fused-prologue kernels cannot stage this shape; run the unfused pair."""


M3_ERR_UNSUPPORTED = 4


class _FusedScanFn(torch.autograd.Function):
    """The scan with the layer's prologue fused in (m3_scan_fwd_fused /
    m3_scan_bwd_fused): y from the raw projections dt (B, L, D) and x_dbl
    (B, L, K) -- softplus, BCNorm and MIMO fold (mamba.py:284-301, 336-337)
    applied as each chunk is staged.  bf16 inputs; equal bit for bit to
    m3_step_inputs + casts to bf16 + the scan, forward and backward.

    forward(dt, x_dbl, b_weight, c_weight, u, Ar_p, Ai_p, Tk_p, cfg) with
    cfg = (n_rot, n_state, mimo_p, off_b, off_c, eps, direction, y_dtype, want_ckpt).
    """

    @staticmethod
    def forward(ctx, dt, x_dbl, wb, wc, u, Ar_p, Ai_p, Tk_p, cfg):
        n_rot, N, P, off_b, off_c, eps, direction, y_dtype, want_ckpt = cfg
        lib = _lib.load()
        dev = _require_cuda(dt, x_dbl, u, Ar_p, Ai_p, Tk_p)
        if not (dt.dtype == x_dbl.dtype == u.dtype == torch.bfloat16):
            raise FusedUnsupported("the fused prologue takes bf16 dt, x_dbl and u")
        dt, x_dbl, u = dt.contiguous(), x_dbl.contiguous(), u.contiguous()
        ar, ai, tk = (x.detach().to(torch.float32).contiguous() for x in (Ar_p, Ai_p, Tk_p))
        w32 = [None if w is None else w.detach().to(torch.float32).contiguous() for w in (wb, wc)]
        B, L, D = u.shape
        desc = ScanDesc(B, L, D, N, int(n_rot), M3_BF16, M3_BF16, int(direction))
        y = torch.empty(B, L, D, device=dev, dtype=y_dtype)
        nck = lib.m3_scan_ckpt_floats(desc) if want_ckpt else 0
        ckpt = torch.empty(nck, device=dev) if nck else None
        with torch.cuda.device(dev):
            rc = lib.m3_scan_fwd_fused(desc, int(P), dt.data_ptr(), x_dbl.data_ptr(),
                                       x_dbl.shape[-1], int(off_b), int(off_c),
                                       ctypes_ptr(w32[0]), ctypes_ptr(w32[1]), float(eps),
                                       u.data_ptr(), ar.data_ptr(), ai.data_ptr(), tk.data_ptr(),
                                       y.data_ptr(), _dt_code(y_dtype), ctypes_ptr(ckpt),
                                       _stream(dev))
        if rc == M3_ERR_UNSUPPORTED:
            raise FusedUnsupported(_lib.strerror(rc))
        _lib.check(rc)
        empty = torch.empty(0, device=dev)
        ctx.save_for_backward(dt, x_dbl, u, ar, ai, tk, ckpt if ckpt is not None else empty,
                              *(w if w is not None else empty for w in w32))
        ctx.cfg = cfg
        ctx.has = (ckpt is not None, w32[0] is not None)
        ctx.w_dtypes = (None if wb is None else wb.dtype, None if wc is None else wc.dtype)
        ctx.p_dtypes = (Ar_p.dtype, Ai_p.dtype, Tk_p.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        dt, x_dbl, u, ar, ai, tk, ckpt, wb, wc = ctx.saved_tensors
        n_rot, N, P, off_b, off_c, eps, direction, _, _ = ctx.cfg
        has_ck, has_w = ctx.has
        dev = dt.device
        B, L, D = u.shape
        desc = ScanDesc(B, L, D, N, int(n_rot), M3_BF16, M3_BF16, int(direction))
        if dy.dtype not in (torch.float32, torch.bfloat16):
            dy = dy.float()
        dy = dy.contiguous()
        d_dt, d_u = torch.empty_like(dt), torch.empty_like(u)
        d_x = torch.zeros_like(x_dbl)
        d_wb = torch.empty_like(wb) if has_w else None
        d_wc = torch.empty_like(wc) if has_w else None
        dAr, dAi, dTk = torch.empty_like(ar), torch.empty_like(ai), torch.empty_like(tk)
        nws = lib.m3_scan_bwd_fused_workspace_bytes(desc, int(P))
        ws = torch.empty(max(nws, 1), device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            _lib.check(lib.m3_scan_bwd_fused(
                desc, int(P), dt.data_ptr(), x_dbl.data_ptr(), x_dbl.shape[-1], int(off_b),
                int(off_c), ctypes_ptr(wb if has_w else None), ctypes_ptr(wc if has_w else None),
                float(eps), u.data_ptr(), ar.data_ptr(), ai.data_ptr(), tk.data_ptr(),
                dy.data_ptr(), _dt_code(dy.dtype), ckpt.data_ptr() if has_ck else None,
                d_dt.data_ptr(), d_u.data_ptr(), d_x.data_ptr(), ctypes_ptr(d_wb),
                ctypes_ptr(d_wc), dAr.data_ptr(), dAi.data_ptr(), dTk.data_ptr(),
                ws.data_ptr(), nws, _stream(dev)))
        wdt = ctx.w_dtypes
        ta, ti, tt = ctx.p_dtypes
        return (d_dt, d_x, None if d_wb is None else d_wb.to(wdt[0]),
                None if d_wc is None else d_wc.to(wdt[1]), d_u, dAr.to(ta), dAi.to(ti),
                dTk.to(tt), None)


def m3_fused_scan(dt, x_dbl, b_weight, c_weight, eps, u, A_real, A_imag, track, n_rot, n_state,
                  mimo_p, off_b, off_c, direction=M3_DIR_FWD, y_dtype=torch.bfloat16):
    """y (without the u*D skip) of the scan whose prologue -- softplus(dt),
    BCNorm of B_raw / C_raw (columns off_b / off_c of x_dbl, N*p each) and the
    MIMO fold -- is fused into its staging; differentiable w.r.t. dt, x_dbl, the
    BCNorm weights, u and the eigenvalues.  Raises FusedUnsupported when the
    kernels cannot stage the shape."""
    Ar_p, Ai_p, Tk_p = pad_params(A_real, A_imag, track, n_rot, n_state, u.shape[-1], u.device)
    # checkpoints only when a backward can follow
    want = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad
        for t in (dt, x_dbl, b_weight, c_weight, u, Ar_p, Ai_p, Tk_p))
    cfg = (int(n_rot), int(n_state), int(mimo_p), int(off_b), int(off_c), float(eps),
           int(direction), y_dtype, bool(want))
    return _FusedScanFn.apply(dt, x_dbl, b_weight, c_weight, u, Ar_p, Ai_p, Tk_p, cfg)


def _scan_nograd(delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p, n_rot, direction, want_state,
                 y_dtype=torch.float32, state_out=None):
    """Forward only (no autograd record, no checkpoints): the inference path.

    ``state_out``: (h, dbu) float32 contiguous (B, D, N) tensors that receive
    the final state instead of new ones (a captured step graph's static cache).
    """
    lib = _lib.load()
    dev = _require_cuda(delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p)
    dl, uu, dt_du = _prep_pair(delta, u)
    bb, cc, dt_bc = _prep_pair(Bc, Cc)
    ar, ai, tk = (x.detach().to(torch.float32).contiguous() for x in (Ar_p, Ai_p, Tk_p))
    B, L, D = uu.shape
    N = bb.shape[-1]
    desc = ScanDesc(B, L, D, N, int(n_rot), dt_du, dt_bc, int(direction))
    y = torch.empty(B, L, D, device=dev, dtype=y_dtype)
    empty = torch.empty(0, device=dev)
    h = dbu = None
    if want_state and state_out is not None:
        h, dbu = state_out
        for t in (h, dbu):
            if (t.shape != (B, D, N) or t.dtype != torch.float32 or not t.is_contiguous()
                    or t.device != dev):
                raise ValueError("state_out: (B, D, N) contiguous float32 tensors on the "
                                 "scan's device")
    elif want_state:
        h = torch.empty(B, D, N, device=dev, dtype=torch.float32)
        dbu = torch.empty_like(h)
    with torch.cuda.device(dev):
        _lib.check(lib.m3_scan_fwd_typed(desc, dl.data_ptr(), uu.data_ptr(), bb.data_ptr(),
                                         cc.data_ptr(), ar.data_ptr(), ai.data_ptr(),
                                         tk.data_ptr(), y.data_ptr(), _dt_code(y_dtype), None,
                                         ctypes_ptr(h), ctypes_ptr(dbu), _stream(dev)))
    return (y, h, dbu) if want_state else (y, empty, empty)


def _apply(delta, u, Bc, Cc, A_real, A_imag, track, n_rot, n_state, direction, want_state,
           y_dtype=None, state_out=None):
    d_inner = u.shape[-1]
    y_dtype = torch.float32 if y_dtype is None else y_dtype
    if y_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"y_dtype must be float32 or bfloat16, not {y_dtype}")
    Ar_p, Ai_p, Tk_p = pad_params(A_real, A_imag, track, n_rot, n_state, d_inner, u.device)
    if not torch.is_grad_enabled():
        return _scan_nograd(delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p, n_rot, direction, want_state,
                            y_dtype, state_out)
    if state_out is not None:
        raise ValueError("state_out is an inference option (autograd disabled)")
    return _TrapezoidalScanFn.apply(delta, u, Bc, Cc, Ar_p, Ai_p, Tk_p,
                                    n_rot, direction, want_state, y_dtype)


def m3_trapezoidal_scan(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                        n_rot, n_state, *, y_dtype=None):
    """Causal scan; drop-in for ``triton_trapezoidal_scan`` (triton_scan.py:318-337).

    Returns y (B, L, D) without the ``u*D`` skip term: float32 as the
    reference, or bfloat16 with ``y_dtype=torch.bfloat16`` (a bf16 layer; the
    state and every accumulation stay fp32).
    """
    return _apply(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                  n_rot, n_state, M3_DIR_FWD, False, y_dtype)[0]


triton_trapezoidal_scan = m3_trapezoidal_scan


def m3_reverse_scan(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                    n_rot, n_state, *, y_dtype=None):
    """flip(scan(flip(x))) without materialising flipped copies."""
    return _apply(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                  n_rot, n_state, M3_DIR_REV, False, y_dtype)[0]


def m3_bidir_scan(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                  n_rot, n_state, *, y_dtype=None):
    """Fused bidirectional scan: scan(x) + flip(scan(flip(x))) (mamba.py:254-260).

    Skip terms excluded; the reference block adds ``u*D`` once per direction.
    """
    return _apply(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                  n_rot, n_state, M3_DIR_BIDIR, False, y_dtype)[0]


def m3_scan_with_state(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                       n_rot, n_state, state_out=None):
    """Causal scan returning ``(y, (h_last, dBu_last))`` (mamba.py:377-379).

    y is differentiable; the state is not.  ``state_out`` (inference only):
    existing (h, dBu) tensors to write the state into.
    """
    y, h, dbu = _apply(delta, u, B_contracted, C_contracted, A_real, A_imag, track,
                       n_rot, n_state, M3_DIR_FWD, True, state_out=state_out)
    return y, (h, dbu)


def m3_step_(h, dbu, delta_t, u_t, Bc_t, Cc_t, A_real, A_imag, track, n_rot, n_state):
    """O(1) step of B rows, updating ``h`` and ``dbu`` IN PLACE; returns y (B, D).

    h, dbu: (B, D, N) contiguous float32 CUDA tensors (the reference cache
    pair, mamba.py:487-498).  delta_t, u_t: (B, D); Bc_t, Cc_t: (B, N).
    The reference step is functional (mamba.py:489-498); callers that keep the
    old state must clone it first (as mars_search.py:640 does).
    """
    lib = _lib.load()
    dev = _require_cuda(h, dbu, delta_t, u_t, Bc_t, Cc_t)
    if h.dtype != torch.float32 or dbu.dtype != torch.float32:
        raise TypeError("m3_step_: the state must be float32")
    if not (h.is_contiguous() and dbu.is_contiguous()):
        raise ValueError("m3_step_: the state must be contiguous (it is updated in place)")
    B, D, N = h.shape
    dl, uu, dt_du = _prep_pair(delta_t, u_t)
    bb, cc, dt_bc = _prep_pair(Bc_t, Cc_t)
    Ar_p, Ai_p, Tk_p = pad_params(A_real, A_imag, track, n_rot, n_state, D, dev)
    ar, ai, tk = (x.detach().to(torch.float32).contiguous() for x in (Ar_p, Ai_p, Tk_p))
    y = torch.empty(B, D, device=dev, dtype=torch.float32)
    desc = StepDesc(B, D, N, int(n_rot), dt_du, dt_bc)
    with torch.cuda.device(dev):
        _lib.check(lib.m3_step(desc, h.data_ptr(), dbu.data_ptr(), dl.data_ptr(),
                               uu.data_ptr(), bb.data_ptr(), cc.data_ptr(), ar.data_ptr(),
                               ai.data_ptr(), tk.data_ptr(), y.data_ptr(), _stream(dev)))
    return y


def factored_state(delta, u, Bc):
    """Factors [delta*u | B] of the last token of a (B, L, .) sequence, (B, D + N) fp32.

    Together with the scan's ``h_last`` this is the factored step state; the
    product is the scan's own fp32 rounding of delta*u.
    """
    return torch.cat([delta[:, -1].float() * u[:, -1].float(), Bc[:, -1].float()], dim=-1)


def m3_step_factored_(h, fac_prev, fac_next, delta_t, u_t, Bc_t, Cc_t, A_real, A_imag, track,
                      n_rot, n_state):
    """O(1) step on the factored state: h (B, D, N) in place, factors
    fac_prev -> fac_next (B, D + N), returns y (B, D).  Equals :func:`m3_step_`
    bit for bit with half its HBM traffic."""
    lib = _lib.load()
    dev = _require_cuda(h, fac_prev, fac_next, delta_t, u_t, Bc_t, Cc_t)
    if h.dtype != torch.float32 or fac_prev.dtype != torch.float32 or \
            fac_next.dtype != torch.float32:
        raise TypeError("m3_step_factored_: the state must be float32")
    if not (h.is_contiguous() and fac_prev.is_contiguous() and fac_next.is_contiguous()):
        raise ValueError("m3_step_factored_: the state must be contiguous")
    B, D, N = h.shape
    dl, uu, dt_du = _prep_pair(delta_t, u_t)
    bb, cc, dt_bc = _prep_pair(Bc_t, Cc_t)
    Ar_p, Ai_p, Tk_p = pad_params(A_real, A_imag, track, n_rot, n_state, D, dev)
    ar, ai, tk = (x.detach().to(torch.float32).contiguous() for x in (Ar_p, Ai_p, Tk_p))
    y = torch.empty(B, D, device=dev, dtype=torch.float32)
    desc = StepDesc(B, D, N, int(n_rot), dt_du, dt_bc)
    with torch.cuda.device(dev):
        _lib.check(lib.m3_step_factored(desc, h.data_ptr(), fac_prev.data_ptr(),
                                        fac_next.data_ptr(), dl.data_ptr(), uu.data_ptr(),
                                        bb.data_ptr(), cc.data_ptr(), ar.data_ptr(),
                                        ai.data_ptr(), tk.data_ptr(), y.data_ptr(), _stream(dev)))
    return y


def _f32_or_bf16(t):
    """t as float32 or bfloat16 (the element types the prologue kernels read)."""
    return t if t.dtype in (torch.float32, torch.bfloat16) else t.float()


def m3_step_inputs(dt, x_dbl, off_b, off_c, b_weight, c_weight, eps, n_state, mimo_p,
                   dt_bias=None):
    """softplus(dt) and the BCNorm'ed, MIMO-folded B and C of one token, one launch.

    dt: (B, D) float32 or bfloat16, dt_proj output with its bias, or without it
    when ``dt_bias`` (D,) is given (added first, one fp32 rounding, as torch's
    matmul followed by the bias add); x_dbl: (B, K) float32 or bfloat16 rows
    of x_proj's output, B_raw at column ``off_b`` and C_raw at ``off_c``
    (N*p columns each); b_weight / c_weight: BCNorm weights (N*p,) or None
    (use_bcnorm=False).  Returns (delta (B, D) in dt's element type, Bc, Cc
    (B, N) in x_dbl's): mamba.py:455-469 and 336-337 for one token.  The
    arithmetic is fp32 (as torch autocast runs softplus and the RMSNorm,
    train.py:268); a bf16 output is that result rounded once, the bits a bf16
    layer's cast gives.
    """
    lib = _lib.load()
    dev = _require_cuda(dt, x_dbl)
    dt, x_dbl = _f32_or_bf16(dt), _f32_or_bf16(x_dbl)
    if dt.stride(-1) != 1 or x_dbl.stride(-1) != 1:
        raise ValueError("m3_step_inputs: rows of dt and x_dbl must be contiguous")
    B, D = dt.shape
    wb = wc = None
    if b_weight is not None:
        wb = b_weight.detach().to(torch.float32).contiguous()
        wc = c_weight.detach().to(torch.float32).contiguous()
    bias = None if dt_bias is None else dt_bias.detach().to(torch.float32).contiguous()
    delta = torch.empty(B, D, device=dev, dtype=dt.dtype)
    bc = torch.empty(B, n_state, device=dev, dtype=x_dbl.dtype)
    cc = torch.empty_like(bc)
    desc = StepDesc(B, D, n_state, 0, _dt_code(dt.dtype), _dt_code(x_dbl.dtype))
    with torch.cuda.device(dev):
        _lib.check(lib.m3_step_inputs(desc, int(mimo_p), dt.data_ptr(), dt.stride(0),
                                      ctypes_ptr(bias), x_dbl.data_ptr(), x_dbl.stride(0),
                                      int(off_b), int(off_c),
                                      ctypes_ptr(wb), ctypes_ptr(wc), float(eps),
                                      delta.data_ptr(), bc.data_ptr(), cc.data_ptr(),
                                      _stream(dev)))
    return delta, bc, cc


class _StepInputsFn(torch.autograd.Function):
    """softplus(dt) and the BCNorm'ed, MIMO-folded B and C over rows, with the
    analytic backward (m3_step_inputs / m3_step_inputs_bwd): the training-path
    prologue of the scan (mamba.py:284-301, 336-337)."""

    @staticmethod
    def forward(ctx, dt, x_dbl, b_weight, c_weight, off_b, off_c, eps, n_state, mimo_p):
        delta, bc, cc = m3_step_inputs(dt, x_dbl, off_b, off_c, b_weight, c_weight, eps,
                                       n_state, mimo_p)
        ctx.save_for_backward(dt, x_dbl, b_weight if b_weight is not None else dt.new_empty(0),
                              c_weight if c_weight is not None else dt.new_empty(0))
        ctx.cfg = (off_b, off_c, float(eps), int(n_state), int(mimo_p), b_weight is not None)
        return delta, bc, cc

    @staticmethod
    def backward(ctx, g_delta, g_bc, g_cc):
        dt, x_dbl, wb, wc = ctx.saved_tensors
        off_b, off_c, eps, n, p, has_w = ctx.cfg
        lib = _lib.load()
        dev = dt.device
        rows, D = dt.shape
        def z(g, shape, dtype):   # an upstream gradient in the element type of its input
            if g is None:
                return torch.zeros(shape, device=dev, dtype=dtype)
            return g.to(dtype).contiguous()
        g_delta = z(g_delta, (rows, D), dt.dtype)
        g_bc, g_cc = z(g_bc, (rows, n), x_dbl.dtype), z(g_cc, (rows, n), x_dbl.dtype)
        d_dt = torch.empty(rows, D, device=dev, dtype=dt.dtype)
        d_x = torch.zeros_like(x_dbl)
        desc = StepDesc(rows, D, n, 0, _dt_code(dt.dtype), _dt_code(x_dbl.dtype))
        d_wb = d_wc = ws = None
        if has_w:
            wb32, wc32 = wb.detach().float().contiguous(), wc.detach().float().contiguous()
            d_wb, d_wc = torch.empty_like(wb32), torch.empty_like(wc32)
            ws = torch.empty(max(1, lib.m3_step_inputs_bwd_workspace_bytes(desc, p)),
                             device=dev, dtype=torch.uint8)
        else:
            wb32 = wc32 = None
        with torch.cuda.device(dev):
            _lib.check(lib.m3_step_inputs_bwd(
                desc, p, dt.data_ptr(), dt.stride(0), x_dbl.data_ptr(), x_dbl.stride(0), off_b,
                off_c, ctypes_ptr(wb32), ctypes_ptr(wc32), eps, g_delta.data_ptr(),
                g_bc.data_ptr(), g_cc.data_ptr(), d_dt.data_ptr(), d_x.data_ptr(),
                ctypes_ptr(d_wb), ctypes_ptr(d_wc), ctypes_ptr(ws),
                0 if ws is None else ws.numel(), _stream(dev)))
        return (d_dt, d_x, None if d_wb is None else d_wb.to(wb.dtype),
                None if d_wc is None else d_wc.to(wc.dtype), None, None, None, None, None)


def step_inputs(dt, x_dbl, off_b, off_c, b_weight, c_weight, eps, n_state, mimo_p):
    """Differentiable :func:`m3_step_inputs` over (rows, .) float32 or bfloat16
    tensors (a bf16 layer's projections stay bf16: the kernels read them and
    write bf16 delta, Bc, Cc and gradients, each rounded once)."""
    dt = _f32_or_bf16(dt).contiguous()
    x_dbl = _f32_or_bf16(x_dbl).contiguous()
    return _StepInputsFn.apply(dt, x_dbl, b_weight, c_weight, off_b, off_c, eps, n_state,
                               mimo_p)


def m3_gate(y, u, z, d_skip, coef=1.0, out=None, out_dtype=None, round_silu=False):
    """(y + coef*u*D) * silu(z) in one launch (mamba.py:262-265).

    y, u: (..., D) contiguous, float32 or bfloat16; z: (..., D) float32 or
    bfloat16 with contiguous rows (a view of in_proj's output); arithmetic in
    fp32.  ``out`` (or a new tensor of ``out_dtype``, default y's dtype) may be
    ``y`` itself."""
    lib = _lib.load()
    dev = _require_cuda(y, u, z, d_skip)
    D = y.shape[-1]
    rows = y.numel() // D
    if not (y.is_contiguous() and u.is_contiguous()) or z.stride(-1) != 1:
        raise ValueError("m3_gate: y and u must be contiguous, z row-contiguous")
    zz = z.reshape(rows, D) if z.dim() > 2 else z
    if zz.stride(-1) != 1:
        raise ValueError("m3_gate: z rows must be contiguous")
    if out is None:
        out = torch.empty(y.shape, device=dev, dtype=y.dtype if out_dtype is None else out_dtype)
    ds = d_skip.detach().to(torch.float32).contiguous()
    with torch.cuda.device(dev):
        _lib.check(lib.m3_gate_typed(rows, D, y.data_ptr(), _dt_code(y.dtype), u.data_ptr(),
                                     _dt_code(u.dtype), zz.data_ptr(), _dt_code(zz.dtype),
                                     zz.stride(0), ds.data_ptr(), float(coef), int(round_silu),
                                     out.data_ptr(), _dt_code(out.dtype), _stream(dev)))
    return out


class _GateFn(torch.autograd.Function):
    """out = (y + coef*u*D) * silu(z) (mamba.py:262-265, 496-497) with its
    backward in one launch (m3_gate / m3_gate_bwd) instead of five elementwise
    ops forward and about eight backward.  silu(z) of a bf16 z is rounded to
    bf16 as F.silu does, so the forward equals torch's formula bit for bit;
    the gradients are computed in fp32 and rounded once (torch rounds some
    intermediates to bf16, so they agree to bf16 rounding)."""

    @staticmethod
    def forward(ctx, y, u, z, d_skip, coef, out_dtype):
        y, u = y.contiguous(), u.contiguous()
        out = m3_gate(y, u, z, d_skip, coef, out_dtype=out_dtype, round_silu=True)
        ctx.save_for_backward(y, u, z, d_skip)
        ctx.coef = float(coef)
        return out

    @staticmethod
    def backward(ctx, g):
        y, u, z, d_skip = ctx.saved_tensors
        lib = _lib.load()
        dev = y.device
        D = y.shape[-1]
        rows = y.numel() // D
        zz = z.reshape(rows, D) if z.dim() > 2 else z
        g = g.contiguous()
        if g.dtype not in (torch.float32, torch.bfloat16):
            g = g.float()
        ds = d_skip.detach().to(torch.float32).contiguous()
        dy = torch.empty_like(y)
        du = torch.empty_like(u)
        dz = torch.empty(z.shape, device=dev, dtype=z.dtype)
        dds = torch.empty(D, device=dev, dtype=torch.float32)
        nws = lib.m3_gate_bwd_workspace_bytes(rows, D)
        ws = torch.empty(max(1, nws), device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            _lib.check(lib.m3_gate_bwd(rows, D, y.data_ptr(), _dt_code(y.dtype), u.data_ptr(),
                                       _dt_code(u.dtype), zz.data_ptr(), _dt_code(zz.dtype),
                                       zz.stride(0), ds.data_ptr(), ctx.coef, 1, g.data_ptr(),
                                       _dt_code(g.dtype), dy.data_ptr(), du.data_ptr(),
                                       dz.data_ptr(), dds.data_ptr(), ws.data_ptr(), nws,
                                       _stream(dev)))
        return dy, du, dz, dds.to(d_skip.dtype), None, None


def gated_output(y, u, z, d_skip, coef=1.0, out_dtype=None):
    """Differentiable (y + coef*u*d_skip) * silu(z) (mamba.py:262-265) on the
    kernels; ``out_dtype`` defaults to torch's promotion of the operands."""
    if out_dtype is None:
        out_dtype = torch.promote_types(torch.promote_types(y.dtype, u.dtype),
                                        torch.promote_types(z.dtype, d_skip.dtype))
    return _GateFn.apply(y, u, z, d_skip, coef, out_dtype)


def m3_step_gated_(state, delta_t, u_t, Bc_t, Cc_t, params, n_rot, z, d_skip):
    """In-place O(1) step whose output is the layer's gated activation
    (y + u*D) * silu(z) (mamba.py:490-497), (B, D) float32.

    ``state`` is (h, dbu) (the reference cache pair) or (h, fac_prev, fac_next)
    (the factored state; the caller swaps the two factor buffers between steps).
    ``params`` are the padded (A_real, A_imag, track) of :func:`pad_params`,
    float32 and contiguous; ``z`` (B, D) may be a row-strided view.
    """
    lib = _lib.load()
    h = state[0]
    dev = _require_cuda(h, delta_t, u_t, Bc_t, Cc_t, z, d_skip)
    B, D, N = h.shape
    if z.dtype != torch.float32:   # a bf16 layer's in_proj output (the step computes in fp32)
        z = z.float()
    if z.stride(-1) != 1:
        raise ValueError("m3_step_gated_: rows of z must be contiguous")
    dl, uu, dt_du = _prep_pair(delta_t, u_t)
    bb, cc, dt_bc = _prep_pair(Bc_t, Cc_t)
    ar, ai, tk = params
    ds = d_skip.detach().to(torch.float32).contiguous()
    out = torch.empty(B, D, device=dev, dtype=torch.float32)
    desc = StepDesc(B, D, N, int(n_rot), dt_du, dt_bc)
    if len(state) == 2:
        dbu, fa, fb = state[1], None, None
    else:
        dbu, fa, fb = None, state[1], state[2]
    with torch.cuda.device(dev):
        _lib.check(lib.m3_step_gated(desc, h.data_ptr(), ctypes_ptr(dbu), ctypes_ptr(fa),
                                     ctypes_ptr(fb), dl.data_ptr(), uu.data_ptr(),
                                     bb.data_ptr(), cc.data_ptr(), ar.data_ptr(), ai.data_ptr(),
                                     tk.data_ptr(), z.data_ptr(), z.stride(0), ds.data_ptr(),
                                     out.data_ptr(), _stream(dev)))
    return out


def m3_silu(x):
    """silu(x) = x / (1 + exp(-x)) over the rows of a (rows, D) float32 view
    whose rows may be strided (the x half of in_proj's output, mamba.py:243,
    452); returns a contiguous (rows, D) float32 tensor.  Same rounding as
    torch's silu: x / (1 + exp(-x)) evaluated in fp32."""
    lib = _lib.load()
    dev = _require_cuda(x)
    if x.dtype != torch.float32 or x.dim() != 2 or x.stride(-1) != 1:
        raise ValueError("m3_silu: a (rows, D) float32 view with contiguous rows")
    rows, D = x.shape
    out = torch.empty(rows, D, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib.check(lib.m3_silu(rows, D, x.data_ptr(), x.stride(0), out.data_ptr(), _stream(dev)))
    return out


SMALL_ROWS = 8          # row limit of the small-batch projection kernels
SMALL_STAGE = 12288     # staged input floats per CTA of those kernels (rows padded to 1/2/4/8)
SMALL_DT_RANK = 64      # dt_rank limit of the small-batch dt product


def small_rows_pad(rows):
    """Rows as the small-batch kernels stage them (1, 2, 4 or 8)."""
    return 1 if rows <= 1 else 2 if rows <= 2 else 4 if rows <= 4 else 8


def _f32_rows(t, name):
    if t.dtype != torch.float32 or t.dim() != 2 or t.stride(-1) != 1:
        raise ValueError(f"{name}: a (rows, n) float32 view with contiguous rows")
    return t


def m3_rows_linear(x, weight, bias=None, norm_weight=None, eps=0.0, residual=None,
                   split=None, silu=False, out0=None, out1=None, overlap=False):
    """Small-batch projection ``act(residual + (bias + norm(x) @ weight.T))``
    in one launch (at most :data:`SMALL_ROWS` rows, fp32).

    ``norm_weight``: apply the RMSNorm x * rsqrt(mean(x^2) + eps) * w first
    (mamba.py:82-89).  Columns ``[0, split)`` are returned in ``out0`` (silu
    applied when ``silu``: the x half of in_proj, mamba.py:450-452) and
    ``[split, d_out)`` in ``out1`` (the z half); ``split`` defaults to d_out.
    ``residual`` (rows, d_out) is added last (mamba.py:595) and may be passed as
    ``out0`` to update it in place.  Returns (out0, out1) -- ``out1`` is None
    when split == d_out -- or None when the shape is past the kernel's limits
    (nothing launched).  ``overlap``: launch as a programmatic dependent launch
    that starts while the previous kernel on the stream finishes and reads the
    first part of ``weight`` before that kernel completes (only when no queued
    kernel writes the weight)."""
    lib = _lib.load()
    dev = _require_cuda(x, weight)
    _f32_rows(x, "m3_rows_linear")
    rows, d_in = x.shape
    d_out = weight.shape[0]
    if weight.dtype != torch.float32 or not weight.is_contiguous() or weight.shape[1] != d_in:
        return None
    split = d_out if split is None else int(split)
    if out0 is None and split > 0:
        out0 = torch.empty(rows, split, device=dev, dtype=torch.float32)
    if out1 is None and split < d_out:
        out1 = torch.empty(rows, d_out - split, device=dev, dtype=torch.float32)
    for t, nm in ((out0, "out0"), (out1, "out1"), (residual, "residual")):
        if t is not None:
            _f32_rows(t, "m3_rows_linear " + nm)
    nw = None if norm_weight is None else norm_weight.detach().to(torch.float32).contiguous()
    b = None if bias is None else bias.detach().to(torch.float32).contiguous()
    with torch.cuda.device(dev):
        rc = lib.m3_rows_linear(rows, d_in, d_out, x.data_ptr(), x.stride(0), ctypes_ptr(nw),
                                float(eps), weight.data_ptr(), ctypes_ptr(b), ctypes_ptr(residual),
                                0 if residual is None else residual.stride(0), split, int(bool(silu)),
                                ctypes_ptr(out0), 0 if out0 is None else out0.stride(0),
                                ctypes_ptr(out1), 0 if out1 is None else out1.stride(0),
                                int(bool(overlap)), _stream(dev))
    if rc == M3_ERR_UNSUPPORTED:
        return None
    _lib.check(rc)
    return out0, out1


def m3_xdt_proj(u, w_x, b_x, w_dt, overlap=False):
    """Small-batch ``x_dbl = u @ w_x.T + b_x`` (mamba.py:454) and
    ``dt = x_dbl[:, :dt_rank] @ w_dt.T`` (dt_proj without its bias,
    mamba.py:463) in one launch; ``dt_rank`` = w_dt.shape[1].  Returns
    (x_dbl, dt), or None when the shape is past the kernel's limits."""
    lib = _lib.load()
    dev = _require_cuda(u, w_x, w_dt)
    _f32_rows(u, "m3_xdt_proj")
    if not u.is_contiguous():
        u = u.contiguous()
    rows, d = u.shape
    n_x, r = w_x.shape[0], w_dt.shape[1]
    for w in (w_x, w_dt):
        if w.dtype != torch.float32 or not w.is_contiguous():
            return None
    if w_x.shape[1] != d or w_dt.shape[0] != d:
        raise ValueError("m3_xdt_proj: weight shapes do not match u")
    b = None if b_x is None else b_x.detach().to(torch.float32).contiguous()
    x_dbl = torch.empty(rows, n_x, device=dev, dtype=torch.float32)
    dt = torch.empty(rows, d, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        rc = lib.m3_xdt_proj(rows, d, n_x, r, u.data_ptr(), w_x.data_ptr(), ctypes_ptr(b),
                             w_dt.data_ptr(), x_dbl.data_ptr(), dt.data_ptr(), int(bool(overlap)),
                             _stream(dev))
    if rc == M3_ERR_UNSUPPORTED:
        return None
    _lib.check(rc)
    return x_dbl, dt


def m3_step_gated_fused_(state, dt, x_dbl, off_b, off_c, b_weight, c_weight, eps, mimo_p,
                         u_t, params, n_rot, z, d_skip, dt_bias=None):
    """:func:`m3_step_inputs` + :func:`m3_step_gated_` in ONE launch
    (mamba.py:455-497): the step kernel computes delta = softplus(dt) and the
    BCNorm'ed, MIMO-folded Bc/Cc of each row from the raw projections itself,
    with the same arithmetic, so state and output are bit-identical to the two
    launches.  ``dt`` (B, D) and ``x_dbl`` (B, ld) float32 rows (x_dbl may be
    the full x_proj output, B_raw / C_raw at columns off_b / off_c); ``dt_bias``
    as for :func:`m3_step_inputs`.

    Returns the gated output (B, D) float32, or None when the fused kernel does
    not serve this shape or layout (nothing launched; the caller runs the two
    launches)."""
    if dt.dtype != torch.float32 or dt.stride(-1) != 1:
        return None
    return _step_gated_fused(state, dt, None, x_dbl, off_b, off_c, b_weight, c_weight, eps,
                             mimo_p, u_t, params, n_rot, z, d_skip, dt_bias)


def m3_step_gated_fused_proj_(state, w_dt, x_dbl, off_b, off_c, b_weight, c_weight, eps,
                              mimo_p, u_t, params, n_rot, z, d_skip, dt_bias=None,
                              overlap=False):
    """:func:`m3_step_gated_fused_` with dt_proj's product formed in the step
    kernel as well (mamba.py:463): dt = x_dbl[:, :r] @ w_dt.T, r =
    w_dt.shape[1] <= 64, then softplus(dt + dt_bias).  The step after x_proj in
    one launch; the dt sum's order is the kernel's own (4 strided partials,
    then pairs).  Returns the gated output, or None when the kernel does not
    serve the shape (nothing launched).  ``overlap``: a programmatic dependent
    launch (see :func:`m3_rows_linear`; this kernel reads nothing before the
    previous kernel completes)."""
    if w_dt.dtype != torch.float32 or not w_dt.is_contiguous():
        return None
    return _step_gated_fused(state, None, w_dt, x_dbl, off_b, off_c, b_weight, c_weight, eps,
                             mimo_p, u_t, params, n_rot, z, d_skip, dt_bias, overlap)


def _step_gated_fused(state, dt, w_dt, x_dbl, off_b, off_c, b_weight, c_weight, eps, mimo_p,
                      u_t, params, n_rot, z, d_skip, dt_bias, overlap=False):
    lib = _lib.load()
    h = state[0]
    dev = _require_cuda(h, dt, w_dt, x_dbl, u_t, z, d_skip)
    B, D, N = h.shape
    if x_dbl.dtype != torch.float32 or x_dbl.stride(-1) != 1 or z.stride(-1) != 1:
        return None
    if z.dtype != torch.float32:
        z = z.float()
    uu = u_t if u_t.is_contiguous() else u_t.contiguous()
    dt_du = _dt_code(uu.dtype)
    ar, ai, tk = params
    ds = d_skip.detach().to(torch.float32).contiguous()
    if (b_weight is None) != (c_weight is None):
        raise ValueError("m3_step_gated_fused_: both BCNorm weights or neither")
    wb = None if b_weight is None else b_weight.detach().to(torch.float32).contiguous()
    wc = None if c_weight is None else c_weight.detach().to(torch.float32).contiguous()
    bias = None if dt_bias is None else dt_bias.detach().to(torch.float32).contiguous()
    out = torch.empty(B, D, device=dev, dtype=torch.float32)
    desc = StepDesc(B, D, N, int(n_rot), dt_du, M3_F32)
    if len(state) == 2:
        dbu, fa, fb = state[1], None, None
    else:
        dbu, fa, fb = None, state[1], state[2]
    tail = (ctypes_ptr(bias), x_dbl.data_ptr(), x_dbl.stride(0), int(off_b), int(off_c),
            ctypes_ptr(wb), ctypes_ptr(wc), float(eps), uu.data_ptr(), ar.data_ptr(),
            ai.data_ptr(), tk.data_ptr(), z.data_ptr(), z.stride(0), ds.data_ptr(),
            out.data_ptr(), _stream(dev))
    with torch.cuda.device(dev):
        if w_dt is None:
            rc = lib.m3_step_gated_fused(desc, int(mimo_p), h.data_ptr(), ctypes_ptr(dbu),
                                         ctypes_ptr(fa), ctypes_ptr(fb), dt.data_ptr(),
                                         dt.stride(0), *tail)
        else:
            rc = lib.m3_step_gated_fused_proj(desc, int(mimo_p), h.data_ptr(), ctypes_ptr(dbu),
                                              ctypes_ptr(fa), ctypes_ptr(fb), w_dt.data_ptr(),
                                              w_dt.shape[1], *tail[:-1], int(bool(overlap)),
                                              tail[-1])
    if rc == M3_ERR_UNSUPPORTED:
        return None
    _lib.check(rc)
    return out


def m3_step(state, delta_t, u_t, Bc_t, Cc_t, A_real, A_imag, track, n_rot, n_state):
    """Functional step: returns (y, (h_new, dbu_new)); ``state`` may be None."""
    B, D = u_t.shape
    N = Bc_t.shape[-1]
    if state is None:
        h = torch.zeros(B, D, N, device=u_t.device, dtype=torch.float32)
        dbu = torch.zeros_like(h)
    else:
        h, dbu = (s.detach().to(torch.float32).clone(memory_format=torch.contiguous_format)
                  for s in state)
    y = m3_step_(h, dbu, delta_t, u_t, Bc_t, Cc_t, A_real, A_imag, track, n_rot, n_state)
    return y, (h, dbu)


def verify(device="cuda", thorough=True, verbose=True):
    """The correctness gate of triton_scan.py:340-398 for these kernels: forward
    and all gradients against a float64 torch recurrence; raises on mismatch."""
    from .verify import verify as _verify
    return _verify(device=device, thorough=thorough, verbose=verbose)


def device_error(clear=True):
    """Device-side error word of the current device (0 = none)."""
    import ctypes
    lib = _lib.load()
    code = ctypes.c_int32(0)
    _lib.check(lib.m3_device_error(ctypes.byref(code), int(bool(clear))))
    return code.value
