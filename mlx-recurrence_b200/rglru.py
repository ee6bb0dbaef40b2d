"""RG-LRU diagonal recurrence ``h_t = a_t * h_{t-1} + x_t``, ``y_t = h_t``.

Drop-in for ``mlx_recurrence/rglru.py`` (v0.3.0): same functions, argument
meaning, shape rules and errors, backed by the sm_100a kernels in
``csrc/diag_scan.cu`` through ``libmlrec.so``. The gates ``a`` and the gated
input ``x = sqrt(1 - a^2) * (i * x_raw)`` are computed by the caller, as in
the reference (``rglru.py:19-27``).

VJP (``rglru.py:36-39``): ``adj_t = gy_t + a_{t+1} adj_{t+1}``,
``grad_x[t] = adj_t``, ``grad_a[t] = adj_t * h_{t-1}``. A cotangent on the
final state of ``rglru_scan_with_state`` seeds ``adj`` (the reference's VJP
drops it, ``rglru.py:226``; its pure loop does not).
"""

from __future__ import annotations

import torch

from . import _lib
from ._chassis import DEFAULT_SEG, check_segment_shape, common_dtype, grad_out, prep, prep_h0, step_state


class _RGLRUScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, x, seg, h0, want_final):
        # an unused output's cotangent arrives as None (no zero tensor is made)
        ctx.set_materialize_grads(False)
        if a.dim() != 3 or x.shape != a.shape:
            raise ValueError(f"a and x must both be [B, L, D], got {tuple(a.shape)} and {tuple(x.shape)}")
        Bt, L, D = a.shape
        check_segment_shape(L, seg, D, "D")  # rglru.py:220
        dev = _lib.require_cuda(a, x)
        dt = common_dtype(a, x)
        a_, x_ = prep(a, dt), prep(x, dt)
        h0_ = prep_h0(h0, (Bt, D), dev)
        y = torch.empty((Bt, L, D), dtype=torch.float32, device=dev)
        ckpt = torch.empty((Bt, L // seg, D), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mr_rglru_fwd_h0", _lib.ptr(a_), _lib.ptr(x_), _lib.DTYPE_CODE[dt], Bt, L, D, seg,
                      _lib.ptr(y), _lib.ptr(ckpt), _lib.ptr(h0_), _lib.stream_of(dev))
        ctx.save_for_backward(a_, x_, ckpt, h0_)
        ctx.seg = seg
        return y, ckpt[:, -1].clone() if want_final else y.new_empty(0)

    @staticmethod
    def backward(ctx, gy, gfinal):
        a_, x_, ckpt, h0_ = ctx.saved_tensors
        Bt, L, D = a_.shape
        dev = a_.device
        dt = a_.dtype
        gy = grad_out(gy, (Bt, L, D), dev)
        gf = None if gfinal is None else gfinal.to(torch.float32).contiguous()
        ga = torch.empty_like(a_)
        gx = torch.empty_like(x_)
        gh0 = torch.empty_like(h0_) if (h0_ is not None and ctx.needs_input_grad[3]) else None
        code = _lib.DTYPE_CODE[dt]
        with torch.cuda.device(dev):
            lib = _lib.load()
            nws = lib.mr_rglru_bwd_workspace_bytes(code, Bt, L, D, ctx.seg)
            ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=dev) if nws else None
            _lib.call("mr_rglru_bwd_h0", _lib.ptr(gy), _lib.ptr(gf), _lib.ptr(ckpt), _lib.ptr(a_),
                      _lib.ptr(x_), code, Bt, L, D, ctx.seg, _lib.ptr(ga), _lib.ptr(gx), _lib.ptr(ws),
                      nws, _lib.ptr(h0_), _lib.ptr(gh0), _lib.stream_of(dev))
        return ga, gx, None, gh0, None


def rglru_scan(a, x, seg=DEFAULT_SEG, h0=None):
    """RG-LRU diagonal linear scan (``rglru.py:234-256``).

    Args:
        a:   [B, L, D] per-channel recurrent gate (any real value).
        x:   [B, L, D] the already-gated input.
        seg: checkpoint segment length (L % seg == 0; default 32).
        h0:  optional initial state [B, D] (float32 state; differentiable).
             Not in the reference, which starts from zero.

    Returns:
        y:   [B, L, D] float32, ``y_t = h_t``.

    ``D`` must be a multiple of 32. State and accumulation are float32; bf16
    and fp16 inputs are widened on read and their gradients are returned in
    the input dtype.
    """
    y, _ = _RGLRUScan.apply(a, x, seg, h0, False)
    return y


def rglru_scan_with_state(a, x, seg=DEFAULT_SEG, h0=None):
    """RG-LRU scan that also returns the final state [B, D] (``rglru.py:259-267``).
    Passing it back as ``h0`` continues the scan (chunked prefill)."""
    return _RGLRUScan.apply(a, x, seg, h0, True)


def rglru_scan_reference(a, x, h0=None):
    """Per-step torch loop (``rglru.py:274-282``). Differentiable, any device."""
    Bt, L, D = a.shape
    ft = torch.promote_types(a.dtype, torch.float32)
    h = torch.zeros((Bt, D), dtype=ft, device=a.device) if h0 is None else h0.to(ft)
    ys = []
    for t in range(L):
        h = a[:, t, :] * h + x[:, t, :]
        ys.append(h)
    return torch.stack(ys, dim=1)


def rglru_step(a, x, state):
    """One decode step (no counterpart in the reference): ``state`` [B, D]
    (float32) <- a * state + x in place (``rglru.py:274-282``); returns the new
    state as y [B, D] float32. ``a``, ``x`` [B, D]. Not differentiable."""
    if a.dim() != 2 or x.shape != a.shape:
        raise ValueError(f"a and x must both be [B, D], got {tuple(a.shape)} and {tuple(x.shape)}")
    Bt, D = a.shape
    dev = _lib.require_cuda(a, x, state)
    state = step_state(state, (Bt, D), dev)
    dt = common_dtype(a, x)
    a_, x_ = prep(a.detach(), dt), prep(x.detach(), dt)
    y = torch.empty((Bt, D), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("mr_rglru_step", _lib.ptr(a_), _lib.ptr(x_), _lib.DTYPE_CODE[dt], Bt, D, _lib.ptr(state),
                  _lib.ptr(y), _lib.stream_of(dev))
    return y


class _RGLRUGatedScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, r, i, lam, c, seg, h0, want_final):
        ctx.set_materialize_grads(False)
        if x.dim() != 3 or r.shape != x.shape or i.shape != x.shape:
            raise ValueError(f"x, r, i must all be [B, L, D], got {tuple(x.shape)}, {tuple(r.shape)}, "
                             f"{tuple(i.shape)}")
        Bt, L, D = x.shape
        if tuple(lam.shape) != (D,):
            raise ValueError(f"lam must be [D] = [{D}], got {tuple(lam.shape)}")
        check_segment_shape(L, seg, D, "D")
        dev = _lib.require_cuda(x, r, i, lam)
        dt = common_dtype(x, r, i)
        x_, r_, i_ = (prep(t, dt) for t in (x, r, i))
        lam_ = lam.detach().to(torch.float32).contiguous()
        h0_ = prep_h0(h0, (Bt, D), dev)
        y = torch.empty((Bt, L, D), dtype=torch.float32, device=dev)
        ckpt = torch.empty((Bt, L // seg, D), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mr_rglru_gated_fwd", _lib.ptr(x_), _lib.ptr(r_), _lib.ptr(i_), _lib.ptr(lam_), float(c),
                      _lib.DTYPE_CODE[dt], Bt, L, D, seg, _lib.ptr(y), _lib.ptr(ckpt), _lib.ptr(h0_),
                      _lib.stream_of(dev))
        ctx.save_for_backward(x_, r_, i_, lam_, ckpt, h0_)
        ctx.seg, ctx.c = seg, float(c)
        return y, ckpt[:, -1].clone() if want_final else y.new_empty(0)

    @staticmethod
    def backward(ctx, gy, gfinal):
        x_, r_, i_, lam_, ckpt, h0_ = ctx.saved_tensors
        Bt, L, D = x_.shape
        dev = x_.device
        code = _lib.DTYPE_CODE[x_.dtype]
        gy = grad_out(gy, (Bt, L, D), dev)
        gf = None if gfinal is None else gfinal.to(torch.float32).contiguous()
        gx, gr, gi = (torch.empty_like(t) for t in (x_, r_, i_))
        glam = torch.empty_like(lam_)
        gh0 = torch.empty_like(h0_) if (h0_ is not None and ctx.needs_input_grad[6]) else None
        with torch.cuda.device(dev):
            lib = _lib.load()
            nws = lib.mr_rglru_gated_bwd_workspace_bytes(code, Bt, L, D, ctx.seg)
            ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=dev)
            _lib.call("mr_rglru_gated_bwd", _lib.ptr(gy), _lib.ptr(gf), _lib.ptr(ckpt), _lib.ptr(x_), _lib.ptr(r_),
                      _lib.ptr(i_), _lib.ptr(lam_), ctx.c, code, Bt, L, D, ctx.seg, _lib.ptr(gx), _lib.ptr(gr),
                      _lib.ptr(gi), _lib.ptr(glam), _lib.ptr(ws), ws.numel(), _lib.ptr(h0_), _lib.ptr(gh0),
                      _lib.stream_of(dev))
        return gx, gr, gi, glam, None, None, gh0, None


def rglru_scan_gated(x, r, i, lam, c=8.0, seg=DEFAULT_SEG, h0=None):
    """RG-LRU with its input gating folded into the scan kernels.

    The reference computes the gate and the gated input in MLX host code ahead
    of the scan (``rglru.py:8-27``) and passes ``a`` and ``b`` through memory;
    here they are formed as the kernels load x, r and i:

        a_t = sigmoid(lam)^(c r_t),  b_t = sqrt(1 - a_t^2) i_t x_t,  h_t = a_t h_{t-1} + b_t

    Args:
        x:   [B, L, D] input.
        r:   [B, L, D] activated recurrence gate (in [0, 1]).
        i:   [B, L, D] activated input gate.
        lam: [D] per-channel Lambda (float32 state of the gate).
        c:   gate exponent scale (8 in Griffin).
        seg, h0: as in :func:`rglru_scan`.

    Returns:
        y:   [B, L, D] float32. Differentiable in x, r, i, lam and h0.
    """
    y, _ = _RGLRUGatedScan.apply(x, r, i, lam, c, seg, h0, False)
    return y


def rglru_scan_gated_with_state(x, r, i, lam, c=8.0, seg=DEFAULT_SEG, h0=None):
    """:func:`rglru_scan_gated` that also returns the final state [B, D]."""
    return _RGLRUGatedScan.apply(x, r, i, lam, c, seg, h0, True)
