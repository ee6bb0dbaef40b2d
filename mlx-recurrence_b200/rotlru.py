"""Rotational LRU pair-diagonal scan ``h_t = a_t R(theta_t) h_{t-1} + x_t``.

Drop-in for ``mlx_recurrence/rotlru.py`` (v0.3.0): same functions, argument
meaning, validation messages and shape rules, backed by the sm_100a kernels
in ``csrc/diag_scan.cu``. Pairs are interleaved in the channel axis
(``x[..., 2p]`` is u, ``x[..., 2p+1]`` is w); ``a``, ``cs = cos(theta)`` and
``sn = sin(theta)`` are per pair. The kernels are range-agnostic: ``a`` may be
negative and ``(cs, sn)`` need not be normalised (``rotlru.py:18-22``).

VJP (``rotlru.py:35-40``): ``adj_t = gy_t + a_{t+1} M_{t+1}^T adj_{t+1}``,
``grad_x = adj``, ``grad_a = adj . (M h_{t-1})``,
``grad_cs = a (adjU u_{t-1} + adjW w_{t-1})``,
``grad_sn = a (adjW u_{t-1} - adjU w_{t-1})``.
"""

from __future__ import annotations

import torch

from . import _lib
from ._chassis import DEFAULT_SEG, check_segment_shape, common_dtype, grad_out, prep, prep_h0, step_state


def _validate(a, cs, sn, x):
    """Shape checks and messages of ``rotlru.py:61-73``."""
    if a.dim() != 3:
        raise ValueError(f"a must be [B, L, Dp], got shape {tuple(a.shape)}")
    if a.shape != cs.shape or a.shape != sn.shape:
        raise ValueError(
            f"a/cs/sn shapes must match, got {tuple(a.shape)}, {tuple(cs.shape)}, {tuple(sn.shape)}"
        )
    B, L, Dp = a.shape
    if tuple(x.shape) != (B, L, 2 * Dp):
        raise ValueError(f"x must be [B, L, 2*Dp] = [{B}, {L}, {2 * Dp}], got {tuple(x.shape)}")
    return B, L, Dp


class _RotLRUScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, cs, sn, x, seg, h0, want_final):
        # an unused output's cotangent arrives as None (no zero tensor is made)
        ctx.set_materialize_grads(False)
        Bt, L, Dp = _validate(a, cs, sn, x)
        check_segment_shape(L, seg, x.shape[2], "D")  # rotlru.py:282
        dev = _lib.require_cuda(a, cs, sn, x)
        dt = common_dtype(a, cs, sn, x)
        a_, c_, s_, x_ = (prep(t, dt) for t in (a, cs, sn, x))
        D = 2 * Dp
        h0_ = prep_h0(h0, (Bt, D), dev)
        y = torch.empty((Bt, L, D), dtype=torch.float32, device=dev)
        ckpt = torch.empty((Bt, L // seg, D), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mr_rotlru_fwd_h0", _lib.ptr(a_), _lib.ptr(c_), _lib.ptr(s_), _lib.ptr(x_),
                      _lib.DTYPE_CODE[dt], Bt, L, Dp, seg, _lib.ptr(y), _lib.ptr(ckpt), _lib.ptr(h0_),
                      _lib.stream_of(dev))
        ctx.save_for_backward(a_, c_, s_, x_, ckpt, h0_)
        ctx.seg = seg
        return y, ckpt[:, -1].clone() if want_final else y.new_empty(0)

    @staticmethod
    def backward(ctx, gy, gfinal):
        a_, c_, s_, x_, ckpt, h0_ = ctx.saved_tensors
        Bt, L, Dp = a_.shape
        dev = a_.device
        code = _lib.DTYPE_CODE[a_.dtype]
        gy = grad_out(gy, (Bt, L, 2 * Dp), dev)
        gf = None if gfinal is None else gfinal.to(torch.float32).contiguous()
        ga, gc, gs, gx = (torch.empty_like(t) for t in (a_, c_, s_, x_))
        gh0 = torch.empty_like(h0_) if (h0_ is not None and ctx.needs_input_grad[5]) else None
        with torch.cuda.device(dev):
            lib = _lib.load()
            nws = lib.mr_rotlru_bwd_workspace_bytes(code, Bt, L, Dp, ctx.seg)
            ws = torch.empty(nws, dtype=torch.uint8, device=dev) if nws else None
            _lib.call("mr_rotlru_bwd_h0", _lib.ptr(gy), _lib.ptr(gf), _lib.ptr(ckpt), _lib.ptr(a_),
                      _lib.ptr(c_), _lib.ptr(s_), _lib.ptr(x_), code, Bt, L, Dp, ctx.seg,
                      _lib.ptr(ga), _lib.ptr(gc), _lib.ptr(gs), _lib.ptr(gx), _lib.ptr(ws), nws,
                      _lib.ptr(h0_), _lib.ptr(gh0), _lib.stream_of(dev))
        return ga, gc, gs, gx, None, gh0, None


def rotlru_scan(a, cs, sn, x, seg=DEFAULT_SEG, h0=None):
    """Rotational LRU pair-diagonal scan (``rotlru.py:297-320``).

    Args:
        a:   [B, L, Dp] per-pair magnitude gate (any real value).
        cs:  [B, L, Dp] cos(theta_t).
        sn:  [B, L, Dp] sin(theta_t).
        x:   [B, L, D]  drive, D = 2*Dp, pairs interleaved (u, w).
        seg: checkpoint segment length (L % seg == 0; default 32).
        h0:  optional initial state [B, D] (pairs interleaved; differentiable).
             Not in the reference, which starts from zero.

    Returns:
        y:   [B, L, D] float32.

    ``D`` must be a multiple of 32. Gradients flow to all four inputs.
    """
    y, _ = _RotLRUScan.apply(a, cs, sn, x, seg, h0, False)
    return y


def rotlru_scan_with_state(a, cs, sn, x, seg=DEFAULT_SEG, h0=None):
    """Rotational LRU scan that also returns the final state [B, D] (``rotlru.py:323-331``).
    Passing it back as ``h0`` continues the scan (chunked prefill)."""
    return _RotLRUScan.apply(a, cs, sn, x, seg, h0, True)


class _RotLRUAngleScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, theta, x, seg, h0, want_final):
        ctx.set_materialize_grads(False)
        if a.dim() == 3 and theta.shape != a.shape:
            raise ValueError(f"a/theta shapes must match, got {tuple(a.shape)}, {tuple(theta.shape)}")
        Bt, L, Dp = _validate(a, theta, theta, x)
        check_segment_shape(L, seg, x.shape[2], "D")
        dev = _lib.require_cuda(a, theta, x)
        dt = common_dtype(a, theta, x)
        a_, t_, x_ = (prep(t, dt) for t in (a, theta, x))
        D = 2 * Dp
        h0_ = prep_h0(h0, (Bt, D), dev)
        y = torch.empty((Bt, L, D), dtype=torch.float32, device=dev)
        ckpt = torch.empty((Bt, L // seg, D), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mr_rotlru_angle_fwd", _lib.ptr(a_), _lib.ptr(t_), _lib.ptr(x_), _lib.DTYPE_CODE[dt], Bt,
                      L, Dp, seg, _lib.ptr(y), _lib.ptr(ckpt), _lib.ptr(h0_), _lib.stream_of(dev))
        ctx.save_for_backward(a_, t_, x_, ckpt, h0_)
        ctx.seg = seg
        return y, ckpt[:, -1].clone() if want_final else y.new_empty(0)

    @staticmethod
    def backward(ctx, gy, gfinal):
        a_, t_, x_, ckpt, h0_ = ctx.saved_tensors
        Bt, L, Dp = a_.shape
        dev = a_.device
        code = _lib.DTYPE_CODE[a_.dtype]
        gy = grad_out(gy, (Bt, L, 2 * Dp), dev)
        gf = None if gfinal is None else gfinal.to(torch.float32).contiguous()
        ga, gt, gx = (torch.empty_like(t) for t in (a_, t_, x_))
        gh0 = torch.empty_like(h0_) if (h0_ is not None and ctx.needs_input_grad[4]) else None
        with torch.cuda.device(dev):
            lib = _lib.load()
            nws = lib.mr_rotlru_bwd_workspace_bytes(code, Bt, L, Dp, ctx.seg)
            ws = torch.empty(nws, dtype=torch.uint8, device=dev) if nws else None
            _lib.call("mr_rotlru_angle_bwd", _lib.ptr(gy), _lib.ptr(gf), _lib.ptr(ckpt), _lib.ptr(a_),
                      _lib.ptr(t_), _lib.ptr(x_), code, Bt, L, Dp, ctx.seg, _lib.ptr(ga), _lib.ptr(gt),
                      _lib.ptr(gx), _lib.ptr(ws), nws, _lib.ptr(h0_), _lib.ptr(gh0), _lib.stream_of(dev))
        return ga, gt, gx, None, gh0, None


def rotlru_scan_angle(a, theta, x, seg=DEFAULT_SEG, h0=None):
    """The rotLRU scan taking the rotation angle itself (no counterpart in the
    reference, whose callers form ``cs = cos(theta)``, ``sn = sin(theta)`` in
    host code and pass both, ``rotlru.py:18-22``). Equal to
    ``rotlru_scan(a, cos(theta), sin(theta), x)``; the kernels form cos and sin
    in float32 as they load each tile, so the scan reads four streams instead of
    five and no cs/sn tensors (or their gradients) are materialised.

    Args:
        a:     [B, L, Dp] per-pair magnitude gate.
        theta: [B, L, Dp] rotation angle (radians).
        x:     [B, L, D]  drive, D = 2*Dp, pairs interleaved (u, w).
        seg:   checkpoint segment length (L % seg == 0).
        h0:    optional initial state [B, D] (differentiable).

    Returns:
        y: [B, L, D] float32. Gradients flow to a, theta, x (and h0):
        ``grad_theta = cos(theta) grad_sn - sin(theta) grad_cs``.
    """
    y, _ = _RotLRUAngleScan.apply(a, theta, x, seg, h0, False)
    return y


def rotlru_scan_angle_with_state(a, theta, x, seg=DEFAULT_SEG, h0=None):
    """:func:`rotlru_scan_angle` that also returns the final state [B, D]."""
    return _RotLRUAngleScan.apply(a, theta, x, seg, h0, True)


def rotlru_scan_reference(a, cs, sn, x, h0=None):
    """Per-step torch loop (``rotlru.py:338-351``). Differentiable, any device."""
    Bt, L, Dp = _validate(a, cs, sn, x)
    xp = x.reshape(Bt, L, Dp, 2)
    ft = torch.promote_types(a.dtype, torch.float32)
    if h0 is None:
        u = torch.zeros((Bt, Dp), dtype=ft, device=a.device)
        w = torch.zeros((Bt, Dp), dtype=ft, device=a.device)
    else:
        hp = h0.to(ft).reshape(Bt, Dp, 2)
        u, w = hp[..., 0], hp[..., 1]
    ys = []
    for t in range(L):
        at, c, s = a[:, t, :], cs[:, t, :], sn[:, t, :]
        un = at * (c * u - s * w) + xp[:, t, :, 0]
        wn = at * (s * u + c * w) + xp[:, t, :, 1]
        u, w = un, wn
        ys.append(torch.stack([u, w], dim=-1).reshape(Bt, 2 * Dp))
    return torch.stack(ys, dim=1)


def rotlru_step(a, cs, sn, x, state):
    """One decode step (no counterpart in the reference): advances ``state``
    [B, 2Dp] (float32, pairs interleaved) in place by one step of
    ``rotlru.py:338-351`` and returns the new state as y [B, 2Dp] float32.
    ``a``, ``cs``, ``sn`` [B, Dp], ``x`` [B, 2Dp]. Not differentiable."""
    if a.dim() != 2 or cs.shape != a.shape or sn.shape != a.shape:
        raise ValueError(f"a/cs/sn must all be [B, Dp], got {tuple(a.shape)}, {tuple(cs.shape)}, "
                         f"{tuple(sn.shape)}")
    Bt, Dp = a.shape
    if tuple(x.shape) != (Bt, 2 * Dp):
        raise ValueError(f"x must be [B, 2*Dp] = [{Bt}, {2 * Dp}], got {tuple(x.shape)}")
    dev = _lib.require_cuda(a, cs, sn, x, state)
    state = step_state(state, (Bt, 2 * Dp), dev)
    dt = common_dtype(a, cs, sn, x)
    a_, c_, s_, x_ = (prep(t.detach(), dt) for t in (a, cs, sn, x))
    y = torch.empty((Bt, 2 * Dp), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("mr_rotlru_step", _lib.ptr(a_), _lib.ptr(c_), _lib.ptr(s_), _lib.ptr(x_), _lib.DTYPE_CODE[dt],
                  Bt, Dp, _lib.ptr(state), _lib.ptr(y), _lib.stream_of(dev))
    return y
