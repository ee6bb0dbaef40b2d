"""Gated linear attention recurrence with a scalar forget gate per head.

Drop-in for ``mlx_recurrence/gla.py`` (v0.3.0). Per head the state is the
``Dh x Dh`` matrix ``h[i, j]``::

    h[i, j] = gate[b,t,head] * h[i, j] + k[b,t,head,i] * v[b,t,head,j]
    o[b,t,head,j] = sum_i q[b,t,head,i] * h[i, j]      (post-update state)

Same functions, argument meaning and shape rules (``L % seg == 0``,
``Dh % 32 == 0``) as the reference, backed by the sm_100a kernels of
``libmlrec.so``. Outputs are float32; state and accumulation float32;
gradients come back in the input dtype.
"""

from __future__ import annotations

import torch

from . import _lib
from ._chassis import DEFAULT_SEG, check_segment_shape, common_dtype, grad_out, prep, prep_h0, step_state


def _validate(q, k, v, gates):
    if q.dim() != 4:
        raise ValueError(f"q must be [B, L, H, Dh], got shape {tuple(q.shape)}")
    Bt, L, H, Dh = q.shape
    for name, t in (("k", k), ("v", v)):
        if t.shape != q.shape:
            raise ValueError(f"{name} must match q's shape {tuple(q.shape)}, got {tuple(t.shape)}")
    if tuple(gates.shape) != (Bt, L, H):
        raise ValueError(f"gates must be [B, L, H] = [{Bt}, {L}, {H}], got {tuple(gates.shape)}")
    return Bt, L, H, Dh


class _GLAScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, gates, seg, h0, want_final):
        # an unused output's cotangent arrives as None (no zero tensor is made)
        ctx.set_materialize_grads(False)
        Bt, L, H, Dh = _validate(q, k, v, gates)
        check_segment_shape(L, seg, Dh, "Dh")  # gla.py:287
        dev = _lib.require_cuda(q, k, v, gates)
        dt = common_dtype(q, k, v, gates)
        q_, k_, v_, g_ = (prep(t, dt) for t in (q, k, v, gates))
        code = _lib.DTYPE_CODE[dt]
        h0_ = prep_h0(h0, (Bt, H, Dh, Dh), dev)
        # The checkpoints are internal (only the last one is returned, gla.py:329):
        # take the spacing of the fastest path for these shapes (same final state).
        seg_i = int(_lib.load().mr_gla_preferred_seg(code, L, Dh, seg))
        y = torch.empty((Bt, L, H, Dh), dtype=torch.float32, device=dev)
        ckpt = torch.empty((Bt, L // seg_i, H, Dh, Dh), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mr_gla_fwd_h0", _lib.ptr(q_), _lib.ptr(k_), _lib.ptr(v_), _lib.ptr(g_),
                      code, Bt, L, H, Dh, seg_i, _lib.ptr(y), _lib.ptr(ckpt), _lib.ptr(h0_),
                      _lib.stream_of(dev))
        ctx.save_for_backward(q_, k_, v_, g_, ckpt, h0_)
        ctx.seg = seg_i
        return y, ckpt[:, -1].clone() if want_final else y.new_empty(0)

    @staticmethod
    def backward(ctx, gy, gfinal):
        q_, k_, v_, g_, ckpt, h0_ = ctx.saved_tensors
        Bt, L, H, Dh = q_.shape
        dev = q_.device
        code = _lib.DTYPE_CODE[q_.dtype]
        gy = grad_out(gy, (Bt, L, H, Dh), dev)
        gf = None if gfinal is None else gfinal.to(torch.float32).contiguous()
        gq, gk, gv, gg = (torch.empty_like(t) for t in (q_, k_, v_, g_))
        gh0 = torch.empty_like(h0_) if (h0_ is not None and ctx.needs_input_grad[5]) else None
        with torch.cuda.device(dev):
            lib = _lib.load()
            nws = lib.mr_gla_bwd_workspace_bytes(code, Bt, L, H, Dh, ctx.seg)
            ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=dev)
            _lib.call("mr_gla_bwd_h0", _lib.ptr(gy), _lib.ptr(gf), _lib.ptr(ckpt), _lib.ptr(q_),
                      _lib.ptr(k_), _lib.ptr(v_), _lib.ptr(g_), code, Bt, L, H, Dh, ctx.seg,
                      _lib.ptr(gq), _lib.ptr(gk), _lib.ptr(gv), _lib.ptr(gg), _lib.ptr(ws),
                      ws.numel(), _lib.ptr(h0_), _lib.ptr(gh0), _lib.stream_of(dev))
        return gq, gk, gv, gg, None, gh0, None


def gla_scan(q, k, v, gates, seg=DEFAULT_SEG, h0=None):
    """Gated linear attention recurrence (``gla.py:301-318``).

    Args:
        q, k, v: [B, L, H, Dh] (q pre-scaled / post-RoPE)
        gates:   [B, L, H] scalar forget gate per head
        seg:     checkpoint segment length (L % seg == 0; default 32)
        h0:      optional initial state [B, H, Dh, Dh] (the final state's layout;
                 differentiable). Not in the reference, which starts from zero.

    Returns:
        y:       [B, L, H, Dh] float32
    """
    y, _ = _GLAScan.apply(q, k, v, gates, seg, h0, False)
    return y


def gla_scan_with_state(q, k, v, gates, seg=DEFAULT_SEG, h0=None):
    """GLA scan that also returns the final state ``[B, H, Dh, Dh]`` (``gla.py:321-329``).
    Passing it back as ``h0`` continues the scan (chunked prefill)."""
    return _GLAScan.apply(q, k, v, gates, seg, h0, True)


def gla_scan_reference(q, k, v, gates, h0=None):
    """Per-step torch loop (``gla.py:336-346``). Differentiable, any device."""
    Bt, L, H, Dh = q.shape
    ft = torch.promote_types(q.dtype, torch.float32)
    h = torch.zeros((Bt, H, Dh, Dh), dtype=ft, device=q.device) if h0 is None else h0.to(ft)
    ys = []
    for t in range(L):
        g = gates[:, t, :, None, None]
        kv = k[:, t, :, :, None] * v[:, t, :, None, :]
        h = g * h + kv
        ys.append(torch.sum(q[:, t, :, :, None] * h, dim=-2))
    return torch.stack(ys, dim=1)


def gla_step(q, k, v, gates, state):
    """One decode step (no counterpart in the reference): advances ``state``
    [B, H, Dh, Dh] (float32, the final state's layout) in place by one step of
    ``gla.py:336-346`` and returns y [B, H, Dh] float32. ``q``, ``k``, ``v``
    [B, H, Dh], ``gates`` [B, H]. Not differentiable."""
    if q.dim() != 3 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v must all be [B, H, Dh], got {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    Bt, H, Dh = q.shape
    if tuple(gates.shape) != (Bt, H):
        raise ValueError(f"gates must be [B, H] = [{Bt}, {H}], got {tuple(gates.shape)}")
    dev = _lib.require_cuda(q, k, v, gates, state)
    state = step_state(state, (Bt, H, Dh, Dh), dev)
    dt = common_dtype(q, k, v, gates)
    q_, k_, v_, g_ = (prep(t.detach(), dt) for t in (q, k, v, gates))
    y = torch.empty((Bt, H, Dh), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("mr_gla_step", _lib.ptr(q_), _lib.ptr(k_), _lib.ptr(v_), _lib.ptr(g_), _lib.DTYPE_CODE[dt],
                  Bt, H, Dh, _lib.ptr(state), _lib.ptr(y), _lib.stream_of(dev))
    return y
