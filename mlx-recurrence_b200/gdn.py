"""Gated DeltaNet recurrence (delta rule with a scalar decay per head).

The reference carries this recurrence as a design only
(``docs/DESIGN_gated_deltanet.md``); this module builds it from that design's
pinned recurrence (section 1) and adjoint (section 4). Per head the state is
the ``Dh x Dh`` matrix ``S[i, j]`` (i the key axis, j the value axis)::

    S_t = alpha_t (I - beta_t k_t k_t^T) S_{t-1} + beta_t k_t v_t^T
    o_t = S_t^T q_t                                   (post-update state)

Input contract (the design's section 7 default): ``q``, ``k`` arrive
L2-normalised per head and ``alpha``, ``beta`` already activated (``alpha`` in
(0, 1], ``beta`` in (0, 1) make every step a contraction); the kernels apply
the recurrence as given to any values. Same chassis as the other plug-ins:
``L % seg == 0``, segment checkpoints, recompute backward; ``Dh`` 32 or 64.
Outputs are float32, state and accumulation float32, gradients in the input
dtype.
"""

from __future__ import annotations

import torch

from . import _lib
from ._chassis import DEFAULT_SEG, check_segment_shape, common_dtype, grad_out, prep, prep_h0, step_state


def _validate(q, k, v, alpha, beta):
    if q.dim() != 4:
        raise ValueError(f"q must be [B, L, H, Dh], got shape {tuple(q.shape)}")
    Bt, L, H, Dh = q.shape
    for name, t in (("k", k), ("v", v)):
        if t.shape != q.shape:
            raise ValueError(f"{name} must match q's shape {tuple(q.shape)}, got {tuple(t.shape)}")
    for name, t in (("alpha", alpha), ("beta", beta)):
        if tuple(t.shape) != (Bt, L, H):
            raise ValueError(f"{name} must be [B, L, H] = [{Bt}, {L}, {H}], got {tuple(t.shape)}")
    if Dh not in (32, 64):
        raise ValueError(f"Dh={Dh} is not supported by the Gated DeltaNet kernels (32 or 64)")
    return Bt, L, H, Dh


class _GDNScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, alpha, beta, seg, h0, want_final):
        ctx.set_materialize_grads(False)
        Bt, L, H, Dh = _validate(q, k, v, alpha, beta)
        check_segment_shape(L, seg, Dh, "Dh")
        dev = _lib.require_cuda(q, k, v, alpha, beta)
        dt = common_dtype(q, k, v, alpha, beta)
        q_, k_, v_, a_, b_ = (prep(t, dt) for t in (q, k, v, alpha, beta))
        code = _lib.DTYPE_CODE[dt]
        h0_ = prep_h0(h0, (Bt, H, Dh, Dh), dev)
        y = torch.empty((Bt, L, H, Dh), dtype=torch.float32, device=dev)
        ckpt = torch.empty((Bt, L // seg, H, Dh, Dh), dtype=torch.float32, device=dev)
        # w of every step, kept for the backward only when a gradient is wanted
        cache = (torch.empty((Bt, L, H, Dh), dtype=torch.float32, device=dev)
                 if any(ctx.needs_input_grad) else None)
        with torch.cuda.device(dev):
            nws = _lib.load().mr_gdn_fwd_workspace_bytes(code, Bt, L, H, Dh, seg)
            ws = torch.empty(nws, dtype=torch.uint8, device=dev) if nws else None
            _lib.call("mr_gdn_fwd", _lib.ptr(q_), _lib.ptr(k_), _lib.ptr(v_), _lib.ptr(a_), _lib.ptr(b_), code,
                      Bt, L, H, Dh, seg, _lib.ptr(y), _lib.ptr(ckpt), _lib.ptr(cache), _lib.ptr(h0_),
                      _lib.ptr(ws), nws, _lib.stream_of(dev))
        ctx.save_for_backward(q_, k_, v_, a_, b_, ckpt, cache, h0_)
        ctx.seg = seg
        return y, ckpt[:, -1].clone() if want_final else y.new_empty(0)

    @staticmethod
    def backward(ctx, gy, gfinal):
        q_, k_, v_, a_, b_, ckpt, cache, h0_ = ctx.saved_tensors
        Bt, L, H, Dh = q_.shape
        dev = q_.device
        code = _lib.DTYPE_CODE[q_.dtype]
        gy = grad_out(gy, (Bt, L, H, Dh), dev)
        gf = None if gfinal is None else gfinal.to(torch.float32).contiguous()
        gq, gk, gv, ga, gb = (torch.empty_like(t) for t in (q_, k_, v_, a_, b_))
        gh0 = torch.empty_like(h0_) if (h0_ is not None and ctx.needs_input_grad[6]) else None
        with torch.cuda.device(dev):
            lib = _lib.load()
            nws = lib.mr_gdn_bwd_workspace_bytes(code, Bt, L, H, Dh, ctx.seg)
            ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=dev)
            _lib.call("mr_gdn_bwd", _lib.ptr(gy), _lib.ptr(gf), _lib.ptr(ckpt), _lib.ptr(cache), _lib.ptr(q_),
                      _lib.ptr(k_), _lib.ptr(v_), _lib.ptr(a_), _lib.ptr(b_), code, Bt, L, H, Dh, ctx.seg,
                      _lib.ptr(gq), _lib.ptr(gk), _lib.ptr(gv), _lib.ptr(ga), _lib.ptr(gb), _lib.ptr(ws),
                      ws.numel(), _lib.ptr(h0_), _lib.ptr(gh0), _lib.stream_of(dev))
        return gq, gk, gv, ga, gb, None, gh0, None


def gated_deltanet_scan(q, k, v, alpha, beta, seg=DEFAULT_SEG, h0=None):
    """Gated DeltaNet recurrence (``docs/DESIGN_gated_deltanet.md`` R1''/R2').

    Args:
        q, k:  [B, L, H, Dh] query and key, L2-normalised per head by the caller
        v:     [B, L, H, Dh] value
        alpha: [B, L, H] decay per head and step (activated, e.g. exp(a), a <= 0)
        beta:  [B, L, H] write strength per head and step (activated, e.g. sigmoid(b))
        seg:   checkpoint segment length (L % seg == 0; default 32)
        h0:    optional initial state [B, H, Dh, Dh] (differentiable)

    Returns:
        o: [B, L, H, Dh] float32. Gradients flow to q, k, v, alpha, beta (and h0).
    """
    y, _ = _GDNScan.apply(q, k, v, alpha, beta, seg, h0, False)
    return y


def gated_deltanet_scan_with_state(q, k, v, alpha, beta, seg=DEFAULT_SEG, h0=None):
    """:func:`gated_deltanet_scan` that also returns the final state [B, H, Dh, Dh];
    passing it back as ``h0`` continues the scan (chunked prefill)."""
    return _GDNScan.apply(q, k, v, alpha, beta, seg, h0, True)


def gated_deltanet_scan_reference(q, k, v, alpha, beta, h0=None):
    """Per-step torch loop of the recurrence (the design's phase-1 reference,
    ``docs/DESIGN_gated_deltanet.md`` section 7). Differentiable, any device."""
    Bt, L, H, Dh = q.shape
    ft = torch.promote_types(q.dtype, torch.float32)
    S = torch.zeros((Bt, H, Dh, Dh), dtype=ft, device=q.device) if h0 is None else h0.to(ft)
    ys = []
    for t in range(L):
        a = alpha[:, t, :, None, None].to(ft)
        bt = beta[:, t, :, None, None].to(ft)
        kt = k[:, t, :, :, None].to(ft)
        p = torch.sum(kt * S, dim=-2, keepdim=True)
        S = a * S - a * bt * kt * p + bt * kt * v[:, t, :, None, :].to(ft)
        ys.append(torch.sum(q[:, t, :, :, None].to(ft) * S, dim=-2))
    return torch.stack(ys, dim=1)


def gated_deltanet_step(q, k, v, alpha, beta, state):
    """One decode step: advances ``state`` [B, H, Dh, Dh] (float32, the final
    state's layout) in place by one step of the recurrence and returns
    o [B, H, Dh] float32. ``q``, ``k``, ``v`` [B, H, Dh], ``alpha``, ``beta``
    [B, H]. Not differentiable."""
    if q.dim() != 3 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v must all be [B, H, Dh], got {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    Bt, H, Dh = q.shape
    for name, t in (("alpha", alpha), ("beta", beta)):
        if tuple(t.shape) != (Bt, H):
            raise ValueError(f"{name} must be [B, H] = [{Bt}, {H}], got {tuple(t.shape)}")
    if Dh not in (32, 64):
        raise ValueError(f"Dh={Dh} is not supported by the Gated DeltaNet kernels (32 or 64)")
    dev = _lib.require_cuda(q, k, v, alpha, beta, state)
    state = step_state(state, (Bt, H, Dh, Dh), dev)
    dt = common_dtype(q, k, v, alpha, beta)
    q_, k_, v_, a_, b_ = (prep(t.detach(), dt) for t in (q, k, v, alpha, beta))
    y = torch.empty((Bt, H, Dh), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("mr_gdn_step", _lib.ptr(q_), _lib.ptr(k_), _lib.ptr(v_), _lib.ptr(a_), _lib.ptr(b_),
                  _lib.DTYPE_CODE[dt], Bt, H, Dh, _lib.ptr(state), _lib.ptr(y), _lib.stream_of(dev))
    return y
