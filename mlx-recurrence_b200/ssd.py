"""Mamba-2-style head-wise SSD selective scan.

Drop-in for ``mlx_recurrence/ssd.py`` (v0.3.0). Per head and channel the
state is ``h[Dh, N]``::

    decay = exp(delta[b,t,head] * A_neg[head,n])
    h[d,n] = decay * h[d,n] + delta[b,t,head] * B[b,t,head,n] * u[b,t,head,d]
    y[b,t,head,d] = sum_n h[d,n] * C[b,t,head,n]

Same functions, argument meaning and shape rules (``L % seg == 0``,
``Dh % 32 == 0``) as the reference; the work runs in the sm_100a kernels of
``libmlrec.so``. ``A_neg`` is ``[H, N]``; a view that is constant along N
(``A.unsqueeze(-1).expand(H, N)``, stride 0) selects the one-rate-per-head
(Mamba-2) path without a device synchronisation. Outputs are float32; state
and accumulation are float32 for every input dtype; gradients come back in
the input dtype (``grad_A`` is summed over the batch, ``ssd.py:305``).
"""

from __future__ import annotations

import torch

from . import _lib
from ._chassis import DEFAULT_SEG, check_segment_shape, common_dtype, grad_out, prep, prep_h0, step_state


def _validate(u, delta, B, C, A_neg):
    if u.dim() != 4:
        raise ValueError(f"u must be [B, L, H, Dh], got shape {tuple(u.shape)}")
    Bt, L, H, Dh = u.shape
    if A_neg.dim() != 2 or A_neg.shape[0] != H:
        raise ValueError(f"A_neg must be [H, N] = [{H}, N], got {tuple(A_neg.shape)}")
    N = A_neg.shape[1]
    if tuple(delta.shape) != (Bt, L, H):
        raise ValueError(f"delta must be [B, L, H] = [{Bt}, {L}, {H}], got {tuple(delta.shape)}")
    for name, t in (("B", B), ("C", C)):
        if tuple(t.shape) != (Bt, L, H, N):
            raise ValueError(f"{name} must be [B, L, H, N] = [{Bt}, {L}, {H}, {N}], got {tuple(t.shape)}")
    return Bt, L, H, Dh, N


def _a_f32(A_neg):
    """float32 decay rates with (stride_h, stride_n) in elements; stride_n 0
    when the caller's view is constant along N."""
    H, N = A_neg.shape
    if A_neg.stride(1) == 0:
        a = A_neg[:, :1].to(torch.float32).contiguous()
        return a, 1, 0
    return A_neg.to(torch.float32).contiguous(), N, 1


class _SSDScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, B, C, A_neg, seg, h0, want_final):
        # an unused output's cotangent arrives as None (no zero tensor is made)
        ctx.set_materialize_grads(False)
        Bt, L, H, Dh, N = _validate(u, delta, B, C, A_neg)
        check_segment_shape(L, seg, Dh, "Dh")  # ssd.py:328
        dev = _lib.require_cuda(u, delta, B, C, A_neg)
        dt = common_dtype(u, delta, B, C)
        u_, d_, B_, C_ = (prep(t, dt) for t in (u, delta, B, C))
        A32, ash, asn = _a_f32(A_neg)
        h0_ = prep_h0(h0, (Bt, H, Dh, N), dev)
        code = _lib.DTYPE_CODE[dt]
        # The checkpoints are internal (only the last one is returned, ssd.py:361/374):
        # take the spacing of the fastest path for these shapes (same final state).
        seg_i = int(_lib.load().mr_ssd_preferred_seg(code, L, Dh, N, seg, asn))
        y = torch.empty((Bt, L, H, Dh), dtype=torch.float32, device=dev)
        ckpt = torch.empty((Bt, L // seg_i, H, N, Dh), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mr_ssd_fwd_h0", _lib.ptr(u_), _lib.ptr(d_), _lib.ptr(B_), _lib.ptr(C_),
                      _lib.ptr(A32), ash, asn, code, Bt, L, H, Dh, N, seg_i,
                      _lib.ptr(y), _lib.ptr(ckpt), _lib.ptr(h0_), _lib.stream_of(dev))
        ctx.save_for_backward(u_, d_, B_, C_, A32, ckpt, h0_)
        ctx.meta = (seg_i, ash, asn, N)
        # last checkpoint [B, H, N, Dh] -> conceptual state [B, H, Dh, N] (ssd.py:373-374);
        # ssd_scan drops it, so it is only copied out for ssd_scan_with_state
        final = ckpt[:, -1].transpose(-1, -2).contiguous() if want_final else y.new_empty(0)
        return y, final

    @staticmethod
    def backward(ctx, gy, gfinal):
        u_, d_, B_, C_, A32, ckpt, h0_ = ctx.saved_tensors
        seg, ash, asn, N = ctx.meta
        Bt, L, H, Dh = u_.shape
        dev = u_.device
        code = _lib.DTYPE_CODE[u_.dtype]
        gy = grad_out(gy, (Bt, L, H, Dh), dev)
        gf = None if gfinal is None else gfinal.to(torch.float32).contiguous()
        gu, gd, gB, gC = (torch.empty_like(t) for t in (u_, d_, B_, C_))
        gA = torch.empty((H, N), dtype=torch.float32, device=dev)
        gh0 = torch.empty_like(h0_) if (h0_ is not None and ctx.needs_input_grad[6]) else None
        # with one rate per head (asn == 0) row h of gA is d loss / d A_h spread
        # evenly over n; autograd's expand-backward sums it back to the head
        with torch.cuda.device(dev):
            lib = _lib.load()
            nws = lib.mr_ssd_bwd_workspace_bytes(code, Bt, L, H, Dh, N, seg, asn)
            ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=dev)
            _lib.call("mr_ssd_bwd_h0", _lib.ptr(gy), _lib.ptr(gf), _lib.ptr(ckpt), _lib.ptr(u_),
                      _lib.ptr(d_), _lib.ptr(B_), _lib.ptr(C_), _lib.ptr(A32), ash, asn, code, Bt, L,
                      H, Dh, N, seg, _lib.ptr(gu), _lib.ptr(gd), _lib.ptr(gB), _lib.ptr(gC),
                      _lib.ptr(gA), _lib.ptr(ws), ws.numel(), _lib.ptr(h0_), _lib.ptr(gh0),
                      _lib.stream_of(dev))
        return gu, gd, gB, gC, gA, None, gh0, None


def ssd_scan(u, delta, B, C, A_neg, seg=DEFAULT_SEG, h0=None):
    """Head-wise SSD (Mamba-2) selective scan (``ssd.py:344-362``).

    Args:
        u:      [B, L, H, Dh] input projected to heads x channels
        delta:  [B, L, H]     per-token, per-head step size (>= 0)
        B:      [B, L, H, N]  input projection
        C:      [B, L, H, N]  output projection
        A_neg:  [H, N]        decay rates (negative)
        seg:    checkpoint segment length (L % seg == 0; default 32)
        h0:     optional initial state [B, H, Dh, N] (the final state's layout;
                differentiable). Not in the reference, which starts from zero.

    Returns:
        y:      [B, L, H, Dh] float32
    """
    y, _ = _SSDScan.apply(u, delta, B, C, A_neg, seg, h0, False)
    return y


def ssd_scan_with_state(u, delta, B, C, A_neg, seg=DEFAULT_SEG, h0=None):
    """SSD scan that also returns the final state ``[B, H, Dh, N]`` (``ssd.py:365-375``).
    Passing it back as ``h0`` continues the scan (chunked prefill)."""
    return _SSDScan.apply(u, delta, B, C, A_neg, seg, h0, True)


def ssd_scan_reference(u, delta, B, C, A_neg, h0=None):
    """Per-step torch loop (``ssd.py:382-394``). Differentiable, any device."""
    Bt, L, H, Dh = u.shape
    N = A_neg.shape[-1]
    ft = torch.promote_types(u.dtype, torch.float32)
    h = torch.zeros((Bt, H, Dh, N), dtype=ft, device=u.device) if h0 is None else h0.to(ft)
    ys = []
    for t in range(L):
        dt = delta[:, t, :, None, None]
        decay = torch.exp(dt * A_neg[None, :, None, :])
        inp = dt * B[:, t, :, None, :] * u[:, t, :, :, None]
        h = decay * h + inp
        ys.append(torch.sum(h * C[:, t, :, None, :], dim=-1))
    return torch.stack(ys, dim=1)


def ssd_step(u, delta, B, C, A_neg, state):
    """One decode step (no counterpart in the reference, where a step is a scan
    of length 1): advances ``state`` [B, H, Dh, N] (float32, the final state's
    layout) in place by one step of ``ssd.py:382-394`` and returns y [B, H, Dh]
    float32. ``u`` [B, H, Dh], ``delta`` [B, H], ``B``/``C`` [B, H, N], ``A_neg``
    [H, N]. Not differentiable."""
    if u.dim() != 3:
        raise ValueError(f"u must be [B, H, Dh], got shape {tuple(u.shape)}")
    Bt, H, Dh = u.shape
    if A_neg.dim() != 2 or A_neg.shape[0] != H:
        raise ValueError(f"A_neg must be [H, N] = [{H}, N], got {tuple(A_neg.shape)}")
    N = A_neg.shape[1]
    if tuple(delta.shape) != (Bt, H):
        raise ValueError(f"delta must be [B, H] = [{Bt}, {H}], got {tuple(delta.shape)}")
    for name, t in (("B", B), ("C", C)):
        if tuple(t.shape) != (Bt, H, N):
            raise ValueError(f"{name} must be [B, H, N] = [{Bt}, {H}, {N}], got {tuple(t.shape)}")
    dev = _lib.require_cuda(u, delta, B, C, A_neg, state)
    state = step_state(state, (Bt, H, Dh, N), dev)
    dt = common_dtype(u, delta, B, C)
    u_, d_, B_, C_ = (prep(t.detach(), dt) for t in (u, delta, B, C))
    A32, ash, asn = _a_f32(A_neg.detach())
    y = torch.empty((Bt, H, Dh), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("mr_ssd_step", _lib.ptr(u_), _lib.ptr(d_), _lib.ptr(B_), _lib.ptr(C_), _lib.ptr(A32), ash,
                  asn, _lib.DTYPE_CODE[dt], Bt, H, Dh, N, _lib.ptr(state), _lib.ptr(y), _lib.stream_of(dev))
    return y
