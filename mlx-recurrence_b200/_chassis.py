"""Shared host-side machinery of the scan plug-ins (mirror of
``mlx_recurrence/_chassis.py``): default segment length, shape validation
with the reference's messages, the library handle, input preparation and the
forward + all-gradient parity helper.
"""

from __future__ import annotations

import torch

from . import _lib

# Segment length of the checkpoint/recompute pattern (_chassis.py:51).
DEFAULT_SEG = 32

# Lane-dimension granularity the reference's shape rule enforces (_chassis.py:55).
SIMD_WIDTH = 32


def get_or_build_kernel(name=None, *args, **kwargs):
    """Return the loaded ``libmlrec.so`` handle.

    The reference JIT-compiles one Metal kernel per shape name
    (``_chassis.py:62-85``). Here every kernel is compiled ahead of time for
    sm_100a into one C-ABI library, so there is nothing to build per shape;
    the arguments are accepted for signature compatibility and ignored.
    """
    return _lib.load()


def check_segment_shape(L, seg, lane_dim, lane_name="lane dimension"):
    """Raise ValueError unless seg > 0, L % seg == 0 and lane_dim % 32 == 0.

    Same rules and messages as ``mlx_recurrence/_chassis.py:92-115``.
    """
    if seg <= 0:
        raise ValueError(f"seg must be positive, got {seg}")
    if L % seg != 0:
        raise ValueError(
            f"sequence length L={L} must be divisible by seg={seg} "
            f"(segment-checkpoint pattern tiles L into L/seg segments)"
        )
    if lane_dim % SIMD_WIDTH != 0:
        raise ValueError(
            f"{lane_name}={lane_dim} must be a multiple of {SIMD_WIDTH} "
            f"(fused gradient reductions use {SIMD_WIDTH}-lane simdgroups)"
        )


def common_dtype(*tensors):
    """The element type the kernels read: float32, bfloat16 or float16.

    Mixed inputs are promoted (float64 computes as float32, as in the
    reference, whose kernels read every input as float).
    """
    dt = tensors[0].dtype
    for t in tensors[1:]:
        dt = torch.promote_types(dt, t.dtype)
    if dt not in _lib.DTYPE_CODE:
        dt = torch.float32
    return dt


def prep(t, dtype):
    """Contiguous, in the kernel element type."""
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


def prep_h0(h0, shape, device):
    """Initial state as float32 contiguous on ``device`` (None stays None).

    ``shape`` is the final state's shape: a returned final state can be passed
    back as ``h0`` to continue a scan (no counterpart in the reference, which
    always starts from zero, ``ssd.py:365-375``)."""
    if h0 is None:
        return None
    if tuple(h0.shape) != tuple(shape):
        raise ValueError(f"h0 must have the final state's shape {tuple(shape)}, got {tuple(h0.shape)}")
    if h0.device != device:
        raise ValueError(f"h0 must be on {device}, got {h0.device}")
    return h0.to(torch.float32).contiguous()


def step_state(state, shape, device):
    """The decode-step state cache: float32, contiguous, on ``device``, in the
    final state's ``shape`` (it is advanced in place, so it is not copied)."""
    if tuple(state.shape) != tuple(shape):
        raise ValueError(f"state must have the final state's shape {tuple(shape)}, got {tuple(state.shape)}")
    if state.dtype != torch.float32 or not state.is_contiguous() or state.device != device:
        raise ValueError("state must be a contiguous float32 tensor on the inputs' device (updated in place)")
    return state


def grad_out(g, shape, device):
    """fp32 contiguous cotangent (zeros when autograd passes None)."""
    if g is None:
        return torch.zeros(shape, dtype=torch.float32, device=device)
    return g.to(torch.float32).contiguous()


def parity_check(
    kernel_fn,
    reference_fn,
    inputs,
    arg_names,
    grad_argnums,
    *,
    w_out=None,
    y_tol=1e-3,
    grad_rtol=1e-3,
    label="",
    verbose=True,
):
    """Compare a kernel with a reference: forward output and every gradient.

    Mirror of ``mlx_recurrence/_chassis.py:122-213`` for torch. The loss is
    ``sum(y * w_out)`` with ``w_out ~ N(0, 1)`` from a generator seeded 1234
    (drawn on the CPU so it is device independent). Forward passes when
    ``max|y_k - y_r| < y_tol``; each gradient passes when
    ``max|g_k - g_r| / (max|g_r| + 1e-8) < grad_rtol``.

    Returns ``(ok, report)`` with ``report[name] = {"abs": .., "rel": ..}``.
    """
    inputs = list(inputs)
    with torch.no_grad():
        y_k = kernel_fn(*inputs)
        y_r = reference_fn(*inputs)
    if w_out is None:
        g = torch.Generator().manual_seed(1234)
        w_out = torch.randn(tuple(y_r.shape), generator=g, dtype=torch.float32).to(y_r.device)

    report = {}
    y_abs = float((y_k.double() - y_r.double()).abs().max())
    y_scale = float(y_r.double().abs().max()) + 1e-8
    report["y"] = {"abs": y_abs, "rel": y_abs / y_scale}
    ok = y_abs < y_tol

    def grads(fn):
        args = [x.detach().clone().requires_grad_(i in grad_argnums) if isinstance(x, torch.Tensor)
                else x for i, x in enumerate(inputs)]
        loss = (fn(*args).float() * w_out.float()).sum()
        return torch.autograd.grad(loss, [args[i] for i in grad_argnums])

    g_k = grads(kernel_fn)
    g_r = grads(reference_fn)
    names = [arg_names[i] for i in grad_argnums]
    for name, gk, gr in zip(names, g_k, g_r):
        a = float((gk.double() - gr.double()).abs().max())
        s = float(gr.double().abs().max()) + 1e-8
        report[f"grad_{name}"] = {"abs": a, "rel": a / s}
        ok = ok and (a / s < grad_rtol)

    if verbose:
        prefix = f"{label}  " if label else ""
        print(f"{prefix}y          max|diff| = {y_abs:.2e}  (rel {report['y']['rel']:.2e})")
        for name in names:
            r = report[f"grad_{name}"]
            print(f"{prefix}grad_{name:<8} max|diff| = {r['abs']:.2e}  (rel {r['rel']:.2e})")
        print(f"{prefix}-> {'PASS' if ok else 'FAIL'}")
    return ok, report
