"""torch-float64 stand-in for the subset of ``mlx.core`` the reference's
v2 pure-loop functions, tests and ``parity_check`` use (golden generation only).

Random draws are rounded to float32 (MLX's default dtype) and then held in
float64, so every array op the reference's loops perform runs in float64.
The RNG is torch's CPU generator, so values differ from MLX's stream; only the
distributions and shapes follow the reference's tests.
"""

from __future__ import annotations

import types

import torch

float32 = torch.float32
float64 = torch.float64
bfloat16 = torch.bfloat16
array = torch.Tensor

_gen = torch.Generator().manual_seed(0)


def _shape(shape):
    if isinstance(shape, int):
        return (shape,)
    return tuple(shape)


def _seed(s):
    _gen.manual_seed(int(s))


def _normal(shape=(), *args, **kw):
    return torch.randn(_shape(shape), generator=_gen, dtype=torch.float32).double()


def _uniform(low=0.0, high=1.0, shape=(), *args, **kw):
    r = torch.rand(_shape(shape), generator=_gen, dtype=torch.float32)
    return (low + (high - low) * r).float().double()


random = types.SimpleNamespace(seed=_seed, normal=_normal, uniform=_uniform)


def zeros(shape, dtype=None):
    return torch.zeros(_shape(shape), dtype=torch.float64)


def ones(shape, dtype=None):
    return torch.ones(_shape(shape), dtype=torch.float64)


exp = torch.exp
abs = torch.abs
sigmoid = torch.sigmoid
cos = torch.cos
sin = torch.sin
sqrt = torch.sqrt


def sum(x, axis=None, keepdims=False):
    if axis is None:
        return torch.sum(x)
    return torch.sum(x, dim=axis, keepdim=keepdims)


def max(x, axis=None):
    if axis is None:
        return torch.max(x)
    return torch.amax(x, dim=axis)


def stack(xs, axis=0):
    return torch.stack(list(xs), dim=axis)


def concatenate(xs, axis=0):
    return torch.cat(list(xs), dim=axis)


def swapaxes(x, a, b):
    return torch.swapaxes(x, a, b)


def repeat(x, repeats, axis=None):
    return torch.repeat_interleave(x, repeats, dim=axis)


def eval(*args):
    return None


def grad(fn, argnums=0):
    single = isinstance(argnums, int)
    nums = (argnums,) if single else tuple(argnums)

    def g(*args):
        args = [a.detach().clone().requires_grad_(i in nums) if isinstance(a, torch.Tensor) else a
                for i, a in enumerate(args)]
        out = fn(*args)
        gs = torch.autograd.grad(out, [args[i] for i in nums])
        gs = tuple(x.detach() for x in gs)
        return gs[0] if single else gs

    return g


def _unavailable(*a, **k):
    raise RuntimeError("Metal kernels are unavailable in the mlx stand-in")


class custom_function:
    """Decorator placeholder: defining a custom function works, calling it
    (which would launch a Metal kernel) raises."""

    def __init__(self, fn):
        self.fn = fn

    def vjp(self, f):
        return f

    def __call__(self, *a, **k):
        _unavailable()


fast = types.SimpleNamespace(metal_kernel=_unavailable)
