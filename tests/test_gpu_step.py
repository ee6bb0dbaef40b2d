"""One-token decode steps (no counterpart in the reference): the state cache
advanced in place and the step's output, against one step of the oracle's
recurrence started from that state, and a run of steps against the scan.
Tolerances as the parity tests (max|diff| / max|ref|): 1e-5 for float32
inputs, 2e-2 for bfloat16."""

import importlib

import numpy as np
import pytest
import torch

from oracle import ref_loops as R

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _mr():
    return importlib.import_module("mlx-recurrence_b200")


def _dev_in(x, dtype, dev):
    return torch.tensor(x, dtype=torch.float32).to(dtype).to(dev)


def _rounded(x, dtype):
    return torch.tensor(x, dtype=torch.float32).to(dtype).to(torch.float64).numpy()


def _err(got, ref):
    return R.rel_err(got.double().cpu().numpy(), ref)


def _case(kind, shape, rng):
    """(inputs of one token, state shape, oracle forward on a length-1 scan)"""
    if kind == "ssd":
        Bt, H, Dh, N = shape
        ins = [rng.standard_normal((Bt, H, Dh)), np.abs(rng.standard_normal((Bt, H))) * 0.3 + 0.01,
               rng.standard_normal((Bt, H, N)), rng.standard_normal((Bt, H, N))]
        return ins, (Bt, H, Dh, N)
    if kind == "gla":
        Bt, H, Dh = shape
        ins = [rng.standard_normal((Bt, H, Dh)) for _ in range(3)] + [rng.uniform(0.5, 1.0, (Bt, H))]
        return ins, (Bt, H, Dh, Dh)
    if kind == "rglru":
        Bt, D = shape
        return [rng.uniform(-1, 1, (Bt, D)), rng.standard_normal((Bt, D))], (Bt, D)
    Bt, Dp = shape
    th = rng.uniform(-0.5, 0.5, (Bt, Dp))
    return [rng.uniform(-1, 1, (Bt, Dp)), np.cos(th), np.sin(th), rng.standard_normal((Bt, 2 * Dp))], (Bt, 2 * Dp)


def _oracle_step(kind, ins_r, state, A=None):
    one = [x[:, None] for x in ins_r]  # a time axis of length 1
    if kind == "ssd":
        y, fin = R.ssd_forward(*one, A, h0=state)
    else:
        y, fin = {"gla": R.gla_forward, "rglru": R.rglru_forward, "rotlru": R.rotlru_forward}[kind](*one, h0=state)
    return y[:, 0], fin


@pytest.mark.parametrize("kind,shape,dtype,per_head", [
    ("ssd", (3, 2, 64, 128), torch.float32, True),
    ("ssd", (2, 3, 32, 16), torch.bfloat16, False),
    ("ssd", (2, 2, 96, 72), torch.float32, False),
    ("gla", (3, 2, 64), torch.float32, None),
    ("gla", (2, 2, 128), torch.bfloat16, None),
    ("gla", (2, 3, 32), torch.float32, None),
    ("rglru", (3, 96), torch.float32, None),
    ("rglru", (5, 2560), torch.bfloat16, None),
    ("rotlru", (3, 48), torch.float32, None),
    ("rotlru", (4, 1024), torch.bfloat16, None),
])
def test_step_matches_oracle(cuda_dev, kind, shape, dtype, per_head):
    mr = _mr()
    rng = np.random.default_rng(sum(shape))
    ins, sshape = _case(kind, shape, rng)
    state0 = rng.standard_normal(sshape)
    state = torch.tensor(state0, dtype=torch.float32, device=cuda_dev)
    args = [_dev_in(x, dtype, cuda_dev) for x in ins]
    A = None
    if kind == "ssd":
        H, N = shape[1], shape[3]
        if per_head:
            a_h = -np.abs(rng.standard_normal(H)) - 0.1
            A = np.repeat(a_h[:, None], N, axis=1)
            args.append(torch.tensor(a_h, dtype=torch.float32, device=cuda_dev)[:, None].expand(H, N))
        else:
            A = -np.abs(rng.standard_normal((H, N))) - 0.1
            args.append(torch.tensor(A, dtype=torch.float32, device=cuda_dev))
    y = getattr(mr, f"{kind}_step")(*args, state)
    torch.cuda.synchronize()
    y_ref, s_ref = _oracle_step(kind, [_rounded(x, dtype) for x in ins], state0, A)
    tol = TOL[dtype]
    assert _err(y, y_ref) <= tol
    assert _err(state, s_ref) <= tol


@pytest.mark.parametrize("kind", ["ssd", "gla", "rglru", "rotlru"])
def test_steps_reproduce_the_scan(cuda_dev, kind):
    """Thirty-two decode steps from a zero state give the scan's outputs and final state."""
    mr = _mr()
    rng = np.random.default_rng(7)
    T = 32
    if kind == "ssd":
        Bt, H, Dh, N = 2, 2, 64, 128
        seq = [rng.standard_normal((Bt, T, H, Dh)), np.abs(rng.standard_normal((Bt, T, H))) * 0.1 + 0.01,
               rng.standard_normal((Bt, T, H, N)), rng.standard_normal((Bt, T, H, N))]
        extra = [torch.tensor(-np.abs(rng.standard_normal((H, N))) - 0.1, dtype=torch.float32, device=cuda_dev)]
        sshape = (Bt, H, Dh, N)
    elif kind == "gla":
        Bt, H, Dh = 2, 2, 64
        seq = [rng.standard_normal((Bt, T, H, Dh)) / 8 for _ in range(3)] + [rng.uniform(0.8, 1.0, (Bt, T, H))]
        extra, sshape = [], (Bt, H, Dh, Dh)
    elif kind == "rglru":
        seq = [rng.uniform(0.5, 0.99, (2, T, 64)), rng.standard_normal((2, T, 64))]
        extra, sshape = [], (2, 64)
    else:
        th = rng.uniform(-0.2, 0.2, (2, T, 32))
        seq = [rng.uniform(0.5, 0.99, (2, T, 32)), np.cos(th), np.sin(th), rng.standard_normal((2, T, 64))]
        extra, sshape = [], (2, 64)
    ts = [torch.tensor(x, dtype=torch.float32, device=cuda_dev) for x in seq]
    y_scan, fin = getattr(mr, f"{kind}_scan_with_state")(*ts, *extra, seg=T)
    state = torch.zeros(sshape, dtype=torch.float32, device=cuda_dev)
    step = getattr(mr, f"{kind}_step")
    ys = [step(*(t[:, i] for t in ts), *extra, state) for i in range(T)]
    y_steps = torch.stack(ys, dim=1)
    assert _err(y_steps, y_scan.double().cpu().numpy()) <= 1e-5
    assert _err(state, fin.double().cpu().numpy()) <= 1e-5


def test_step_state_must_be_float32_contiguous(cuda_dev):
    mr = _mr()
    a = torch.rand(2, 64, device=cuda_dev)
    with pytest.raises(ValueError, match="contiguous float32"):
        mr.rglru_step(a, a, torch.zeros(2, 64, device=cuda_dev, dtype=torch.float64))
    with pytest.raises(ValueError, match="final state's shape"):
        mr.rglru_step(a, a, torch.zeros(2, 32, device=cuda_dev))
