"""Initial state h0 (no counterpart in the reference): forward, final state and
every gradient, h0's included, against the oracle, on each kernel path —
per-step (float32), tensor-core chunks (bf16, SSD/GLA), diagonal scans
(RG-LRU/rotLRU, with segments shorter and longer than a block) — and the
chunked-prefill property (a scan continued from a returned final state equals
the whole scan). Tolerances as the parity tests: max|diff| / max|ref| within
1e-5 for float32 inputs, 2e-2 for bfloat16."""

import importlib

import numpy as np
import pytest
import torch

from oracle import ref_loops as R

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _mr():
    return importlib.import_module("mlx-recurrence_b200")


def _rounded(x, dtype):
    """The values the kernels read: x rounded to dtype, as float64."""
    return torch.tensor(x, dtype=torch.float32).to(dtype).to(torch.float64).numpy()


def _check(got, ref, tol, what):
    err = R.rel_err(got.detach().double().cpu().numpy(), ref)
    assert err <= tol, f"{what}: rel err {err:.3e} > {tol}"


def _inputs(kind, shape, seed):
    rng = np.random.default_rng(seed)
    if kind == "ssd":
        Bt, L, H, Dh, N = shape
        ins = [rng.standard_normal((Bt, L, H, Dh)), np.abs(rng.standard_normal((Bt, L, H))) * 0.1 + 0.01,
               rng.standard_normal((Bt, L, H, N)), rng.standard_normal((Bt, L, H, N))]
        A = -np.abs(rng.standard_normal(H)) - 0.1
        return ins, A, (Bt, H, Dh, N), (Bt, L, H, Dh)
    if kind == "gla":
        Bt, L, H, Dh = shape
        ins = [rng.standard_normal((Bt, L, H, Dh)) / 8 for _ in range(3)]
        ins.append(1.0 / (1.0 + np.exp(-(rng.standard_normal((Bt, L, H)) + 2.0))))
        return ins, None, (Bt, H, Dh, Dh), (Bt, L, H, Dh)
    if kind == "rglru":
        Bt, L, D = shape
        return [rng.uniform(0.5, 0.99, (Bt, L, D)), rng.standard_normal((Bt, L, D))], None, (Bt, D), (Bt, L, D)
    Bt, L, Dp = shape
    th = rng.uniform(-0.2, 0.2, (Bt, L, Dp))
    ins = [rng.uniform(0.5, 0.99, (Bt, L, Dp)), np.cos(th), np.sin(th), rng.standard_normal((Bt, L, 2 * Dp))]
    return ins, None, (Bt, 2 * Dp), (Bt, L, 2 * Dp)


def _run(kind, shape, seg, dtype, dev, seed):
    mr = _mr()
    ins, A, fshape, yshape = _inputs(kind, shape, seed)
    rng = np.random.default_rng(seed + 1)
    h0 = rng.standard_normal(fshape)
    w = rng.standard_normal(yshape)
    wf = rng.standard_normal(fshape)
    ts = [torch.tensor(x, dtype=torch.float32).to(dtype).to(dev).requires_grad_(True) for x in ins]
    h0_t = torch.tensor(h0, dtype=torch.float32, device=dev).requires_grad_(True)
    args = list(ts)
    if kind == "ssd":
        A_h = torch.tensor(A, dtype=torch.float32, device=dev).requires_grad_(True)
        N = shape[-1]
        # per-head rates as a stride-0 view: the tensor-core path for bf16, Dh=64, N=128
        args.append(A_h[:, None].expand(len(A), N))
    fn = getattr(mr, f"{kind}_scan_with_state")
    y, fin = fn(*args, seg=seg, h0=h0_t)
    loss = (y * torch.tensor(w, dtype=torch.float32, device=dev)).sum() + \
        (fin * torch.tensor(wf, dtype=torch.float32, device=dev)).sum()
    loss.backward()
    ins_r = [_rounded(x, dtype) for x in ins]
    tol = TOL[dtype]
    if kind == "ssd":
        A_r = np.repeat(A[:, None], shape[-1], axis=1)
        y_ref, f_ref = R.ssd_forward(*ins_r, A_r, h0=h0)
        grads = R.ssd_backward(*ins_r, A_r, w, wf, h0=h0)
        got = [t.grad for t in ts] + [A_h.grad]
        ref = list(grads[:4]) + [grads[4].sum(axis=1)]
    else:
        fwd, bwd = {"gla": (R.gla_forward, R.gla_backward), "rglru": (R.rglru_forward, R.rglru_backward),
                    "rotlru": (R.rotlru_forward, R.rotlru_backward)}[kind]
        y_ref, f_ref = fwd(*ins_r, h0=h0)
        grads = bwd(*ins_r, w, wf, h0=h0)
        got = [t.grad for t in ts]
        ref = list(grads[:-1])
    _check(y, y_ref, tol, f"{kind} y")
    _check(fin, f_ref, tol, f"{kind} final")
    for i, (g, r) in enumerate(zip(got, ref)):
        _check(g, r, tol, f"{kind} grad {i}")
    _check(h0_t.grad, grads[-1], tol, f"{kind} grad h0")


@pytest.mark.parametrize("kind,shape,seg,dtype", [
    ("ssd", (2, 64, 2, 32, 16), 16, torch.float32),          # per-step kernels
    ("ssd", (1, 256, 2, 64, 128), 32, torch.bfloat16),       # tensor-core chunks
    ("gla", (2, 64, 2, 32), 16, torch.float32),
    ("gla", (1, 256, 2, 64), 32, torch.bfloat16),
    ("rglru", (2, 256, 64), 32, torch.float32),
    ("rglru", (2, 512, 96), 256, torch.bfloat16),            # segments longer than a block
    ("rotlru", (2, 256, 32), 32, torch.float32),
    ("rotlru", (2, 256, 48), 128, torch.bfloat16),
])
def test_initial_state_matches_oracle(cuda_dev, kind, shape, seg, dtype):
    _run(kind, shape, seg, dtype, cuda_dev, seed=sum(map(ord, kind)) + seg)


@pytest.mark.parametrize("kind,shape,dtype", [
    ("ssd", (1, 512, 2, 64, 128), torch.bfloat16),
    ("gla", (1, 512, 2, 64), torch.bfloat16),
    ("rglru", (2, 512, 64), torch.float32),
    ("rotlru", (2, 512, 32), torch.float32),
])
def test_chunked_prefill_continues_the_scan(cuda_dev, kind, shape, dtype):
    """scan(x) == scan(x[:, cut:], h0=final(scan(x[:, :cut]))) on the GPU."""
    mr = _mr()
    ins, A, _, _ = _inputs(kind, shape, seed=5)
    ts = [torch.tensor(x, dtype=torch.float32).to(dtype).to(cuda_dev) for x in ins]
    extra = []
    if kind == "ssd":
        extra = [torch.tensor(A, dtype=torch.float32, device=cuda_dev)[:, None].expand(len(A), shape[-1])]
    fn = getattr(mr, f"{kind}_scan_with_state")
    cut = 256
    y, fin = fn(*ts, *extra)
    y1, f1 = fn(*(t[:, :cut] for t in ts), *extra)
    y2, f2 = fn(*(t[:, cut:] for t in ts), *extra, h0=f1)
    tol = TOL[dtype]
    _check(torch.cat([y1, y2], dim=1), y.double().cpu().numpy(), tol, f"{kind} y")
    _check(f2, fin.double().cpu().numpy(), tol, f"{kind} final")


def test_h0_shape_is_checked(cuda_dev):
    mr = _mr()
    a = torch.rand(1, 64, 32, device=cuda_dev)
    with pytest.raises(ValueError, match="h0 must have the final state's shape"):
        mr.rglru_scan(a, a, h0=torch.zeros(1, 31, device=cuda_dev))
