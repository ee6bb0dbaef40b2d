"""RG-LRU with its input gating inside the kernels (rglru_scan_gated; the
reference leaves the gating to host code, rglru.py:8-27): forward, final state
and the gradients of x, r, i, lam (and h0) against the oracle, and against
autograd through the unfused composition (the gates formed in torch, then
rglru_scan). Tolerances (max|diff| / max|ref|): 1e-5 for float32 inputs, 2e-2
for bfloat16 and float16 (1e-2 between the two bf16 computations)."""

import importlib

import numpy as np
import pytest
import torch

from oracle import ref_loops as R

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}
C = 8.0


def _mr():
    return importlib.import_module("mlx-recurrence_b200")


def _inputs(Bt, L, D, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((Bt, L, D))
    r = 1.0 / (1.0 + np.exp(-rng.standard_normal((Bt, L, D))))
    i = 1.0 / (1.0 + np.exp(-rng.standard_normal((Bt, L, D))))
    lam = rng.uniform(2.2, 6.9, D)
    return x, r, i, lam


def _rounded(x, dtype):
    return torch.tensor(x, dtype=torch.float32).to(dtype).to(torch.float64).numpy()


def _err(got, ref):
    return R.rel_err(got.detach().double().cpu().numpy(), ref)


@pytest.mark.parametrize("Bt,L,D,seg,dtype,with_h0", [
    (2, 256, 64, 32, torch.float32, False),
    (2, 512, 96, 256, torch.float32, True),    # segments longer than a block
    (3, 384, 128, 128, torch.bfloat16, True),
    (1, 4096, 256, 64, torch.bfloat16, False),
    (2, 256, 96, 32, torch.float16, True),
])
def test_gated_matches_oracle(cuda_dev, Bt, L, D, seg, dtype, with_h0):
    mr = _mr()
    x, r, i, lam = _inputs(Bt, L, D, seed=L + D)
    rng = np.random.default_rng(1)
    w = rng.standard_normal((Bt, L, D))
    wf = rng.standard_normal((Bt, D))
    h0 = rng.standard_normal((Bt, D)) if with_h0 else None
    ts = [torch.tensor(v, dtype=torch.float32).to(dtype).to(cuda_dev).requires_grad_(True) for v in (x, r, i)]
    lam_t = torch.tensor(lam, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    h0_t = None if h0 is None else torch.tensor(h0, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    y, fin = mr.rglru_scan_gated_with_state(*ts, lam_t, C, seg=seg, h0=h0_t)
    loss = (y * torch.tensor(w, dtype=torch.float32, device=cuda_dev)).sum() + \
        (fin * torch.tensor(wf, dtype=torch.float32, device=cuda_dev)).sum()
    loss.backward()
    xr, rr, ir = (_rounded(v, dtype) for v in (x, r, i))
    y_ref, f_ref = R.rglru_gated_forward(xr, rr, ir, lam, C, h0=h0)
    grads = R.rglru_gated_backward(xr, rr, ir, lam, C, w, wf, h0=h0)
    tol = TOL[dtype]
    assert _err(y, y_ref) <= tol
    assert _err(fin, f_ref) <= tol
    for name, got, ref in zip(("x", "r", "i", "lam"), [t.grad for t in ts] + [lam_t.grad], grads[:4]):
        assert _err(got, ref) <= tol, name
    if with_h0:
        assert _err(h0_t.grad, grads[4]) <= tol


def test_gated_equals_unfused_composition(cuda_dev):
    """The fused kernels against autograd through the gates formed in torch and
    the plain scan (bf16 inputs, both on the GPU)."""
    mr = _mr()
    Bt, L, D = 2, 1024, 128
    x, r, i, lam = _inputs(Bt, L, D, seed=3)
    dtype = torch.bfloat16
    mk = lambda v: torch.tensor(v, dtype=torch.float32).to(dtype).to(cuda_dev).requires_grad_(True)
    xs, rs, is_ = mk(x), mk(r), mk(i)
    lam_t = torch.tensor(lam, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    gy = torch.randn(Bt, L, D, device=cuda_dev, generator=torch.Generator(device=cuda_dev).manual_seed(0))
    y = mr.rglru_scan_gated(xs, rs, is_, lam_t, C, seg=64)
    (y * gy).sum().backward()
    fused = [y.detach(), xs.grad, rs.grad, is_.grad, lam_t.grad]
    xu, ru, iu = mk(x), mk(r), mk(i)
    lam_u = torch.tensor(lam, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    a = torch.exp(C * ru.float() * torch.nn.functional.logsigmoid(lam_u))
    b = torch.sqrt(1 - a * a) * iu.float() * xu.float()
    y2 = mr.rglru_scan(a, b, seg=64)
    (y2 * gy).sum().backward()
    unfused = [y2.detach(), xu.grad, ru.grad, iu.grad, lam_u.grad]
    # both sides round their bf16 gradients once: within a few bf16 steps
    for name, f, u in zip(("y", "x", "r", "i", "lam"), fused, unfused):
        assert _err(f, u.double().cpu().numpy()) <= 1e-2, name
