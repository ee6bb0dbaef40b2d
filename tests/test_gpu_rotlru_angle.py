"""rotLRU taking the rotation angle (rotlru_scan_angle; the reference's callers
form cos and sin in host code, rotlru.py:18-22): forward, final state and the
gradients of a, theta, x (and h0) against the oracle, and against autograd
through the unfused composition (cos, sin formed in torch, then rotlru_scan).
Tolerances (max|diff| / max|ref|): 1e-5 for float32 inputs, 2e-2 for
bfloat16 and float16."""

import importlib

import numpy as np
import pytest
import torch

from oracle import ref_loops as R

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _mr():
    return importlib.import_module("mlx-recurrence_b200")


def _inputs(Bt, L, Dp, seed, span=3.0):
    rng = np.random.default_rng(seed)
    a = rng.uniform(0.5, 0.99, (Bt, L, Dp))
    th = rng.uniform(-span, span, (Bt, L, Dp))
    x = rng.standard_normal((Bt, L, 2 * Dp))
    return a, th, x


def _rounded(x, dtype):
    return torch.tensor(x, dtype=torch.float32).to(dtype).to(torch.float64).numpy()


def _err(got, ref):
    return R.rel_err(got.detach().double().cpu().numpy(), ref)


@pytest.mark.parametrize("Bt,L,Dp,seg,dtype,with_h0", [
    (2, 256, 32, 32, torch.float32, False),
    (2, 512, 48, 256, torch.float32, True),    # segments longer than a block
    (3, 384, 64, 128, torch.bfloat16, True),
    (1, 2048, 160, 64, torch.bfloat16, False),  # a ragged channel tile
    (2, 256, 64, 32, torch.float16, True),
])
def test_angle_matches_oracle(cuda_dev, Bt, L, Dp, seg, dtype, with_h0):
    mr = _mr()
    a, th, x = _inputs(Bt, L, Dp, seed=L + Dp)
    rng = np.random.default_rng(2)
    w = rng.standard_normal((Bt, L, 2 * Dp))
    wf = rng.standard_normal((Bt, 2 * Dp))
    h0 = rng.standard_normal((Bt, 2 * Dp)) if with_h0 else None
    ts = [torch.tensor(v, dtype=torch.float32).to(dtype).to(cuda_dev).requires_grad_(True) for v in (a, th, x)]
    h0_t = None if h0 is None else torch.tensor(h0, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    y, fin = mr.rotlru_scan_angle_with_state(*ts, seg=seg, h0=h0_t)
    loss = (y * torch.tensor(w, dtype=torch.float32, device=cuda_dev)).sum() + \
        (fin * torch.tensor(wf, dtype=torch.float32, device=cuda_dev)).sum()
    loss.backward()
    ar, thr, xr = (_rounded(v, dtype) for v in (a, th, x))
    y_ref, f_ref = R.rotlru_angle_forward(ar, thr, xr, h0=h0)
    grads = R.rotlru_angle_backward(ar, thr, xr, w, wf, h0=h0)
    tol = TOL[dtype]
    assert _err(y, y_ref) <= tol
    assert _err(fin, f_ref) <= tol
    for name, got, ref in zip(("a", "theta", "x"), [t.grad for t in ts], grads[:3]):
        assert _err(got, ref) <= tol, name
    if with_h0:
        assert _err(h0_t.grad, grads[3]) <= tol


def test_angle_equals_unfused_composition(cuda_dev):
    """The fused kernels against autograd through cos, sin formed in torch and
    the plain scan (float32, both on the GPU)."""
    mr = _mr()
    Bt, L, Dp = 2, 1024, 64
    a, th, x = _inputs(Bt, L, Dp, seed=4)
    mk = lambda v: torch.tensor(v, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    gy = torch.randn(Bt, L, 2 * Dp, device=cuda_dev, generator=torch.Generator(device=cuda_dev).manual_seed(0))
    a1, t1, x1 = mk(a), mk(th), mk(x)
    y1 = mr.rotlru_scan_angle(a1, t1, x1, seg=64)
    (y1 * gy).sum().backward()
    a2, t2, x2 = mk(a), mk(th), mk(x)
    y2 = mr.rotlru_scan(a2, torch.cos(t2), torch.sin(t2), x2, seg=64)
    (y2 * gy).sum().backward()
    for name, f, u in zip(("y", "a", "theta", "x"), (y1, a1.grad, t1.grad, x1.grad),
                          (y2, a2.grad, t2.grad, x2.grad)):
        assert _err(f, u.detach().double().cpu().numpy()) <= 1e-5, name


def test_angle_shape_is_checked(cuda_dev):
    mr = _mr()
    a = torch.rand(1, 64, 16, device=cuda_dev)
    with pytest.raises(ValueError, match="a/theta shapes must match"):
        mr.rotlru_scan_angle(a, a[:, :, :8], torch.rand(1, 64, 32, device=cuda_dev))


def test_angle_cos_sin_accuracy(cuda_dev):
    """The kernels' cos and sin of the angle: with a = 1, x = 0 and h0 = (1, 0)
    per pair, step 0 returns (cos theta, sin theta). Against float64 over a
    dense grid, random angles up to the reduction's limit, the boundaries of
    the quadrants, arguments beyond the limit (computed out of line), and
    non-finite angles (NaN out)."""
    mr = _mr()
    Bt, L, Dp = 16, 64, 8192
    rng = np.random.default_rng(0)
    n = Bt * Dp
    half_pi = np.pi / 2
    specials = np.concatenate([
        [0.0, -0.0, 1e-30, np.pi, -np.pi, 2e5, 2.1e5, -3e5, 1e6, 1e20, 3.4e38, -3.4e38],
        (np.arange(-40, 41) + 0.5) * half_pi,              # quadrant boundaries
        np.nextafter(np.float32((np.arange(-40, 41) + 0.5) * half_pi), np.float32(np.inf)),
    ]).astype(np.float32)
    th0 = np.concatenate([
        specials,
        np.linspace(-60.0, 60.0, n // 2, dtype=np.float32),
        rng.uniform(-2.05e5, 2.05e5, n).astype(np.float32),
    ])[:n]
    th = np.zeros((Bt, L, Dp), dtype=np.float32)
    th[:, 0, :] = th0.reshape(Bt, Dp)
    dev_f = dict(dtype=torch.float32, device=cuda_dev)
    a = torch.ones((Bt, L, Dp), **dev_f)
    x = torch.zeros((Bt, L, 2 * Dp), **dev_f)
    h0 = torch.zeros((Bt, Dp, 2), **dev_f)
    h0[..., 0] = 1.0
    y = mr.rotlru_scan_angle(a, torch.tensor(th, device=cuda_dev), x, seg=64, h0=h0.reshape(Bt, 2 * Dp))
    got = y[:, 0].reshape(Bt, Dp, 2).double().cpu().numpy().reshape(-1, 2)
    t64 = th0.astype(np.float64)
    assert np.max(np.abs(got[:, 0] - np.cos(t64))) <= 1.5e-7
    assert np.max(np.abs(got[:, 1] - np.sin(t64))) <= 1.5e-7
    bad = np.array([np.inf, -np.inf, np.nan], dtype=np.float32)
    th[0, 0, :3] = bad
    y = mr.rotlru_scan_angle(a, torch.tensor(th, device=cuda_dev), x, seg=64, h0=h0.reshape(Bt, 2 * Dp))
    assert torch.isnan(y[0, 0, :6]).all()
