"""SSD with a dense A_neg [H, N] (one decay rate per head and state column, the
reference's general contract, ssd.py:62, 96) on the tensor-core path: bf16/fp16,
Dh = 64, N = 128, L a multiple of 128. Forward, final state and every gradient
(grad_A per (head, column)) against the float64 oracle at 2e-2 (max|diff| /
max|ref|). Units whose chunks decay beyond the path's exponent range are
recomputed by the per-step kernels, which the strong-decay cases exercise."""

import importlib
import os

import numpy as np
import pytest
import torch

import _cases as K
import ref_loops as R

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _lib():
    L = importlib.import_module("mlx-recurrence_b200._lib")
    return L, L.load()


def _run(mr, ins, dtype, dev, w, wf=None, h0=None):
    ts = [torch.tensor(x, dtype=torch.float32).to(dtype).to(dev).requires_grad_(True) for x in ins[:4]]
    A = torch.tensor(ins[4], dtype=torch.float32, device=dev, requires_grad=True)
    leaves = ts + [A]
    h0_t = None
    if h0 is not None:
        h0_t = torch.tensor(h0, dtype=torch.float32, device=dev, requires_grad=True)
        leaves.append(h0_t)
    y, fin = mr.ssd_scan_with_state(*ts, A, seg=32, h0=h0_t)
    loss = (y * torch.tensor(w, dtype=torch.float32, device=dev)).sum()
    if wf is not None:
        loss = loss + (fin * torch.tensor(wf, dtype=torch.float32, device=dev)).sum()
    grads = torch.autograd.grad(loss, leaves)
    rounded = [t.detach().double().cpu().numpy() for t in ts] + [np.asarray(ins[4], dtype=np.float64)]
    out = lambda t: t.detach().double().cpu().numpy()
    return out(y), out(fin), [out(g) for g in grads], rounded


def _check(y, fin, grads, rounded, w, wf=None, h0=None):
    yo, fo = R.ssd_forward(*rounded, h0=h0)
    ref = R.ssd_backward(*rounded, w, wf, h0=h0)
    assert K.rel_err(y, yo) < TOL, f"y: {K.rel_err(y, yo):.2e}"
    assert K.rel_err(fin, fo) < TOL, f"final: {K.rel_err(fin, fo):.2e}"
    for n, g, r in zip(("u", "delta", "B", "C", "A_neg", "h0"), grads, ref):
        err = K.rel_err(g, r)
        assert err < TOL, f"grad_{n}: {err:.2e}"


def _inputs(Bt, L, H, seed, dt_scale=0.1, a_scale=0.5):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((Bt, L, H, 64)), np.abs(rng.standard_normal((Bt, L, H))) * dt_scale + 0.01,
            rng.standard_normal((Bt, L, H, 128)), rng.standard_normal((Bt, L, H, 128)),
            -np.exp(rng.standard_normal((H, 128)) * a_scale)]


def test_dense_path_is_taken_for_the_shapes():
    L, lib = _lib()
    assert lib.mr_ssd_preferred_seg(L.MR_BF16, 512, 64, 128, 32, 1) == 128
    assert lib.mr_ssd_preferred_seg(L.MR_F32, 512, 64, 128, 32, 1) == 32  # float32: the per-step kernels


def test_golden_dense_case_from_the_reference(mr, cuda_dev):
    """The reference's own input maker with its own dense A_neg (tests/test_v2_ssd.py:15-23)
    at L=256, Dh=64, N=128, bf16-representable inputs; the reference's pure loop's outputs."""
    case = K.load(os.path.join(K.GOLDEN, "ssd_tc_dense_parity_widened.npz"))
    ins, names = K.inputs_of(case)
    assert not np.all(ins[4] == ins[4][:, :1])  # a genuinely dense A_neg
    ts = [torch.tensor(x, dtype=torch.float32).to(torch.bfloat16).to(cuda_dev).requires_grad_(True) for x in ins[:4]]
    for t, x in zip(ts, ins):
        assert np.array_equal(t.detach().double().cpu().numpy(), x)
    A = torch.tensor(ins[4], dtype=torch.float32, device=cuda_dev, requires_grad=True)
    y = mr.ssd_scan(*ts, A, seg=32)
    w = torch.tensor(case["w_out"], dtype=torch.float32, device=cuda_dev)
    grads = torch.autograd.grad((y * w).sum(), ts + [A])
    assert K.rel_err(y.detach().double().cpu().numpy(), case["y"]) < TOL, "y"
    for n, g in zip(names, grads):
        err = K.rel_err(g.double().cpu().numpy(), case["grad_" + n])
        assert err < TOL, f"grad_{n}: {err:.2e}"


@pytest.mark.parametrize("Bt,L,H,dtype", [
    (2, 512, 3, torch.bfloat16),
    (1, 256, 2, torch.float16),
    (1, 1024, 16, torch.bfloat16),  # H % 8 == 0: delta arrives by TMA
])
def test_dense_matches_oracle(mr, cuda_dev, Bt, L, H, dtype):
    ins = _inputs(Bt, L, H, seed=L + H)
    rng = np.random.default_rng(1)
    w = rng.standard_normal((Bt, L, H, 64))
    wf = rng.standard_normal((Bt, H, 64, 128))
    y, fin, grads, rounded = _run(mr, ins, dtype, cuda_dev, w, wf)
    _check(y, fin, grads, rounded, w, wf)


def test_dense_with_initial_state(mr, cuda_dev):
    ins = _inputs(2, 384, 2, seed=9)
    rng = np.random.default_rng(2)
    w = rng.standard_normal((2, 384, 2, 64))
    wf = rng.standard_normal((2, 2, 64, 128))
    h0 = rng.standard_normal((2, 2, 64, 128))
    y, fin, grads, rounded = _run(mr, ins, torch.bfloat16, cuda_dev, w, wf, h0=h0)
    _check(y, fin, grads, rounded, w, wf, h0=h0)


@pytest.mark.parametrize("mode", ["all", "some"])
def test_dense_strong_decay_falls_back_per_unit(mr, cuda_dev, mode):
    """Decays beyond the operand factors' range (max_n |a_n| |D_t - c| > 80 within a chunk)
    send the unit to the per-step kernels; with 'some', only batch row 1 does, so the
    tensor-core results of row 0 and the per-step results of row 1 meet in one call."""
    ins = _inputs(2, 256, 3, seed=4, dt_scale=0.1, a_scale=0.3)
    if mode == "all":
        ins[1] = ins[1] * 20.0
    else:
        ins[1][1] = ins[1][1] * 20.0
    rng = np.random.default_rng(3)
    w = rng.standard_normal((2, 256, 3, 64))
    wf = rng.standard_normal((2, 3, 64, 128))
    y, fin, grads, rounded = _run(mr, ins, torch.bfloat16, cuda_dev, w, wf)
    _check(y, fin, grads, rounded, w, wf)
