"""Gated DeltaNet kernels (the reference carries the recurrence as a design
only, docs/DESIGN_gated_deltanet.md): forward, final state and every gradient
(q, k, v, alpha, beta, h0) against the oracle, with segments that are and are
not multiples of the backward's four-step sub-blocks, Dh 32 and 64, float32 and
bfloat16, a final-state cotangent and an initial state; the kernels against
autograd through the plug-in's torch loop on the GPU; the chunked-prefill
property. Tolerances (max|diff| / max|ref|): 1e-5 for float32 inputs, 2e-2 for
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


def _inputs(Bt, L, H, Dh, seed):
    rng = np.random.default_rng(seed)

    def nrm(x):
        return x / np.linalg.norm(x, axis=-1, keepdims=True)
    q = nrm(rng.standard_normal((Bt, L, H, Dh)))
    k = nrm(rng.standard_normal((Bt, L, H, Dh)))
    v = rng.standard_normal((Bt, L, H, Dh))
    al = np.exp(-np.logaddexp(0.0, rng.standard_normal((Bt, L, H)) - 3.0))  # exp(-softplus): (0, 1)
    be = 1.0 / (1.0 + np.exp(-rng.standard_normal((Bt, L, H))))
    return [q, k, v, al, be]


def _rounded(x, dtype):
    return torch.tensor(x, dtype=torch.float32).to(dtype).to(torch.float64).numpy()


def _err(got, ref):
    return R.rel_err(got.detach().double().cpu().numpy(), ref)


@pytest.mark.parametrize("Bt,L,H,Dh,seg,dtype,with_h0,with_gf", [
    (2, 64, 2, 64, 16, torch.float32, False, False),
    (1, 128, 3, 32, 32, torch.float32, True, True),
    (2, 96, 2, 64, 6, torch.float32, True, False),     # sub-blocks of 4 + 2
    (1, 40, 2, 32, 5, torch.float32, False, True),     # sub-blocks of 4 + 1
    (1, 16, 2, 64, 1, torch.float32, True, True),      # one step per segment
    (2, 256, 4, 64, 64, torch.bfloat16, True, True),
    (3, 192, 5, 32, 48, torch.bfloat16, False, False),
    (2, 128, 3, 64, 32, torch.float16, True, True),
    # chunkwise (WY) forward: 2-byte inputs, Dh = 64, L % 128 == 0, seg % 64 == 0
    (2, 512, 3, 64, 128, torch.bfloat16, True, True),
    (1, 384, 2, 64, 64, torch.float16, False, False),
    (2, 128, 2, 64, 128, torch.bfloat16, True, True),     # a single chunk
])
def test_gdn_matches_oracle(cuda_dev, Bt, L, H, Dh, seg, dtype, with_h0, with_gf):
    mr = _mr()
    ins = _inputs(Bt, L, H, Dh, seed=L + Dh + seg)
    rng = np.random.default_rng(3)
    w = rng.standard_normal((Bt, L, H, Dh))
    wf = rng.standard_normal((Bt, H, Dh, Dh)) if with_gf else None
    h0 = rng.standard_normal((Bt, H, Dh, Dh)) * 0.5 if with_h0 else None
    ts = [torch.tensor(x, dtype=torch.float32).to(dtype).to(cuda_dev).requires_grad_(True) for x in ins]
    h0_t = None if h0 is None else torch.tensor(h0, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    y, fin = mr.gated_deltanet_scan_with_state(*ts, seg=seg, h0=h0_t)
    loss = (y * torch.tensor(w, dtype=torch.float32, device=cuda_dev)).sum()
    if with_gf:
        loss = loss + (fin * torch.tensor(wf, dtype=torch.float32, device=cuda_dev)).sum()
    loss.backward()
    ins_r = [_rounded(x, dtype) for x in ins]
    y_ref, f_ref = R.gdn_forward(*ins_r, h0=h0)
    grads = R.gdn_backward(*ins_r, w, wf, h0=h0)
    tol = TOL[dtype]
    assert _err(y, y_ref) <= tol
    assert _err(fin, f_ref) <= tol
    for name, t, ref in zip(("q", "k", "v", "alpha", "beta"), ts, grads[:5]):
        assert _err(t.grad, ref) <= tol, name
    if with_h0:
        assert _err(h0_t.grad, grads[5]) <= tol


def test_gdn_equals_torch_loop_autograd(cuda_dev):
    """The kernels against autograd through gated_deltanet_scan_reference (float32, GPU)."""
    mr = _mr()
    Bt, L, H, Dh = 2, 128, 3, 64
    ins = _inputs(Bt, L, H, Dh, seed=11)
    gy = torch.randn(Bt, L, H, Dh, device=cuda_dev, generator=torch.Generator(device=cuda_dev).manual_seed(0))
    mk = lambda x: torch.tensor(x, dtype=torch.float32, device=cuda_dev).requires_grad_(True)
    a = [mk(x) for x in ins]
    y1 = mr.gated_deltanet_scan(*a, seg=32)
    (y1 * gy).sum().backward()
    b = [mk(x) for x in ins]
    y2 = mr.gated_deltanet_scan_reference(*b)
    (y2 * gy).sum().backward()
    assert _err(y1, y2.detach().double().cpu().numpy()) <= 1e-5
    for name, s, t in zip(("q", "k", "v", "alpha", "beta"), a, b):
        assert _err(s.grad, t.grad.double().cpu().numpy()) <= 1e-5, name


def test_gdn_chunked_prefill_continues_the_scan(cuda_dev):
    mr = _mr()
    ins = _inputs(2, 256, 2, 64, seed=4)
    ts = [torch.tensor(x, dtype=torch.float32).to(torch.bfloat16).to(cuda_dev) for x in ins]
    y, fin = mr.gated_deltanet_scan_with_state(*ts)
    y1, f1 = mr.gated_deltanet_scan_with_state(*(t[:, :96] for t in ts))
    y2, f2 = mr.gated_deltanet_scan_with_state(*(t[:, 96:] for t in ts), h0=f1)
    assert _err(torch.cat([y1, y2], dim=1), y.double().cpu().numpy()) <= 1e-5
    assert _err(f2, fin.double().cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("Dh,dtype", [(64, torch.float32), (32, torch.bfloat16)])
def test_gdn_step_matches_oracle(cuda_dev, Dh, dtype):
    """One decode step from a random state against one step of the oracle."""
    mr = _mr()
    Bt, H = 3, 2
    ins = [x[:, 0] for x in _inputs(Bt, 1, H, Dh, seed=Dh)]
    state0 = np.random.default_rng(1).standard_normal((Bt, H, Dh, Dh))
    state = torch.tensor(state0, dtype=torch.float32, device=cuda_dev)
    args = [torch.tensor(x, dtype=torch.float32).to(dtype).to(cuda_dev) for x in ins]
    y = mr.gated_deltanet_step(*args, state)
    torch.cuda.synchronize()
    y_ref, s_ref = R.gdn_forward(*[_rounded(x, dtype)[:, None] for x in ins], h0=state0)
    tol = TOL[dtype]
    assert _err(y, y_ref[:, 0]) <= tol
    assert _err(state, s_ref) <= tol


def test_gdn_steps_reproduce_the_scan(cuda_dev):
    mr = _mr()
    Bt, T, H, Dh = 2, 32, 2, 64
    ts = [torch.tensor(x, dtype=torch.float32, device=cuda_dev) for x in _inputs(Bt, T, H, Dh, seed=9)]
    y_scan, fin = mr.gated_deltanet_scan_with_state(*ts, seg=T)
    state = torch.zeros((Bt, H, Dh, Dh), dtype=torch.float32, device=cuda_dev)
    ys = [mr.gated_deltanet_step(*(t[:, i] for t in ts), state) for i in range(T)]
    assert _err(torch.stack(ys, dim=1), y_scan.double().cpu().numpy()) <= 1e-5
    assert _err(state, fin.double().cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("Bt,L,H,Dh,seg", [
    (130, 8, 32, 32, 8),      # 4160 units: backward CTAs walk more than one unit
    (1, 256, 2, 64, 128),     # a segment of 8 staged blocks and 32 sub-blocks
])
def test_gdn_edge_shapes(cuda_dev, Bt, L, H, Dh, seg):
    mr = _mr()
    ins = _inputs(Bt, L, H, Dh, seed=Bt + L)
    w = np.random.default_rng(2).standard_normal((Bt, L, H, Dh))
    ts = [torch.tensor(x, dtype=torch.float32, device=cuda_dev).requires_grad_(True) for x in ins]
    y = mr.gated_deltanet_scan(*ts, seg=seg)
    (y * torch.tensor(w, dtype=torch.float32, device=cuda_dev)).sum().backward()
    y_ref, _ = R.gdn_forward(*ins)
    grads = R.gdn_backward(*ins, w)
    assert _err(y, y_ref) <= 1e-5
    for name, t, ref in zip(("q", "k", "v", "alpha", "beta"), ts, grads):
        assert _err(t.grad, ref) <= 1e-5, name


def test_gdn_long_segment_backward_walks_units(cuda_dev):
    """seg = L = 4096 at Dh = 32 needs 4 MB of scratch per backward CTA, so the
    1 GiB budget caps the grid at 256 CTAs for 288 units (CTAs walk units): the
    gradients equal those of the same problem with short segments."""
    mr = _mr()
    Bt, L, H, Dh = 9, 4096, 32, 32
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    q = torch.nn.functional.normalize(torch.randn(Bt, L, H, Dh, device=cuda_dev, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(Bt, L, H, Dh, device=cuda_dev, generator=g), dim=-1)
    v = torch.randn(Bt, L, H, Dh, device=cuda_dev, generator=g)
    al = torch.exp(-torch.nn.functional.softplus(torch.randn(Bt, L, H, device=cuda_dev, generator=g) - 3))
    be = torch.sigmoid(torch.randn(Bt, L, H, device=cuda_dev, generator=g))
    gy = torch.randn(Bt, L, H, Dh, device=cuda_dev, generator=g)
    out = {}
    for seg in (L, 64):
        ts = [t.clone().requires_grad_(True) for t in (q, k, v, al, be)]
        (mr.gated_deltanet_scan(*ts, seg=seg) * gy).sum().backward()
        out[seg] = [t.grad for t in ts]
    for name, a, b in zip(("q", "k", "v", "alpha", "beta"), out[L], out[64]):
        assert _err(a, b.double().cpu().numpy()) <= 1e-5, name


@pytest.mark.parametrize("case", ["strong_decay", "reset", "alpha_above_one"])
def test_gdn_chunked_forward_edge_gates(cuda_dev, case):
    """The chunkwise forward with strong decays (alpha down to 1e-4), exact
    resets (alpha = 0) and, on one unit, alphas above 1 (that unit is flagged and
    recomputed step by step), against the oracle."""
    mr = _mr()
    Bt, L, H, Dh = 2, 256, 2, 64
    ins = _inputs(Bt, L, H, Dh, seed=17)
    rng = np.random.default_rng(4)
    if case == "strong_decay":
        ins[3] = rng.uniform(1e-4, 0.5, (Bt, L, H))
    elif case == "reset":
        ins[3][:, ::37] = 0.0
    else:
        ins[3][1, 100:110, 0] = 1.05
    w = rng.standard_normal((Bt, L, H, Dh))
    ts = [torch.tensor(x, dtype=torch.float32).to(torch.bfloat16).to(cuda_dev).requires_grad_(True) for x in ins]
    y, fin = mr.gated_deltanet_scan_with_state(*ts, seg=64)
    (y * torch.tensor(w, dtype=torch.float32, device=cuda_dev)).sum().backward()
    ins_r = [_rounded(x, torch.bfloat16) for x in ins]
    y_ref, f_ref = R.gdn_forward(*ins_r)
    grads = R.gdn_backward(*ins_r, w)
    assert _err(y, y_ref) <= 2e-2
    assert _err(fin, f_ref) <= 2e-2
    for name, t, ref in zip(("q", "k", "v", "alpha", "beta"), ts, grads):
        assert _err(t.grad, ref) <= 2e-2, name


def test_gdn_chunked_forward_matches_per_step_forward(cuda_dev):
    """The two forward forms on the same bf16 inputs: chunkwise (seg 64) against
    per-step (seg 32, which the chunkwise form does not take)."""
    mr = _mr()
    ins = _inputs(4, 1024, 4, 64, seed=23)
    ts = [torch.tensor(x, dtype=torch.float32).to(torch.bfloat16).to(cuda_dev) for x in ins]
    y1, f1 = mr.gated_deltanet_scan_with_state(*ts, seg=64)
    y2, f2 = mr.gated_deltanet_scan_with_state(*ts, seg=32)
    assert _err(y1, y2.double().cpu().numpy()) <= 1e-2
    assert _err(f1, f2.double().cpu().numpy()) <= 1e-2
