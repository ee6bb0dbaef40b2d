"""Pins the Gated DeltaNet oracle (the reference carries this recurrence as a
design only, docs/DESIGN_gated_deltanet.md): the hand-derived adjoint against
central differences and against torch autograd through the plug-in's own
per-step torch loop (float64, CPU), the forward against that loop, and the
split-scan property of the initial state."""

import importlib

import numpy as np
import pytest
import torch

from oracle import ref_loops as R


def _inputs(rng, Bt, T, H, Dh):
    def nrm(x):
        return x / np.linalg.norm(x, axis=-1, keepdims=True)
    q = nrm(rng.standard_normal((Bt, T, H, Dh)))
    k = nrm(rng.standard_normal((Bt, T, H, Dh)))
    v = rng.standard_normal((Bt, T, H, Dh))
    al = rng.uniform(0.5, 1.0, (Bt, T, H))
    be = rng.uniform(0.1, 0.9, (Bt, T, H))
    return q, k, v, al, be


def test_gdn_gradients_match_finite_difference():
    rng = np.random.default_rng(21)
    Bt, T, H, Dh = 2, 5, 2, 3
    args = list(_inputs(rng, Bt, T, H, Dh)) + [rng.standard_normal((Bt, H, Dh, Dh))]
    w = rng.standard_normal((Bt, T, H, Dh))
    wf = rng.standard_normal((Bt, H, Dh, Dh))

    def loss(q, k, v, al, be, h0):
        o, f = R.gdn_forward(q, k, v, al, be, h0=h0)
        return np.sum(o * w) + np.sum(f * wf)

    grads = R.gdn_backward(*args[:5], w, wf, h0=args[5])
    eps = 1e-6
    for n, g in enumerate(grads):
        fd = np.zeros(args[n].size)
        for j in range(args[n].size):
            p, m = [a.copy() for a in args], [a.copy() for a in args]
            p[n].reshape(-1)[j] += eps
            m[n].reshape(-1)[j] -= eps
            fd[j] = (loss(*p) - loss(*m)) / (2 * eps)
        np.testing.assert_allclose(np.asarray(g).reshape(-1), fd, rtol=1e-5, atol=1e-7)


def test_gdn_oracle_matches_torch_loop_and_autograd():
    mr = importlib.import_module("mlx-recurrence_b200")
    rng = np.random.default_rng(5)
    Bt, T, H, Dh = 2, 7, 3, 4
    ins = _inputs(rng, Bt, T, H, Dh)
    h0 = rng.standard_normal((Bt, H, Dh, Dh))
    w = rng.standard_normal((Bt, T, H, Dh))
    ts = [torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in ins]
    h0_t = torch.tensor(h0, dtype=torch.float64, requires_grad=True)
    y = mr.gated_deltanet_scan_reference(*ts, h0=h0_t)
    y_ref, _ = R.gdn_forward(*ins, h0=h0)
    np.testing.assert_allclose(y.detach().numpy(), y_ref, rtol=1e-12, atol=1e-12)
    (y * torch.tensor(w)).sum().backward()
    grads = R.gdn_backward(*ins, w, None, h0=h0)
    for t, g in zip(ts + [h0_t], grads):
        np.testing.assert_allclose(t.grad.numpy(), g, rtol=1e-10, atol=1e-12)


def test_gdn_split_equals_whole():
    rng = np.random.default_rng(8)
    Bt, T, H, Dh, cut = 2, 11, 2, 3, 4
    ins = _inputs(rng, Bt, T, H, Dh)
    gy = rng.standard_normal((Bt, T, H, Dh))
    gf = rng.standard_normal((Bt, H, Dh, Dh))
    y, fin = R.gdn_forward(*ins)
    g_full = R.gdn_backward(*ins, gy, gf)
    p1 = [x[:, :cut] for x in ins]
    p2 = [x[:, cut:] for x in ins]
    y1, f1 = R.gdn_forward(*p1)
    y2, f2 = R.gdn_forward(*p2, h0=f1)
    np.testing.assert_allclose(np.concatenate([y1, y2], axis=1), y, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(f2, fin, rtol=1e-10, atol=1e-12)
    g2 = R.gdn_backward(*p2, gy[:, cut:], gf, h0=f1)
    g1 = R.gdn_backward(*p1, gy[:, :cut], g2[-1])
    for i in range(5):
        np.testing.assert_allclose(np.concatenate([g1[i], g2[i]], axis=1), g_full[i], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("bad", ["dh", "alpha"])
def test_gdn_shape_rules(bad):
    mr = importlib.import_module("mlx-recurrence_b200")
    Dh = 48 if bad == "dh" else 32
    q = torch.zeros(1, 32, 2, Dh)
    al = torch.zeros(1, 32, 3 if bad == "alpha" else 2)
    with pytest.raises(ValueError, match="Dh=48 is not supported" if bad == "dh" else "alpha must be"):
        mr.gated_deltanet_scan(q, q, q, al, torch.zeros(1, 32, 2))


def test_c_oracle_gdn_matches_numpy_oracle():
    """The float32 C restatement (the timed CPU baseline of the Gated DeltaNet
    bench configuration) against the float64 oracle, with a final-state cotangent."""
    import c_oracle
    rng = np.random.default_rng(13)
    Bt, T, H, Dh, seg = 2, 48, 2, 8, 16
    ins = [np.asarray(x, np.float32).astype(np.float64) for x in _inputs(rng, Bt, T, H, Dh)]
    y, f = R.gdn_forward(*ins)
    w, wf = rng.standard_normal(y.shape), rng.standard_normal(f.shape)
    ref = R.gdn_backward(*ins, w, wf)
    out = c_oracle.run("gdn", ins, seg, gy=w, g_final=wf)
    assert R.rel_err(out["y"], y) < 1e-5
    assert R.rel_err(out["final"], f) < 1e-5
    for g, r in zip(out["grads"], ref):
        assert R.rel_err(g, r) < 1e-5


@pytest.mark.parametrize("C", [1, 4, 16, 7])
def test_gdn_chunked_wy_form_equals_the_recurrence(C):
    """The chunkwise WY algebra (the design's phase-1 gate: chunk form against
    the sequential reference) reproduces the per-step recurrence, its outputs,
    final state and the per-step w = beta (v - alpha S^T k), for chunk lengths
    that do and do not divide L."""
    rng = np.random.default_rng(C)
    Bt, T, H, Dh = 2, 32, 2, 6
    ins = list(_inputs(rng, Bt, T, H, Dh))
    ins[3] = rng.uniform(0.05, 1.0, (Bt, T, H))      # strong decays too
    h0 = rng.standard_normal((Bt, H, Dh, Dh))
    y, fin = R.gdn_forward(*ins, h0=h0)
    yc, finc, w = R.gdn_chunked_forward(*ins, C, h0=h0)
    np.testing.assert_allclose(yc, y, rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(finc, fin, rtol=1e-9, atol=1e-10)
    q, k, v, al, be = ins
    S = h0.copy()
    for t in range(T):
        p = np.einsum("bhij,bhi->bhj", S, k[:, t])
        wt = be[:, t, :, None] * (v[:, t] - al[:, t, :, None] * p)
        np.testing.assert_allclose(w[:, t], wt, rtol=1e-9, atol=1e-10)
        S = al[:, t, :, None, None] * S + k[:, t, :, :, None] * wt[:, :, None, :]
