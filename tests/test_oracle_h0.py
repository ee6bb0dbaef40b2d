"""Pins the oracle's initial-state extension (no counterpart in the reference)
on its zero-start restatement: a scan split in two, the second part started
from the first part's final state, equals the whole scan — forward, final
state, and every gradient, with the second part's h0 gradient fed back as the
first part's final-state cotangent."""

import numpy as np
import pytest

from oracle import ref_loops as R

RNG = np.random.default_rng(11)
L, CUT = 12, 5


def _close(a, b):
    np.testing.assert_allclose(np.asarray(a), np.asarray(b), rtol=1e-10, atol=1e-12)


def _split(x, axis=1):
    return np.take(x, range(CUT), axis=axis), np.take(x, range(CUT, x.shape[axis]), axis=axis)


def _ssd():
    Bt, H, Dh, N = 2, 2, 3, 4
    ins = (RNG.standard_normal((Bt, L, H, Dh)), np.abs(RNG.standard_normal((Bt, L, H))) * 0.3,
           RNG.standard_normal((Bt, L, H, N)), RNG.standard_normal((Bt, L, H, N)))
    A = -np.abs(RNG.standard_normal((H, N)))
    return ins, A, (Bt, H, Dh, N)


def test_ssd_split_equals_whole():
    (u, d, B, C), A, fshape = _ssd()
    gy = RNG.standard_normal(u.shape)
    gf = RNG.standard_normal(fshape)
    y, fin = R.ssd_forward(u, d, B, C, A)
    g_full = R.ssd_backward(u, d, B, C, A, gy, gf)
    p1 = [_split(t)[0] for t in (u, d, B, C)]
    p2 = [_split(t)[1] for t in (u, d, B, C)]
    y1, f1 = R.ssd_forward(*p1, A)
    y2, f2 = R.ssd_forward(*p2, A, h0=f1)
    _close(np.concatenate([y1, y2], axis=1), y)
    _close(f2, fin)
    g2 = R.ssd_backward(*p2, A, _split(gy)[1], gf, h0=f1)
    g1 = R.ssd_backward(*p1, A, _split(gy)[0], g2[-1])
    for i in range(4):
        _close(np.concatenate([g1[i], g2[i]], axis=1), g_full[i])
    _close(g1[4] + g2[4], g_full[4])


def test_gla_split_equals_whole():
    Bt, H, Dh = 2, 2, 3
    q, k, v = (RNG.standard_normal((Bt, L, H, Dh)) for _ in range(3))
    g = RNG.uniform(0.5, 1.0, (Bt, L, H))
    gy = RNG.standard_normal(q.shape)
    gf = RNG.standard_normal((Bt, H, Dh, Dh))
    y, fin = R.gla_forward(q, k, v, g)
    g_full = R.gla_backward(q, k, v, g, gy, gf)
    p1 = [_split(t)[0] for t in (q, k, v, g)]
    p2 = [_split(t)[1] for t in (q, k, v, g)]
    y1, f1 = R.gla_forward(*p1)
    y2, f2 = R.gla_forward(*p2, h0=f1)
    _close(np.concatenate([y1, y2], axis=1), y)
    _close(f2, fin)
    g2 = R.gla_backward(*p2, _split(gy)[1], gf, h0=f1)
    g1 = R.gla_backward(*p1, _split(gy)[0], g2[-1])
    for i in range(4):
        _close(np.concatenate([g1[i], g2[i]], axis=1), g_full[i])


def test_rglru_split_equals_whole():
    Bt, D = 2, 5
    a = RNG.uniform(-1.0, 1.0, (Bt, L, D))
    x = RNG.standard_normal((Bt, L, D))
    gy = RNG.standard_normal(x.shape)
    gf = RNG.standard_normal((Bt, D))
    y, fin = R.rglru_forward(a, x)
    g_full = R.rglru_backward(a, x, gy, gf)
    (a1, a2), (x1, x2), (gy1, gy2) = _split(a), _split(x), _split(gy)
    y1, f1 = R.rglru_forward(a1, x1)
    y2, f2 = R.rglru_forward(a2, x2, h0=f1)
    _close(np.concatenate([y1, y2], axis=1), y)
    _close(f2, fin)
    g2 = R.rglru_backward(a2, x2, gy2, gf, h0=f1)
    g1 = R.rglru_backward(a1, x1, gy1, g2[-1])
    for i in range(2):
        _close(np.concatenate([g1[i], g2[i]], axis=1), g_full[i])


def test_rotlru_split_equals_whole():
    Bt, Dp = 2, 3
    a = RNG.uniform(-1.0, 1.0, (Bt, L, Dp))
    th = RNG.uniform(-0.5, 0.5, (Bt, L, Dp))
    cs, sn = np.cos(th), np.sin(th)
    x = RNG.standard_normal((Bt, L, 2 * Dp))
    gy = RNG.standard_normal(x.shape)
    gf = RNG.standard_normal((Bt, 2 * Dp))
    y, fin = R.rotlru_forward(a, cs, sn, x)
    g_full = R.rotlru_backward(a, cs, sn, x, gy, gf)
    p1 = [_split(t)[0] for t in (a, cs, sn, x)]
    p2 = [_split(t)[1] for t in (a, cs, sn, x)]
    y1, f1 = R.rotlru_forward(*p1)
    y2, f2 = R.rotlru_forward(*p2, h0=f1)
    _close(np.concatenate([y1, y2], axis=1), y)
    _close(f2, fin)
    g2 = R.rotlru_backward(*p2, _split(gy)[1], gf, h0=f1)
    g1 = R.rotlru_backward(*p1, _split(gy)[0], g2[-1])
    for i in range(4):
        _close(np.concatenate([g1[i], g2[i]], axis=1), g_full[i])


@pytest.mark.parametrize("kind", ["ssd", "gla", "rglru", "rotlru"])
def test_h0_gradient_matches_finite_difference(kind):
    """d <y, w> / d h0 from the backward against a central difference."""
    rng = np.random.default_rng(3)
    if kind == "ssd":
        (u, d, B, C), A, fshape = _ssd()
        ins, fwd, bwd = (u, d, B, C, A), R.ssd_forward, R.ssd_backward
    elif kind == "gla":
        ins = tuple(rng.standard_normal((1, 6, 2, 3)) for _ in range(3)) + (rng.uniform(0.5, 1, (1, 6, 2)),)
        fshape, fwd, bwd = (1, 2, 3, 3), R.gla_forward, R.gla_backward
    elif kind == "rglru":
        ins = (rng.uniform(-1, 1, (1, 6, 4)), rng.standard_normal((1, 6, 4)))
        fshape, fwd, bwd = (1, 4), R.rglru_forward, R.rglru_backward
    else:
        th = rng.uniform(-0.5, 0.5, (1, 6, 2))
        ins = (rng.uniform(-1, 1, (1, 6, 2)), np.cos(th), np.sin(th), rng.standard_normal((1, 6, 4)))
        fshape, fwd, bwd = (1, 4), R.rotlru_forward, R.rotlru_backward
    h0 = rng.standard_normal(fshape)
    y0, _ = fwd(*ins, h0=h0)
    w = rng.standard_normal(y0.shape)
    gh0 = bwd(*ins, w, None, h0=h0)[-1]
    eps = 1e-6
    fd = np.zeros(h0.size)
    for i in range(h0.size):
        hp, hm = h0.copy().reshape(-1), h0.copy().reshape(-1)
        hp[i] += eps
        hm[i] -= eps
        fd[i] = (np.sum(fwd(*ins, h0=hp.reshape(fshape))[0] * w) -
                 np.sum(fwd(*ins, h0=hm.reshape(fshape))[0] * w)) / (2 * eps)
    np.testing.assert_allclose(np.asarray(gh0).reshape(-1), fd, rtol=1e-6, atol=1e-8)


def test_rglru_gated_gradients_match_finite_difference():
    """The gated RG-LRU oracle (input gating ahead of the scan, rglru.py:8-27):
    every gradient against central differences of <y, w> + <final, wf>."""
    rng = np.random.default_rng(9)
    Bt, T, D, c = 2, 5, 3, 8.0
    x = rng.standard_normal((Bt, T, D))
    r = rng.uniform(0.1, 0.9, (Bt, T, D))
    i = rng.uniform(0.1, 0.9, (Bt, T, D))
    lam = rng.uniform(2.2, 6.9, D)
    h0 = rng.standard_normal((Bt, D))
    w = rng.standard_normal((Bt, T, D))
    wf = rng.standard_normal((Bt, D))

    def loss(x_, r_, i_, lam_, h0_):
        y, f = R.rglru_gated_forward(x_, r_, i_, lam_, c, h0=h0_)
        return np.sum(y * w) + np.sum(f * wf)

    grads = R.rglru_gated_backward(x, r, i, lam, c, w, wf, h0=h0)
    args = [x, r, i, lam, h0]
    eps = 1e-6
    for k, g in enumerate(grads):
        fd = np.zeros(args[k].size)
        for j in range(args[k].size):
            p, m = [a.copy() for a in args], [a.copy() for a in args]
            p[k].reshape(-1)[j] += eps
            m[k].reshape(-1)[j] -= eps
            fd[j] = (loss(*p) - loss(*m)) / (2 * eps)
        np.testing.assert_allclose(np.asarray(g).reshape(-1), fd, rtol=1e-5, atol=1e-7)


def test_rotlru_angle_gradients_match_finite_difference():
    """The rotLRU angle oracle (cs = cos theta, sn = sin theta ahead of the
    scan, rotlru.py:18-22): every gradient against central differences."""
    rng = np.random.default_rng(13)
    Bt, T, Dp = 2, 5, 2
    a = rng.uniform(-1.0, 1.0, (Bt, T, Dp))
    th = rng.uniform(-3.0, 3.0, (Bt, T, Dp))
    x = rng.standard_normal((Bt, T, 2 * Dp))
    h0 = rng.standard_normal((Bt, 2 * Dp))
    w = rng.standard_normal((Bt, T, 2 * Dp))
    wf = rng.standard_normal((Bt, 2 * Dp))

    def loss(a_, th_, x_, h0_):
        y, f = R.rotlru_angle_forward(a_, th_, x_, h0=h0_)
        return np.sum(y * w) + np.sum(f * wf)

    grads = R.rotlru_angle_backward(a, th, x, w, wf, h0=h0)
    args = [a, th, x, h0]
    eps = 1e-6
    for k, g in enumerate(grads):
        fd = np.zeros(args[k].size)
        for j in range(args[k].size):
            p, m = [v.copy() for v in args], [v.copy() for v in args]
            p[k].reshape(-1)[j] += eps
            m[k].reshape(-1)[j] -= eps
            fd[j] = (loss(*p) - loss(*m)) / (2 * eps)
        np.testing.assert_allclose(np.asarray(g).reshape(-1), fd, rtol=1e-5, atol=1e-7)
