"""The CPU oracle against golden vectors from the reference's own code, and
against every property the reference's v2 tests assert (CPU only)."""

import math
import os

import numpy as np
import pytest

import _cases as K
import ref_loops as R

PIN_TOL = 1e-6  # golden arrays are float32; the oracle computes in float64


@pytest.mark.parametrize("path", K.parity_files(), ids=os.path.basename)
def test_oracle_matches_reference_golden(path):
    case = K.load(path)
    kind = case["meta"]["kind"]
    ins, names = K.inputs_of(case)
    y, _ = K.oracle_fwd(kind, ins)
    assert K.rel_err(y, case["y"]) < PIN_TOL
    grads = K.oracle_bwd(kind, ins, case["w_out"])
    for g, n in zip(grads, names):
        assert K.rel_err(g, case["grad_" + n]) < PIN_TOL, n


@pytest.mark.parametrize("kind", ["ssd", "gla", "rglru"])
def test_oracle_final_state_matches_reference_loop(kind):
    case = K.load(os.path.join(K.GOLDEN, f"{kind}_final_state.npz"))
    ins = [case["in_" + n] for n in case["meta"]["arg_names"]]
    _, final = K.oracle_fwd(kind, ins)
    assert K.rel_err(final, case["final"]) < PIN_TOL


def test_oracle_rotlru_properties_match_reference():
    # test_v2_rotlru.py:77-94: theta = 0 reduces to RG-LRU with the gate per pair
    c = K.load(os.path.join(K.GOLDEN, "rotlru_theta_zero_reduces_to_rglru.npz"))
    y, _ = R.rotlru_forward(c["in_a"], c["in_cs"], c["in_sn"], c["in_x"])
    assert K.rel_err(y, c["y_rot"]) < PIN_TOL
    a_full = np.repeat(c["in_a"][..., None], 2, axis=-1).reshape(c["in_x"].shape)
    yr, _ = R.rglru_forward(a_full, c["in_x"])
    assert np.max(np.abs(y - yr)) < 1e-4
    # test_v2_rotlru.py:97-115: pure rotation preserves the pair norm
    c = K.load(os.path.join(K.GOLDEN, "rotlru_pure_rotation_preserves_norm.npz"))
    y, _ = R.rotlru_forward(c["in_a"], c["in_cs"], c["in_sn"], c["in_x"])
    assert K.rel_err(y, c["y"]) < PIN_TOL
    yp = y.reshape(y.shape[0], y.shape[1], -1, 2)
    norms = np.sqrt(yp[..., 0] ** 2 + yp[..., 1] ** 2)
    assert np.max(np.abs(norms[:, -1] - norms[:, 0])) < 1e-4
    # test_v2_rotlru.py:118-123: final state is the last output step
    c = K.load(os.path.join(K.GOLDEN, "rotlru_with_state_matches_last_step.npz"))
    y, final = R.rotlru_forward(c["in_a"], c["in_cs"], c["in_sn"], c["in_x"])
    assert K.rel_err(y, c["y"]) < PIN_TOL
    assert np.max(np.abs(final - y[:, -1])) < 1e-6


def _fd_check(fwd, bwd, ins, idx, seed=0, eps=1e-6):
    """Directional finite difference of <y, w> + <final, wf> against the adjoint."""
    rng = np.random.default_rng(seed)
    y, f = fwd(*ins)
    w = rng.standard_normal(y.shape)
    wf = rng.standard_normal(f.shape)
    grads = bwd(*ins, w, wf)
    d = rng.standard_normal(np.shape(ins[idx]))
    plus = [np.array(x, dtype=np.float64) for x in ins]
    minus = [np.array(x, dtype=np.float64) for x in ins]
    plus[idx] = plus[idx] + eps * d
    minus[idx] = minus[idx] - eps * d
    yp, fp = fwd(*plus)
    ym, fm = fwd(*minus)
    fd = (np.sum((yp - ym) * w) + np.sum((fp - fm) * wf)) / (2 * eps)
    an = np.sum(grads[idx] * d)
    assert abs(fd - an) <= 1e-6 * max(1.0, abs(an)), (fd, an)


def test_oracle_adjoints_include_final_state_cotangent():
    rng = np.random.default_rng(1)
    B, L, H, Dh, N = 1, 12, 2, 4, 3
    ssd_in = [rng.standard_normal((B, L, H, Dh)), np.abs(rng.standard_normal((B, L, H))) * 0.1 + 0.01,
              rng.standard_normal((B, L, H, N)), rng.standard_normal((B, L, H, N)),
              -np.abs(rng.standard_normal((H, N))) - 0.1]
    for i in range(5):
        _fd_check(R.ssd_forward, R.ssd_backward, ssd_in, i)
    gla_in = [rng.standard_normal((B, L, H, Dh)) for _ in range(3)] + [1 / (1 + np.exp(-rng.standard_normal((B, L, H)) - 2))]
    for i in range(4):
        _fd_check(R.gla_forward, R.gla_backward, gla_in, i)
    rg_in = [rng.uniform(-0.99, 0.99, (2, L, 8)), rng.standard_normal((2, L, 8))]
    for i in range(2):
        _fd_check(R.rglru_forward, R.rglru_backward, rg_in, i)
    th = rng.uniform(0, math.pi, (2, L, 4))
    rot_in = [rng.uniform(-0.99, 0.99, (2, L, 4)), np.cos(th), np.sin(th), rng.standard_normal((2, L, 8))]
    for i in range(4):
        _fd_check(R.rotlru_forward, R.rotlru_backward, rot_in, i)


@pytest.mark.parametrize("path", K.parity_files(), ids=os.path.basename)
def test_c_oracle_matches_reference_golden(path):
    """The float32 C restatement (the timed CPU baseline) against the golden
    vectors, forward and every gradient, at the fp32 gate."""
    import c_oracle
    case = K.load(path)
    kind = case["meta"]["kind"]
    ins, names = K.inputs_of(case)
    seg = case["meta"].get("params", {}).get("seg", 32)
    out = c_oracle.run(kind, ins, seg, gy=case["w_out"])
    assert K.rel_err(out["y"], case["y"]) < 1e-5
    for g, n in zip(out["grads"], names):
        assert K.rel_err(g, case["grad_" + n]) < 1e-5, n


def test_c_oracle_final_state_cotangent_matches_numpy_oracle():
    import c_oracle
    rng = np.random.default_rng(5)
    B, L, H, Dh, N = 2, 48, 2, 8, 5
    ins = [rng.standard_normal((B, L, H, Dh)), np.abs(rng.standard_normal((B, L, H))) * 0.1 + 0.01,
           rng.standard_normal((B, L, H, N)), rng.standard_normal((B, L, H, N)),
           -np.abs(rng.standard_normal((H, N))) - 0.1]
    ins = [np.asarray(x, np.float32).astype(np.float64) for x in ins]
    y, f = R.ssd_forward(*ins)
    w, wf = rng.standard_normal(y.shape), rng.standard_normal(f.shape)
    ref = R.ssd_backward(*ins, w, wf)
    out = c_oracle.run("ssd", ins, 16, gy=w, g_final=wf)
    assert K.rel_err(out["final"], f) < 1e-5
    for g, r in zip(out["grads"], ref):
        assert K.rel_err(g, r) < 1e-5


@pytest.mark.parametrize("seg", [1, 7, 40, 1000])
def test_segmented_backwards_equal_plain(seg):
    """The segmented float64 backwards (states regenerated per segment, used
    for full-length configurations) give the same numbers as the plain ones,
    including the final-state cotangent and h0."""
    rng = np.random.default_rng(seg)
    B, L, H, Dh, N = 2, 80, 2, 8, 5
    u = rng.standard_normal((B, L, H, Dh))
    d = np.abs(rng.standard_normal((B, L, H))) * 0.1 + 0.01
    Bm, Cm = rng.standard_normal((B, L, H, N)), rng.standard_normal((B, L, H, N))
    A = -np.abs(rng.standard_normal((H, N))) - 0.1
    gy = rng.standard_normal((B, L, H, Dh))
    gf, h0 = rng.standard_normal((B, H, Dh, N)), rng.standard_normal((B, H, Dh, N))
    for a, b in zip(R.ssd_backward(u, d, Bm, Cm, A, gy, gf, h0=h0),
                    R.ssd_backward_segmented(u, d, Bm, Cm, A, gy, gf, h0=h0, seg=seg)):
        assert np.array_equal(a, b)
    q, k, v = (rng.standard_normal((B, L, H, Dh)) for _ in range(3))
    g = 1 / (1 + np.exp(-rng.standard_normal((B, L, H)) - 2))
    gf2 = rng.standard_normal((B, H, Dh, Dh))
    for a, b in zip(R.gla_backward(q, k, v, g, gy, gf2), R.gla_backward_segmented(q, k, v, g, gy, gf2, seg=seg)):
        assert np.array_equal(a, b)
