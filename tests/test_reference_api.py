"""The package's own pure per-step functions and its parity helper (CPU only).

``ssd_scan_reference``, ``gla_scan_reference``, ``rglru_scan_reference`` and
``rotlru_scan_reference`` are public API (the reference exports them from
``mlx_recurrence/__init__.py:21-90``; their definitions are ``ssd.py:382-394``,
``gla.py:336-346``, ``rglru.py:274-282``, ``rotlru.py:338-351``). Each is run
in float64 on the golden inputs and compared with the reference's own outputs
and gradients (the golden vectors), and with the oracle. ``parity_check``
(``_chassis.py:122-213``) is exercised on a passing and on a failing pair.
"""

import os

import numpy as np
import pytest
import torch

import _cases as K

FNS = {"ssd": "ssd_scan_reference", "gla": "gla_scan_reference", "rglru": "rglru_scan_reference",
       "rotlru": "rotlru_scan_reference"}


@pytest.mark.parametrize("path", K.parity_files(), ids=os.path.basename)
def test_scan_reference_matches_golden_and_oracle(mr, path):
    case = K.load(path)
    kind = case["meta"]["kind"]
    ins, names = K.inputs_of(case)
    ts = [torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in ins]
    y = getattr(mr, FNS[kind])(*ts)
    w = torch.tensor(case["w_out"], dtype=torch.float64)
    grads = torch.autograd.grad((y * w).sum(), ts)
    # the golden values are float32 roundings of the reference's float64 run
    assert K.rel_err(y.detach().numpy(), case["y"]) < 1e-6
    for n, g in zip(names, grads):
        assert K.rel_err(g.numpy(), case["grad_" + n]) < 1e-6, n
    yo, _ = K.oracle_fwd(kind, ins)
    assert K.rel_err(y.detach().numpy(), yo) < 1e-12
    go = K.oracle_bwd(kind, ins, case["w_out"])
    for n, g, r in zip(names, grads, go):
        assert K.rel_err(g.numpy(), r) < 1e-10, n


def test_rglru_scan_reference_last_step_is_final_state(mr):
    """For the diagonal scan y_t = h_t, so the pure loop's last step equals the
    reference's final-state hand loop (test_v2_rglru.py:39-51)."""
    case = K.load(os.path.join(K.GOLDEN, "rglru_final_state.npz"))
    ins = [case["in_" + n] for n in case["meta"]["arg_names"]]
    y = mr.rglru_scan_reference(*(torch.tensor(x, dtype=torch.float64) for x in ins))
    assert K.rel_err(y[:, -1].numpy(), case["final"]) < 1e-6


def test_rotlru_scan_reference_properties(mr):
    """theta = 0 reduces to RG-LRU, rotation preserves the pair norm, the last
    step equals the final state (test_v2_rotlru.py:77-123), on the golden inputs."""
    c = K.load(os.path.join(K.GOLDEN, "rotlru_theta_zero_reduces_to_rglru.npz"))
    ins = [torch.tensor(c["in_" + n], dtype=torch.float64) for n in ("a", "cs", "sn", "x")]
    y = mr.rotlru_scan_reference(*ins).numpy()
    assert K.rel_err(y, c["y_rot"]) < 1e-6
    assert np.max(np.abs(y - c["y_rglru"])) < 1e-4
    c = K.load(os.path.join(K.GOLDEN, "rotlru_pure_rotation_preserves_norm.npz"))
    ins = [torch.tensor(c["in_" + n], dtype=torch.float64) for n in ("a", "cs", "sn", "x")]
    y = mr.rotlru_scan_reference(*ins).numpy()
    assert K.rel_err(y, c["y"]) < 1e-6
    c = K.load(os.path.join(K.GOLDEN, "rotlru_with_state_matches_last_step.npz"))
    ins = [torch.tensor(c["in_" + n], dtype=torch.float64) for n in ("a", "cs", "sn", "x")]
    y = mr.rotlru_scan_reference(*ins).numpy()
    assert K.rel_err(y[:, -1], c["final"]) < 1e-6


def _rglru_golden():
    c = K.load(os.path.join(K.GOLDEN, "rglru_rglru_parity_0.npz"))
    return [torch.tensor(c["in_a"], dtype=torch.float64), torch.tensor(c["in_x"], dtype=torch.float64)]


def _rglru_closed_form(a, x):
    """y_t = sum_{s <= t} (prod_{r in (s, t]} a_r) x_s as one matrix product per
    channel (positive gates): an independent restatement of the recurrence."""
    la = torch.cumsum(torch.log(a), dim=1)                         # [B, L, D]
    L = a.shape[1]
    tri = torch.tril(torch.ones(L, L, dtype=a.dtype))
    M = torch.exp(la[:, :, None, :] - la[:, None, :, :]) * tri[None, :, :, None]
    return torch.einsum("btsd,bsd->btd", M, x)


def test_parity_check_passes_a_matching_pair(mr):
    ins = _rglru_golden()
    assert float(ins[0].min()) > 0
    ok, report = mr.parity_check(mr.rglru_scan_reference, _rglru_closed_form, ins, ["a", "x"], (0, 1),
                                 verbose=False)
    assert ok
    assert set(report) == {"y", "grad_a", "grad_x"}
    assert report["y"]["abs"] < 1e-10 and report["grad_a"]["rel"] < 1e-10


def test_parity_check_fails_a_wrong_pair(mr, capsys):
    ins = _rglru_golden()
    wrong = lambda a, x: mr.rglru_scan_reference(a, x * 1.01)
    ok, report = mr.parity_check(mr.rglru_scan_reference, wrong, ins, ["a", "x"], (0, 1), label="wrong")
    assert not ok
    # forward: max|y_k - y_r| against the absolute y_tol (default 1e-3)
    y_r = wrong(*ins)
    y_k = mr.rglru_scan_reference(*ins)
    assert report["y"]["abs"] == pytest.approx(float((y_k - y_r).abs().max()))
    assert report["y"]["abs"] > 1e-3
    # gradient metric: max|g_k - g_r| / (max|g_r| + 1e-8), against grad_rtol (default 1e-3)
    assert report["grad_x"]["rel"] > 1e-3
    assert "FAIL" in capsys.readouterr().out


def test_parity_check_w_out_is_seeded(mr):
    """The loss weights come from a generator seeded 1234 (_chassis.py:166-169):
    two runs report identical numbers."""
    ins = _rglru_golden()
    wrong = lambda a, x: mr.rglru_scan_reference(a * 0.999, x)
    r1 = mr.parity_check(mr.rglru_scan_reference, wrong, ins, ["a", "x"], (0, 1), verbose=False)[1]
    r2 = mr.parity_check(mr.rglru_scan_reference, wrong, ins, ["a", "x"], (0, 1), verbose=False)[1]
    assert r1 == r2
