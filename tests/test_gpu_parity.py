"""CUDA path vs the oracle: forward and every gradient, through the public
API (torch.autograd over libmlrec.so). Tolerances (max|diff| / max|ref|):
1e-5 for float32 inputs, 2e-2 for bfloat16 inputs."""

import os

import numpy as np
import pytest
import torch

import _cases as K

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _run(mr, kind, ins_np, seg, dtype, dev, w=None, wf=None):
    """Run the scan (with state) on dev; return y, final, grads (float64 numpy)."""
    ts = []
    for i, x in enumerate(ins_np):
        t = torch.tensor(np.asarray(x), dtype=torch.float32)
        if not (kind == "ssd" and i == 4):
            t = t.to(dtype)
        ts.append(t.to(dev).requires_grad_(True))
    fn = getattr(mr, f"{kind}_scan_with_state")
    y, fin = fn(*ts, seg=seg)
    loss = 0.0
    if w is not None:
        loss = loss + (y * torch.tensor(w, dtype=torch.float32, device=dev)).sum()
    if wf is not None:
        loss = loss + (fin * torch.tensor(wf, dtype=torch.float32, device=dev)).sum()
    grads = torch.autograd.grad(loss, ts) if (w is not None or wf is not None) else None
    out = lambda t: t.detach().double().cpu().numpy()
    return out(y), out(fin), None if grads is None else [out(g) for g in grads]


def _rounded(ins, dtype, kind):
    """Inputs as the kernel sees them (rounded to dtype; SSD's A_neg stays f32)."""
    r = []
    for i, x in enumerate(ins):
        if kind == "ssd" and i == 4:
            r.append(np.asarray(x, dtype=np.float64))
        else:
            r.append(torch.tensor(np.asarray(x), dtype=torch.float32).to(dtype).double().numpy())
    return r


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("path", K.parity_files(), ids=os.path.basename)
def test_parity_golden_cases(mr, cuda_dev, path, dtype):
    case = K.load(path)
    kind = case["meta"]["kind"]
    seg = case["meta"].get("params", {}).get("seg", 32)
    ins, names = K.inputs_of(case)
    y, _, grads = _run(mr, kind, ins, seg, dtype, cuda_dev, w=case["w_out"])
    tol = TOL[dtype]
    if dtype == torch.float32:
        ref_y = case["y"]
        ref_g = [case["grad_" + n] for n in names]
    else:
        rins = _rounded(ins, dtype, kind)
        ref_y, _ = K.oracle_fwd(kind, rins)
        ref_g = K.oracle_bwd(kind, rins, case["w_out"])
    assert K.rel_err(y, ref_y) < tol, "y"
    for g, r, n in zip(grads, ref_g, names):
        assert K.rel_err(g, r) < tol, f"grad_{n}: {K.rel_err(g, r):.2e}"


@pytest.mark.parametrize("kind", ["ssd", "gla", "rglru"])
def test_final_state_matches_reference_loop(mr, cuda_dev, kind):
    case = K.load(os.path.join(K.GOLDEN, f"{kind}_final_state.npz"))
    ins = [case["in_" + n] for n in case["meta"]["arg_names"]]
    _, fin, _ = _run(mr, kind, ins, case["meta"].get("seg") or 32, torch.float32, cuda_dev)
    assert K.rel_err(fin, case["final"]) < 1e-5


def test_rotlru_reference_properties(mr, cuda_dev):
    c = K.load(os.path.join(K.GOLDEN, "rotlru_theta_zero_reduces_to_rglru.npz"))
    ins = [c["in_" + n] for n in ("a", "cs", "sn", "x")]
    y, _, _ = _run(mr, "rotlru", ins, 32, torch.float32, cuda_dev)
    assert np.max(np.abs(y - c["y_rglru"])) < 1e-4           # test_v2_rotlru.py:313
    c = K.load(os.path.join(K.GOLDEN, "rotlru_pure_rotation_preserves_norm.npz"))
    ins = [c["in_" + n] for n in ("a", "cs", "sn", "x")]
    y, _, _ = _run(mr, "rotlru", ins, 32, torch.float32, cuda_dev)
    yp = y.reshape(y.shape[0], y.shape[1], -1, 2)
    n = np.sqrt(yp[..., 0] ** 2 + yp[..., 1] ** 2)
    assert np.max(np.abs(n[:, -1] - n[:, 0])) < 1e-4         # test_v2_rotlru.py:334
    c = K.load(os.path.join(K.GOLDEN, "rotlru_with_state_matches_last_step.npz"))
    ins = [c["in_" + n] for n in ("a", "cs", "sn", "x")]
    y, fin, _ = _run(mr, "rotlru", ins, 32, torch.float32, cuda_dev)
    assert fin.shape == (2, 64)
    assert np.max(np.abs(fin - y[:, -1])) < 1e-6             # test_v2_rotlru.py:342


def _rand_inputs(kind, shape, seed):
    rng = np.random.default_rng(seed)
    if kind == "ssd":
        B, L, H, Dh, N = shape
        return [rng.standard_normal((B, L, H, Dh)) * 0.5, np.abs(rng.standard_normal((B, L, H))) * 0.05 + 0.001,
                rng.standard_normal((B, L, H, N)) * 0.5, rng.standard_normal((B, L, H, N)) * 0.5,
                -np.abs(rng.standard_normal((H, N))) - 0.1]
    if kind == "gla":
        B, L, H, Dh = shape
        return [rng.standard_normal((B, L, H, Dh)) * Dh ** -0.5, rng.standard_normal((B, L, H, Dh)) * 0.5,
                rng.standard_normal((B, L, H, Dh)) * 0.5, 1 / (1 + np.exp(-rng.standard_normal((B, L, H)) - 2))]
    if kind == "rglru":
        B, L, D = shape
        return [rng.uniform(-0.99, 0.99, (B, L, D)), rng.standard_normal((B, L, D)) * 0.5]
    B, L, Dp = shape
    th = rng.uniform(0, np.pi, (B, L, Dp))
    return [rng.uniform(-0.99, 0.99, (B, L, Dp)), np.cos(th), np.sin(th), rng.standard_normal((B, L, 2 * Dp)) * 0.5]


EDGE = [
    # (kind, shape, seg): single segment, seg not dividing the block, long
    # segments (workspace path), partial channel tiles, odd N
    ("rglru", (2, 96, 32), 48),
    ("rglru", (1, 64, 96), 64),
    ("rglru", (2, 512, 64), 256),
    ("rglru", (1, 40, 32), 40),
    ("rglru", (3, 1, 32), 1),
    ("rotlru", (2, 96, 48), 96),
    ("rotlru", (1, 512, 16), 128),
    ("rotlru", (2, 100, 80), 20),
    ("ssd", (1, 48, 3, 32, 5), 16),
    ("ssd", (2, 64, 2, 96, 40), 64),
    ("ssd", (1, 64, 1, 128, 128), 32),
    ("gla", (1, 48, 3, 32), 16),
    ("gla", (1, 64, 2, 96), 64),
    ("gla", (1, 32, 1, 128), 32),
    # the per-step kernels stage 16 steps (fewer for wide rows) at a time: L and seg that
    # leave partial staged blocks in the forward and in the backward's segments
    ("ssd", (2, 40, 2, 64, 16), 20),
    ("gla", (2, 40, 2, 64), 20),
]


@pytest.mark.parametrize("kind,shape,seg", EDGE, ids=[f"{k}-{'x'.join(map(str, s))}-seg{g}" for k, s, g in EDGE])
def test_edge_shapes_with_final_state_cotangent(mr, cuda_dev, kind, shape, seg):
    ins = _rand_inputs(kind, shape, seed=sum(shape) + seg)
    yo, fo = K.oracle_fwd(kind, ins)
    rng = np.random.default_rng(7)
    w = rng.standard_normal(yo.shape)
    wf = rng.standard_normal(fo.shape)
    y, fin, grads = _run(mr, kind, ins, seg, torch.float32, cuda_dev, w=w, wf=wf)
    assert K.rel_err(y, yo) < 1e-5
    assert K.rel_err(fin, fo) < 1e-5
    ref = K.oracle_bwd(kind, ins, w, wf)
    for i, (g, r) in enumerate(zip(grads, ref)):
        assert K.rel_err(g, r) < 1e-5, f"grad {i}: {K.rel_err(g, r):.2e}"


def test_ssd_per_head_rate_view_matches_dense(mr, cuda_dev):
    """A_neg given as a stride-0 view along N equals the dense [H, N] tensor."""
    ins = _rand_inputs("ssd", (2, 64, 3, 64, 16), seed=3)
    A_h = -np.abs(np.random.default_rng(0).standard_normal(3)) - 0.1
    dense = np.repeat(A_h[:, None], 16, axis=1)
    ts = [torch.tensor(x, dtype=torch.float32, device=cuda_dev) for x in ins[:4]]
    Av = torch.tensor(A_h, dtype=torch.float32, device=cuda_dev)[:, None].expand(3, 16)
    Ad = torch.tensor(dense, dtype=torch.float32, device=cuda_dev)
    y1 = mr.ssd_scan(*ts, Av)
    y2 = mr.ssd_scan(*ts, Ad)
    assert K.rel_err(y1.double().cpu().numpy(), y2.double().cpu().numpy()) < 1e-6


@pytest.mark.parametrize("Bt,L,H,seg,dtype", [
    (2, 256, 3, 32, torch.bfloat16),
    (1, 384, 2, 128, torch.float16),
    (1, 256, 2, 64, torch.bfloat16),
])
def test_ssd_tensor_core_path_through_api(mr, cuda_dev, Bt, L, H, seg, dtype):
    """bf16/fp16, Dh=64, N=128, one decay rate per head (an [H] parameter
    broadcast over N): the chunked tcgen05 path, forward and every gradient
    (the [H] parameter's gradient for A) against the float64 oracle."""
    rng = np.random.default_rng(L + H)
    u = rng.standard_normal((Bt, L, H, 64))
    delta = np.abs(rng.standard_normal((Bt, L, H))) * 0.1 + 0.01
    Bm = rng.standard_normal((Bt, L, H, 128))
    Cm = rng.standard_normal((Bt, L, H, 128))
    A_h = -np.exp(rng.standard_normal(H) * 0.5)
    ts = [torch.tensor(x, dtype=torch.float32).to(dtype).to(cuda_dev).requires_grad_(True) for x in (u, delta, Bm, Cm)]
    A_t = torch.tensor(A_h, dtype=torch.float32, device=cuda_dev, requires_grad=True)
    y, fin = mr.ssd_scan_with_state(*ts, A_t[:, None].expand(H, 128), seg=seg)
    w = rng.standard_normal(tuple(y.shape))
    wf = rng.standard_normal(tuple(fin.shape))
    loss = (y * torch.tensor(w, dtype=torch.float32, device=cuda_dev)).sum() + \
           (fin * torch.tensor(wf, dtype=torch.float32, device=cuda_dev)).sum()
    grads = torch.autograd.grad(loss, ts + [A_t])
    ins = [t.detach().double().cpu().numpy() for t in ts] + [np.repeat(A_h[:, None], 128, axis=1)]
    yo, fo = K.oracle_fwd("ssd", ins)
    ref = K.oracle_bwd("ssd", ins, w, wf)
    assert K.rel_err(y.detach().double().cpu().numpy(), yo) < 2e-2
    assert K.rel_err(fin.detach().double().cpu().numpy(), fo) < 2e-2
    for name, g, r in zip(("u", "delta", "B", "C"), grads[:4], ref[:4]):
        assert K.rel_err(g.double().cpu().numpy(), r) < 2e-2, name
    assert K.rel_err(grads[4].double().cpu().numpy(), ref[4].sum(1)) < 2e-2, "A (per head)"


@pytest.mark.parametrize("kind", ["ssd", "gla"])
def test_golden_widened_case_on_tensor_core_path(mr, cuda_dev, kind):
    """The reference's own outputs at a shape the chunked tcgen05 kernels take
    (L=256, Dh=64, N=128, bf16-representable inputs, SSD with one rate per
    head passed as an [H] parameter broadcast over N): forward and every
    gradient of the bf16 run against the golden float32 values at 2e-2."""
    import importlib
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    lib = Lm.load()
    case = K.load(os.path.join(K.GOLDEN, f"{kind}_tc_parity_widened.npz"))
    ins, names = K.inputs_of(case)
    Bt, L, H, Dh = ins[0].shape
    ts = [torch.tensor(x, dtype=torch.float32).to(torch.bfloat16).to(cuda_dev).requires_grad_(True)
          for x in (ins[:4] if kind == "ssd" else ins)]
    # the bf16 rounding is exact: the golden inputs are bf16 values
    for t, x in zip(ts, ins):
        assert np.array_equal(t.detach().double().cpu().numpy(), x)
    args = list(ts)
    if kind == "ssd":
        A_rows = ins[4]
        assert np.all(A_rows == A_rows[:, :1])
        A_t = torch.tensor(A_rows[:, 0], dtype=torch.float32, device=cuda_dev, requires_grad=True)
        args.append(A_t[:, None].expand(H, A_rows.shape[1]))
        leaves = ts + [A_t]
        # the tensor-core path checkpoints every 128-step chunk
        assert lib.mr_ssd_preferred_seg(Lm.MR_BF16, L, Dh, A_rows.shape[1], 32, 0) == 128
        y = mr.ssd_scan(*args, seg=32)
    else:
        leaves = ts
        assert lib.mr_gla_preferred_seg(Lm.MR_BF16, L, Dh, 32) == 128
        y = mr.gla_scan(*args, seg=32)
    w = torch.tensor(case["w_out"], dtype=torch.float32, device=cuda_dev)
    grads = torch.autograd.grad((y * w).sum(), leaves)
    assert K.rel_err(y.detach().double().cpu().numpy(), case["y"]) < 2e-2, "y"
    for n, g in zip(names, grads):
        ref = case["grad_" + n]
        if kind == "ssd" and n == "A_neg":
            ref = ref.sum(axis=1)  # d loss / d (one rate per head)
        err = K.rel_err(g.double().cpu().numpy(), ref)
        assert err < 2e-2, f"grad_{n}: {err:.2e}"
