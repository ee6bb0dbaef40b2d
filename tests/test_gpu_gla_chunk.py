"""The tcgen05 chunked GLA kernels through the C-ABI (bf16/fp16 inputs, Dh = 64,
checkpoints every 128-step chunk), against the float64 per-step oracle on the
same (rounded) inputs: outputs, every checkpoint, the final state and every
gradient. Tolerance 2e-2 (max|diff| / max|ref|). Units (batch row, head) with
a gate outside [1e-3, 1] are recomputed by the per-step kernels; their float32
outputs are checked to 1e-4 and their bf16 gradients to 5e-3."""

import importlib

import numpy as np
import pytest
import torch

import _cases as K

pytestmark = pytest.mark.gpu

DH = 64
SEG = 128


def _oracle_states(q, k, v, g, seg):
    """y and the states h[i, j] at every seg boundary, float64 (gla.py:336-346)."""
    Bt, L, H, Dh = q.shape
    h = np.zeros((Bt, H, Dh, Dh))
    y = np.empty((Bt, L, H, Dh))
    ck = []
    for t in range(L):
        h = g[:, t, :, None, None] * h + k[:, t, :, :, None] * v[:, t, :, None, :]
        y[:, t] = np.sum(q[:, t, :, :, None] * h, axis=-2)
        if (t + 1) % seg == 0:
            ck.append(h.copy())
    return y, np.stack(ck, axis=1)


def _inputs(Bt, L, H, seed, gates="sigmoid", dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    s = DH ** -0.5
    q, k, v = (torch.randn(Bt, L, H, DH, generator=g) * s for _ in range(3))
    if gates == "sigmoid":  # the reference's distribution: sigmoid(N(2, 1))
        gt = torch.sigmoid(torch.randn(Bt, L, H, generator=g) + 2.0)
    else:  # strong decay: gates down to 1e-3, spans far above e^40 per 16-step block
        gt = torch.rand(Bt, L, H, generator=g) * 0.3 + 1e-3
    return [t.to(dtype) for t in (q, k, v, gt)]


def _run(Lm, cuda_dev, ins, dtype, gy=None, gf=None):
    lib = Lm.load()
    Bt, L, H, _ = ins[0].shape
    code = Lm.DTYPE_CODE[dtype]
    dev = [t.to(cuda_dev).contiguous() for t in ins]
    y = torch.full((Bt, L, H, DH), float("nan"), device=cuda_dev)
    ck = torch.full((Bt, L // SEG, H, DH, DH), float("nan"), device=cuda_dev)
    lib.mr_device_error_status(1)
    Lm.call("mr_gla_fwd", *(Lm.ptr(t) for t in dev), code, Bt, L, H, DH, SEG, Lm.ptr(y), Lm.ptr(ck),
            Lm.stream_of(cuda_dev))
    grads = None
    if gy is not None:
        grads = [torch.full_like(t, float("nan")) for t in dev]
        nws = lib.mr_gla_bwd_workspace_bytes(code, Bt, L, H, DH, SEG)
        ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda_dev)
        gy_d = gy.to(cuda_dev).contiguous()
        gf_d = None if gf is None else gf.to(cuda_dev).contiguous()
        Lm.call("mr_gla_bwd", Lm.ptr(gy_d), Lm.ptr(gf_d), Lm.ptr(ck), *(Lm.ptr(t) for t in dev), code,
                Bt, L, H, DH, SEG, *(Lm.ptr(t) for t in grads), Lm.ptr(ws), ws.numel(),
                Lm.stream_of(cuda_dev))
    torch.cuda.synchronize()
    assert lib.mr_device_error_status(1) == 0
    return y, ck, grads


@pytest.mark.parametrize("Bt,L,H,gates,dtype", [
    (2, 512, 3, "sigmoid", torch.bfloat16),
    (1, 384, 2, "strong", torch.bfloat16),
    (1, 256, 2, "sigmoid", torch.float16),
])
def test_gla_chunk_forward_matches_oracle(cuda_dev, Bt, L, H, gates, dtype):
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    ins = _inputs(Bt, L, H, seed=L + H, gates=gates, dtype=dtype)
    y, ck, _ = _run(Lm, cuda_dev, ins, dtype)
    yo, cko = _oracle_states(*[t.double().numpy() for t in ins], SEG)
    assert K.rel_err(y.double().cpu().numpy(), yo) < 2e-2
    assert K.rel_err(ck.double().cpu().numpy(), cko) < 2e-2
    assert K.rel_err(ck[:, -1].double().cpu().numpy(), cko[:, -1]) < 5e-3


@pytest.mark.parametrize("Bt,L,H,gates,with_final,dtype", [
    (2, 512, 3, "sigmoid", True, torch.bfloat16),
    (1, 384, 2, "strong", False, torch.bfloat16),
    (1, 256, 2, "sigmoid", True, torch.float16),
    (1, 256, 16, "sigmoid", True, torch.bfloat16),  # H % 8 == 0: the gates arrive by TMA
])
def test_gla_chunk_backward_matches_oracle(cuda_dev, Bt, L, H, gates, with_final, dtype):
    """Every gradient of <y, gy> + <final, g_final>."""
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    ins = _inputs(Bt, L, H, seed=3 * L + H, gates=gates, dtype=dtype)
    g = torch.Generator().manual_seed(5)
    gy = torch.randn(Bt, L, H, DH, generator=g)
    gf = torch.randn(Bt, H, DH, DH, generator=g) if with_final else None
    _, _, grads = _run(Lm, cuda_dev, ins, dtype, gy, gf)
    ref = K.oracle_bwd("gla", [t.double().numpy() for t in ins], gy.double().numpy(),
                       None if gf is None else gf.double().numpy())
    for name, got, r in zip(("q", "k", "v", "gates"), grads, ref):
        err = K.rel_err(got.double().cpu().numpy(), r)
        assert err < 2e-2, f"grad_{name}: {err:.2e}"


def test_gla_out_of_range_gates_are_recomputed(cuda_dev):
    """Units holding a gate of 0, a negative gate, a gate above 1 or a tiny one
    take the per-step kernels after the chunk kernels: float32-exact there,
    chunk accuracy elsewhere, forward and backward."""
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    Bt, L, H = 2, 256, 3
    q, k, v, gt = _inputs(Bt, L, H, seed=99, dtype=torch.float32)
    gt[0, 40, 0] = 0.0
    gt[0, 200, 1] = -0.7
    gt[1, 7, 2] = 1.25
    gt[1, 130, 0] = 1e-5
    ins = [t.to(torch.bfloat16) for t in (q, k, v, gt)]
    bad = [(0, 0), (0, 1), (1, 2), (1, 0)]
    g = torch.Generator().manual_seed(8)
    gy = torch.randn(Bt, L, H, DH, generator=g)
    gf = torch.randn(Bt, H, DH, DH, generator=g)
    y, ck, grads = _run(Lm, cuda_dev, ins, torch.bfloat16, gy, gf)
    i64 = [t.double().numpy() for t in ins]
    yo, cko = _oracle_states(*i64, SEG)
    ref = K.oracle_bwd("gla", i64, gy.double().numpy(), gf.double().numpy())
    y, ck = y.double().cpu().numpy(), ck.double().cpu().numpy()
    got = [t.double().cpu().numpy() for t in grads]
    for b in range(Bt):
        for h in range(H):
            # float32 outputs of the per-step kernels are float32-exact; the gradients
            # come back in bf16 (relative rounding 2^-9)
            tol, gtol = (1e-4, 5e-3) if (b, h) in bad else (2e-2, 2e-2)
            assert K.rel_err(y[b, :, h], yo[b, :, h]) < tol, (b, h)
            assert K.rel_err(ck[b, :, h], cko[b, :, h]) < tol, (b, h)
            for name, gt_, r in zip(("q", "k", "v", "gates"), got, ref):
                err = K.rel_err(gt_[b, :, h], r[b, :, h])
                assert err < gtol, f"grad_{name} unit {(b, h)}: {err:.2e}"


def test_gla_public_api_takes_the_tensor_core_path(cuda_dev):
    """gla_scan_with_state at a qualifying shape: checkpoint spacing 128 is
    chosen whatever seg divides it, and forward + autograd match the oracle."""
    mr = importlib.import_module("mlx-recurrence_b200")
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    assert Lm.load().mr_gla_preferred_seg(Lm.DTYPE_CODE[torch.bfloat16], 256, DH, 32) == SEG
    assert Lm.load().mr_gla_preferred_seg(Lm.DTYPE_CODE[torch.float32], 256, DH, 32) == 32
    Bt, L, H = 1, 256, 2
    ins = _inputs(Bt, L, H, seed=21)
    xs = [t.to(cuda_dev).requires_grad_(True) for t in ins]
    y, final = mr.gla_scan_with_state(*xs, seg=32)
    g = torch.Generator().manual_seed(4)
    gy = torch.randn(Bt, L, H, DH, generator=g)
    gf = torch.randn(Bt, H, DH, DH, generator=g)
    ((y * gy.to(cuda_dev)).sum() + (final * gf.to(cuda_dev)).sum()).backward()
    i64 = [t.double().numpy() for t in ins]
    yo, fo = K.oracle_fwd("gla", i64)
    assert K.rel_err(y.detach().double().cpu().numpy(), yo) < 2e-2
    assert K.rel_err(final.detach().double().cpu().numpy(), fo) < 2e-2
    ref = K.oracle_bwd("gla", i64, gy.double().numpy(), gf.double().numpy())
    for name, x, r in zip(("q", "k", "v", "gates"), xs, ref):
        err = K.rel_err(x.grad.double().cpu().numpy(), r)
        assert err < 2e-2, f"grad_{name}: {err:.2e}"
