"""The tcgen05 chunked SSD kernels through the C-ABI (bf16/fp16 inputs, one
decay rate per head, checkpoints every 128-step chunk or a multiple), against
the float64 oracle on the same (rounded) inputs: outputs, every checkpoint
and the final state. Tolerance 2e-2 (max|diff| / max|ref|)."""

import importlib

import numpy as np
import pytest
import torch

import _cases as K

pytestmark = pytest.mark.gpu


def _oracle_states(u, delta, B, C, A, seg):
    """y and the states at every seg boundary, float64 (ssd.py:382-394)."""
    Bt, L, H, Dh = u.shape
    N = A.shape[-1]
    h = np.zeros((Bt, H, Dh, N))
    y = np.empty((Bt, L, H, Dh))
    ck = []
    for t in range(L):
        dt = delta[:, t, :, None, None]
        h = np.exp(dt * A[None, :, None, :]) * h + dt * B[:, t, :, None, :] * u[:, t, :, :, None]
        y[:, t] = np.sum(h * C[:, t, :, None, :], axis=-1)
        if (t + 1) % seg == 0:
            ck.append(np.swapaxes(h, -1, -2).copy())  # [B, H, N, Dh]
    return y, np.stack(ck, axis=1)


def _inputs(Bt, L, H, seed, dt_scale=0.1, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(Bt, L, H, 64, generator=g)
    delta = torch.randn(Bt, L, H, generator=g).abs() * dt_scale + 0.01
    Bm = torch.randn(Bt, L, H, 128, generator=g)
    Cm = torch.randn(Bt, L, H, 128, generator=g)
    A = -torch.exp(torch.randn(H, generator=g) * 0.5)
    return [t.to(dtype) for t in (u, delta, Bm, Cm)], A


@pytest.mark.parametrize("Bt,L,H,seg,dt_scale,dtype", [
    (2, 512, 3, 128, 0.1, torch.bfloat16),
    (1, 1024, 2, 256, 0.1, torch.bfloat16),
    (1, 384, 2, 128, 2.0, torch.bfloat16),   # strong decay: exponents far below zero
    (1, 256, 2, 128, 0.1, torch.float16),
])
def test_chunk_forward_matches_oracle(cuda_dev, Bt, L, H, seg, dt_scale, dtype):
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    lib = Lm.load()
    (u, delta, Bm, Cm), A = _inputs(Bt, L, H, seed=L + H, dt_scale=dt_scale, dtype=dtype)
    dev = [t.to(cuda_dev).contiguous() for t in (u, delta, Bm, Cm)]
    A_d = A.to(cuda_dev).float().contiguous()
    y = torch.full((Bt, L, H, 64), float("nan"), device=cuda_dev)
    ck = torch.full((Bt, L // seg, H, 128, 64), float("nan"), device=cuda_dev)
    lib.mr_device_error_status(1)
    Lm.call("mr_ssd_fwd", *(Lm.ptr(t) for t in dev), Lm.ptr(A_d), 1, 0, Lm.DTYPE_CODE[dtype],
            Bt, L, H, 64, 128, seg, Lm.ptr(y), Lm.ptr(ck), Lm.stream_of(cuda_dev))
    torch.cuda.synchronize()
    assert lib.mr_device_error_status(1) == 0
    ins = [t.double().numpy() for t in (u, delta, Bm, Cm)]
    A_full = np.repeat(A.double().numpy()[:, None], 128, axis=1)
    yo, cko = _oracle_states(*ins, A_full, seg)
    assert K.rel_err(y.double().cpu().numpy(), yo) < 2e-2
    assert K.rel_err(ck.double().cpu().numpy(), cko) < 2e-2
    # the float32 state carried across chunks stays tight
    assert K.rel_err(ck[:, -1].double().cpu().numpy(), cko[:, -1]) < 5e-3


@pytest.mark.parametrize("Bt,L,H,dt_scale,with_final,dtype", [
    (2, 512, 3, 0.1, True, torch.bfloat16),
    (1, 384, 2, 2.0, False, torch.bfloat16),
    (1, 256, 2, 0.1, True, torch.float16),
    (1, 256, 16, 0.1, True, torch.bfloat16),  # H % 8 == 0: delta arrives by TMA
])
def test_chunk_backward_matches_oracle(cuda_dev, Bt, L, H, dt_scale, with_final, dtype):
    """Every gradient of <y, gy> + <final, g_final>; grad_A as the per-head
    total (the sum of its row), which is the derivative for a per-head rate."""
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    lib = Lm.load()
    seg = 128
    (u, delta, Bm, Cm), A = _inputs(Bt, L, H, seed=7 * L + H, dt_scale=dt_scale, dtype=dtype)
    g = torch.Generator().manual_seed(11)
    gy = torch.randn(Bt, L, H, 64, generator=g)
    gf = torch.randn(Bt, H, 64, 128, generator=g) if with_final else None
    dev = [t.to(cuda_dev).contiguous() for t in (u, delta, Bm, Cm)]
    A_d = A.to(cuda_dev).float().contiguous()
    y = torch.empty((Bt, L, H, 64), device=cuda_dev)
    ck = torch.empty((Bt, L // seg, H, 128, 64), device=cuda_dev)
    code = Lm.DTYPE_CODE[dtype]
    Lm.call("mr_ssd_fwd", *(Lm.ptr(t) for t in dev), Lm.ptr(A_d), 1, 0, code, Bt, L, H, 64, 128, seg,
            Lm.ptr(y), Lm.ptr(ck), Lm.stream_of(cuda_dev))
    grads = [torch.full_like(t, float("nan")) for t in dev]
    gA = torch.full((H, 128), float("nan"), device=cuda_dev)
    nws = lib.mr_ssd_bwd_workspace_bytes(code, Bt, L, H, 64, 128, seg, 0)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda_dev)
    gy_d = gy.to(cuda_dev)
    gf_d = None if gf is None else gf.to(cuda_dev).contiguous()
    lib.mr_device_error_status(1)
    Lm.call("mr_ssd_bwd", Lm.ptr(gy_d), Lm.ptr(gf_d), Lm.ptr(ck), *(Lm.ptr(t) for t in dev), Lm.ptr(A_d), 1, 0,
            code, Bt, L, H, 64, 128, seg, *(Lm.ptr(t) for t in grads), Lm.ptr(gA), Lm.ptr(ws), ws.numel(),
            Lm.stream_of(cuda_dev))
    torch.cuda.synchronize()
    assert lib.mr_device_error_status(1) == 0
    ins = [t.double().numpy() for t in (u, delta, Bm, Cm)]
    A_full = np.repeat(A.double().numpy()[:, None], 128, axis=1)
    ref = K.oracle_bwd("ssd", ins + [A_full], gy.double().numpy(),
                       None if gf is None else gf.double().numpy())
    for name, got, r in zip(("u", "delta", "B", "C"), grads, ref[:4]):
        err = K.rel_err(got.double().cpu().numpy(), r)
        assert err < 2e-2, f"grad_{name}: {err:.2e}"
    err = K.rel_err(gA.double().cpu().numpy().sum(1), ref[4].sum(1))
    assert err < 2e-2, f"grad_A (per head): {err:.2e}"
