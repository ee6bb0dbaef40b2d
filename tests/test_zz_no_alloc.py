"""The allocation-free SSD backward (mr_ssd_bwd_noalloc).

It serves callers that cannot allocate device memory while the backward runs
(code inside an allocator's callback, where allocating would re-enter the
allocator, or embedders that own all device memory and hand over only
pre-placed buffers): instead of a caller-provided workspace it uses a built-in device
array. The GPU test calls it through the C-ABI twice in a row and checks each
result against the workspace-taking mr_ssd_bwd on the same inputs. This file
is collected last so that a failure here comes after every other test ran.
"""

import ctypes
import importlib

import pytest
import torch

import _cases as K


def _lib():
    L = importlib.import_module("mlx-recurrence_b200._lib")
    return L, L.load()


def test_no_alloc_rejects_problems_beyond_its_scratch():
    """batch*H above 65,536 is refused before any device work."""
    L, lib = _lib()
    p = ctypes.c_void_p(256)
    rc = lib.mr_ssd_bwd_noalloc(p, None, p, p, p, p, p, p, 1, 0, L.MR_BF16, 65535, 128, 2, 64, 128, 128,
                                p, p, p, p, p, None)
    assert rc == L.MR_E_WORKSPACE
    assert b"exceeds the built-in scratch" in lib.mr_last_error()


@pytest.mark.gpu
def test_no_alloc_backward_matches_workspace_backward(cuda_dev):
    L, lib = _lib()
    Bt, Lq, H, Dh, N, seg = 2, 384, 3, 64, 128, 128
    g = torch.Generator().manual_seed(5)
    u = torch.randn(Bt, Lq, H, Dh, generator=g).to(torch.bfloat16)
    delta = (torch.randn(Bt, Lq, H, generator=g).abs() * 0.1 + 0.01).to(torch.bfloat16)
    Bm = torch.randn(Bt, Lq, H, N, generator=g).to(torch.bfloat16)
    Cm = torch.randn(Bt, Lq, H, N, generator=g).to(torch.bfloat16)
    A = -torch.exp(torch.randn(H, generator=g) * 0.5)
    gy = torch.randn(Bt, Lq, H, Dh, generator=g)
    gf = torch.randn(Bt, H, Dh, N, generator=g)
    dev = [t.to(cuda_dev).contiguous() for t in (u, delta, Bm, Cm)]
    A_d, gy_d, gf_d = A.to(cuda_dev), gy.to(cuda_dev), gf.to(cuda_dev)
    st = L.stream_of(cuda_dev)
    y = torch.empty(Bt, Lq, H, Dh, device=cuda_dev)
    ck = torch.empty(Bt, Lq // seg, H, N, Dh, device=cuda_dev)
    L.call("mr_ssd_fwd", *(L.ptr(t) for t in dev), L.ptr(A_d), 1, 0, L.MR_BF16, Bt, Lq, H, Dh, N, seg,
           L.ptr(y), L.ptr(ck), st)

    def grads_like():
        return [torch.full_like(t, float("nan")) for t in dev] + [torch.full((H, N), float("nan"), device=cuda_dev)]

    ref = grads_like()
    nws = lib.mr_ssd_bwd_workspace_bytes(L.MR_BF16, Bt, Lq, H, Dh, N, seg, 0)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda_dev)
    L.call("mr_ssd_bwd", L.ptr(gy_d), L.ptr(gf_d), L.ptr(ck), *(L.ptr(t) for t in dev), L.ptr(A_d), 1, 0,
           L.MR_BF16, Bt, Lq, H, Dh, N, seg, *(L.ptr(t) for t in ref), L.ptr(ws), ws.numel(), st)
    for _ in range(2):  # two calls in a row share the built-in scratch
        got = grads_like()
        L.call("mr_ssd_bwd_noalloc", L.ptr(gy_d), L.ptr(gf_d), L.ptr(ck), *(L.ptr(t) for t in dev), L.ptr(A_d),
               1, 0, L.MR_BF16, Bt, Lq, H, Dh, N, seg, *(L.ptr(t) for t in got), st)
        torch.cuda.synchronize()
        assert lib.mr_device_error_status(1) == 0
        for name, a, b in zip(("u", "delta", "B", "C", "A"), got, ref):
            err = K.rel_err(a.double().cpu().numpy(), b.double().cpu().numpy())
            assert err < 2e-2, f"grad_{name}: {err:.2e}"
