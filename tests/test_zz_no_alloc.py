"""The allocation-free SSD backward (mr_ssd_bwd_noalloc).

It serves callers that cannot allocate device memory while the backward runs
(code inside an allocator's callback, where allocating would re-enter the
allocator, or embedders that own all device memory and hand over only
pre-placed buffers): instead of a caller-provided workspace it uses a built-in device
array. The GPU test calls it through the C-ABI twice in a row and checks each
result against the workspace-taking mr_ssd_bwd on the same inputs: the two run
the same kernels on the same per-(batch row, head) partials with no atomics,
so they must agree bit for bit. A larger problem runs first, so stale entries
of the shared array would show. This file is collected last so that a failure
here comes after every other test ran.
"""

import ctypes
import importlib

import pytest
import torch


def _lib():
    L = importlib.import_module("mlx-recurrence_b200._lib")
    return L, L.load()


def _call_args(L, Bt, H):
    p = ctypes.c_void_p(256)
    return (p, None, p, p, p, p, p, p, 1, 0, L.MR_BF16, Bt, 128, H, 64, 128, 128, p, p, p, p, p, None)


def test_no_alloc_rejects_problems_beyond_its_scratch():
    """batch*H above 65,536 is refused before any device work."""
    L, lib = _lib()
    rc = lib.mr_ssd_bwd_noalloc(*_call_args(L, 65535, 2))
    assert rc == L.MR_E_WORKSPACE
    assert b"exceeds the built-in scratch" in lib.mr_last_error()


@pytest.mark.skipif(torch.cuda.is_available(), reason="host-only: on a GPU the call would launch on fake pointers")
def test_no_alloc_accepts_its_largest_problem():
    """batch*H == 65,536 passes the size check; without a GPU the call then
    stops at the device lookup (MR_E_DEVICE), before any launch."""
    L, lib = _lib()
    rc = lib.mr_ssd_bwd_noalloc(*_call_args(L, 32768, 2))
    assert rc != L.MR_E_WORKSPACE, lib.mr_last_error()
    assert rc == L.MR_E_DEVICE


def _problem(cuda_dev, Bt, Lq, H, seed):
    Dh, N, seg = 64, 128, 128
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(Bt, Lq, H, Dh, generator=g).to(torch.bfloat16)
    delta = (torch.randn(Bt, Lq, H, generator=g).abs() * 0.1 + 0.01).to(torch.bfloat16)
    Bm = torch.randn(Bt, Lq, H, N, generator=g).to(torch.bfloat16)
    Cm = torch.randn(Bt, Lq, H, N, generator=g).to(torch.bfloat16)
    A = -torch.exp(torch.randn(H, generator=g) * 0.5)
    gy = torch.randn(Bt, Lq, H, Dh, generator=g)
    gf = torch.randn(Bt, H, Dh, N, generator=g)
    dev = [t.to(cuda_dev).contiguous() for t in (u, delta, Bm, Cm)]
    return dict(Bt=Bt, Lq=Lq, H=H, Dh=Dh, N=N, seg=seg, dev=dev, A=A.to(cuda_dev), gy=gy.to(cuda_dev),
                gf=gf.to(cuda_dev))


def _forward(L, P, st):
    y = torch.empty(P["Bt"], P["Lq"], P["H"], P["Dh"], device=P["A"].device)
    ck = torch.empty(P["Bt"], P["Lq"] // P["seg"], P["H"], P["N"], P["Dh"], device=P["A"].device)
    L.call("mr_ssd_fwd", *(L.ptr(t) for t in P["dev"]), L.ptr(P["A"]), 1, 0, L.MR_BF16, P["Bt"], P["Lq"], P["H"],
           P["Dh"], P["N"], P["seg"], L.ptr(y), L.ptr(ck), st)
    return ck


def _grads_like(P):
    return [torch.full_like(t, float("nan")) for t in P["dev"]] + \
        [torch.full((P["H"], P["N"]), float("nan"), device=P["A"].device)]


def _noalloc(L, P, ck, st):
    got = _grads_like(P)
    L.call("mr_ssd_bwd_noalloc", L.ptr(P["gy"]), L.ptr(P["gf"]), L.ptr(ck), *(L.ptr(t) for t in P["dev"]),
           L.ptr(P["A"]), 1, 0, L.MR_BF16, P["Bt"], P["Lq"], P["H"], P["Dh"], P["N"], P["seg"],
           *(L.ptr(t) for t in got), st)
    return got


@pytest.mark.gpu
def test_no_alloc_backward_matches_workspace_backward(cuda_dev):
    L, lib = _lib()
    st = L.stream_of(cuda_dev)
    big = _problem(cuda_dev, 4, 256, 5, seed=9)       # 20 units: fills more of the shared array
    P = _problem(cuda_dev, 2, 384, 3, seed=5)         # 6 units: the compared problem
    ck_big = _forward(L, big, st)
    ck = _forward(L, P, st)
    ref = _grads_like(P)
    nws = lib.mr_ssd_bwd_workspace_bytes(L.MR_BF16, P["Bt"], P["Lq"], P["H"], P["Dh"], P["N"], P["seg"], 0)
    ws = torch.empty(max(nws, 16), dtype=torch.uint8, device=cuda_dev)
    L.call("mr_ssd_bwd", L.ptr(P["gy"]), L.ptr(P["gf"]), L.ptr(ck), *(L.ptr(t) for t in P["dev"]), L.ptr(P["A"]),
           1, 0, L.MR_BF16, P["Bt"], P["Lq"], P["H"], P["Dh"], P["N"], P["seg"], *(L.ptr(t) for t in ref),
           L.ptr(ws), ws.numel(), st)
    lib.mr_device_error_status(1)
    _noalloc(L, big, ck_big, st)  # leaves its own partials in the shared array
    for _ in range(2):  # two calls in a row share the built-in scratch
        got = _noalloc(L, P, ck, st)
        torch.cuda.synchronize()
        assert lib.mr_device_error_status(1) == 0
        for name, a, b in zip(("u", "delta", "B", "C", "A"), got, ref):
            assert not torch.isnan(b).any(), f"grad_{name}: reference has NaN"
            assert torch.equal(a, b), f"grad_{name}: differs from mr_ssd_bwd"
