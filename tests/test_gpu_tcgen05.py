"""tcgen05 building blocks: every shared-memory operand form used by the
chunked kernels, on one 128x128x128 bf16 tile, against a float64 matmul."""

import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_umma_operand_forms(cuda_dev):
    L = importlib.import_module("mlx-recurrence_b200._lib")
    lib = L.load()
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    A = torch.randn(128, 128, generator=g, device=cuda_dev).to(torch.bfloat16)
    Bk = torch.randn(128, 128, generator=g, device=cuda_dev).to(torch.bfloat16)
    Bmn = torch.randn(128, 64, generator=g, device=cuda_dev).to(torch.bfloat16)
    Amn = torch.randn(128, 128, generator=g, device=cuda_dev).to(torch.bfloat16)
    D1 = torch.full((128, 128), float("nan"), device=cuda_dev)
    D2 = torch.full((128, 64), float("nan"), device=cuda_dev)
    D3 = torch.full((128, 64), float("nan"), device=cuda_dev)
    lib.mr_device_error_status(1)
    L.call("mr_selftest_umma", *(L.ptr(t) for t in (A, Bk, Bmn, Amn, D1, D2, D3)), L.stream_of(cuda_dev))
    torch.cuda.synchronize()
    assert lib.mr_device_error_status(1) == 0
    refs = [A.double() @ Bk.double().T, A.double() @ Bmn.double(), Amn.double().T @ Bmn.double()]
    for name, got, ref in zip(("K x K", "K x MN", "MN x MN"), (D1, D2, D3), refs):
        err = float((got.double() - ref).abs().max() / ref.abs().max())
        assert err < 1e-5, f"{name}: {err:.2e}"
