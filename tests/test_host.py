"""Host-side behaviour that needs no GPU: shape rules and messages, the C-ABI
library's exports and host-only entry points, the public API surface, and
that there is no CPU fallback."""

import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mlrec.h")


def _declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MR_API\s+[\w\s\*]+?\b(mr_\w+)\s*\(", text)))


def test_header_declares_every_entry_point():
    syms = _declared_symbols()
    for s in ("mr_ssd_fwd", "mr_ssd_bwd", "mr_gla_fwd", "mr_gla_bwd", "mr_rglru_fwd",
              "mr_rglru_bwd", "mr_rotlru_fwd", "mr_rotlru_bwd", "mr_last_error", "mr_abi_version",
              "mr_check_segment_shape"):
        assert s in syms


def test_library_loads_and_exports_every_declared_symbol(mr):
    from importlib import import_module
    lib_mod = import_module("mlx-recurrence_b200._lib")
    lib = lib_mod.load()
    for s in _declared_symbols():
        assert hasattr(lib, s), s
        assert s in lib_mod.SIGNATURES, s
    assert lib.mr_abi_version() == 7


def test_c_abi_shape_check_messages(mr):
    from importlib import import_module
    L = import_module("mlx-recurrence_b200._lib").load()
    assert L.mr_check_segment_shape(64, 32, 64, b"Dh") == 0
    assert L.mr_check_segment_shape(30, 32, 64, b"Dh") == 1
    assert b"must be divisible by seg=32" in L.mr_last_error()
    assert L.mr_check_segment_shape(64, 32, 16, b"Dh") == 1
    assert b"Dh=16 must be a multiple of 32" in L.mr_last_error()
    assert L.mr_check_segment_shape(64, 0, 64, b"D") == 1
    assert b"seg must be positive" in L.mr_last_error()


def test_c_abi_rejects_bad_arguments_before_launch(mr):
    """Shape, dtype and null-pointer errors come back as status codes with no
    device work (pointers here are never dereferenced)."""
    from importlib import import_module
    lm = import_module("mlx-recurrence_b200._lib")
    L = lm.load()
    p = ctypes.c_void_p(16)
    # L % seg != 0
    rc = L.mr_rglru_fwd(p, p, 1, 2, 30, 64, 32, p, p, None)
    assert rc == lm.MR_E_SHAPE
    # bad dtype
    rc = L.mr_rglru_fwd(p, p, 7, 2, 64, 64, 32, p, p, None)
    assert rc == lm.MR_E_DTYPE
    # misaligned pointer
    rc = L.mr_rglru_fwd(ctypes.c_void_p(18), p, 1, 2, 64, 64, 32, p, p, None)
    assert rc == lm.MR_E_ALIGN
    # SSD head dim not a multiple of 32
    rc = L.mr_ssd_fwd(p, p, p, p, p, 8, 1, 1, 1, 32, 2, 16, 8, 32, p, p, None)
    assert rc == lm.MR_E_SHAPE and b"Dh=16" in L.mr_last_error()
    # missing workspace
    rc = L.mr_ssd_bwd(p, None, p, p, p, p, p, p, 8, 1, 1, 1, 64, 2, 64, 8, 32, p, p, p, p, p, None, 0, None)
    assert rc == lm.MR_E_WORKSPACE


def test_workspace_sizes_are_host_only(mr):
    from importlib import import_module
    L = import_module("mlx-recurrence_b200._lib").load()
    assert L.mr_rglru_bwd_workspace_bytes(1, 8, 4096, 2560, 32) == 0
    assert L.mr_rglru_bwd_workspace_bytes(1, 8, 4096, 2560, 1024) > 0
    assert L.mr_rotlru_bwd_workspace_bytes(1, 16, 8192, 1024, 32) == 0
    assert L.mr_ssd_bwd_workspace_bytes(0, 3, 512, 12, 64, 16, 32, 1) > 0
    assert L.mr_gla_bwd_workspace_bytes(1, 3, 512, 12, 64, 32) > 0


def test_check_segment_shape_messages(mr):
    mr.check_segment_shape(64, 32, 64, "Dh")
    with pytest.raises(ValueError, match="must be divisible by seg=32"):
        mr.check_segment_shape(30, 32, 64, "Dh")
    with pytest.raises(ValueError, match="Dh=16 must be a multiple of 32"):
        mr.check_segment_shape(32, 32, 16, "Dh")
    with pytest.raises(ValueError, match="seg must be positive"):
        mr.check_segment_shape(32, 0, 32, "Dh")
    assert mr.DEFAULT_SEG == 32


def _ssd_in(B, L, H, Dh, N):
    g = torch.Generator().manual_seed(0)
    return (torch.randn(B, L, H, Dh, generator=g), torch.rand(B, L, H, generator=g) * 0.05 + 0.001,
            torch.randn(B, L, H, N, generator=g), torch.randn(B, L, H, N, generator=g),
            -torch.rand(H, N, generator=g) - 0.1)


def test_invalid_shapes_raise_value_error(mr):
    # reference: tests/test_v2_ssd.py:63-72, test_v2_gla.py:56-63, test_v2_rglru.py:54-61
    with pytest.raises(ValueError):
        mr.ssd_scan(*_ssd_in(1, 30, 2, 32, 8), seg=32)
    with pytest.raises(ValueError):
        mr.ssd_scan(*_ssd_in(1, 32, 2, 16, 8), seg=32)
    q = torch.randn(1, 30, 2, 32)
    with pytest.raises(ValueError):
        mr.gla_scan(q, q, q, torch.rand(1, 30, 2), seg=32)
    q = torch.randn(1, 32, 2, 16)
    with pytest.raises(ValueError):
        mr.gla_scan(q, q, q, torch.rand(1, 32, 2), seg=32)
    with pytest.raises(ValueError):
        mr.rglru_scan(torch.rand(1, 30, 32), torch.rand(1, 30, 32), seg=32)
    with pytest.raises(ValueError):
        mr.rglru_scan(torch.rand(1, 32, 16), torch.rand(1, 32, 16), seg=32)


def test_rotlru_constraint_violations_raise(mr):
    # reference: tests/test_v2_rotlru.py:126-135
    def inp(B, L, Dp):
        return torch.rand(B, L, Dp), torch.rand(B, L, Dp), torch.rand(B, L, Dp), torch.rand(B, L, 2 * Dp)
    with pytest.raises(ValueError):
        mr.rotlru_scan(*inp(1, 48, 16))
    with pytest.raises(ValueError):
        mr.rotlru_scan(*inp(1, 64, 8))
    a, cs, sn, x = inp(1, 64, 16)
    with pytest.raises(ValueError, match=r"x must be \[B, L, 2\*Dp\]"):
        mr.rotlru_scan(a, cs, sn, x[:, :, :-2])


def test_no_cpu_fallback(mr):
    """Valid CPU inputs are refused: the scans run only through libmlrec on a GPU."""
    with pytest.raises(RuntimeError, match="CUDA"):
        mr.rglru_scan(torch.rand(1, 32, 32), torch.rand(1, 32, 32))
    with pytest.raises(RuntimeError, match="CUDA"):
        mr.ssd_scan(*_ssd_in(1, 32, 2, 32, 8))


def test_public_api_matches_reference_v2_names(mr):
    for name in ("ssd_scan", "ssd_scan_with_state", "ssd_scan_reference", "gla_scan",
                 "gla_scan_with_state", "gla_scan_reference", "rglru_scan", "rglru_scan_with_state",
                 "rglru_scan_reference", "rotlru_scan", "rotlru_scan_with_state",
                 "rotlru_scan_reference", "DEFAULT_SEG", "get_or_build_kernel",
                 "check_segment_shape", "parity_check"):
        assert hasattr(mr, name), name


def test_reference_loops_match_oracle_on_cpu(mr):
    """The package's per-step *_reference functions equal the oracle (float64)."""
    import numpy as np
    import ref_loops as R
    u, d, B, C, A = [t.double() for t in _ssd_in(2, 16, 2, 32, 4)]
    y = mr.ssd_scan_reference(u, d, B, C, A).numpy()
    yo, _ = R.ssd_forward(u.numpy(), d.numpy(), B.numpy(), C.numpy(), A.numpy())
    assert np.max(np.abs(y - yo)) < 1e-12


def test_gdn_backward_workspace_is_bounded(mr):
    """Long Gated DeltaNet segments (few checkpoints) do not grow the backward's
    scratch past its budget: the CTAs walk more units instead."""
    from importlib import import_module
    lib = import_module("mlx-recurrence_b200._lib").load()
    small = lib.mr_gdn_bwd_workspace_bytes(1, 32, 2048, 32, 64, 64)
    huge = lib.mr_gdn_bwd_workspace_bytes(1, 32, 65536, 32, 64, 65536)
    assert small == 1024 * 16 * 64 * 64 * 4
    assert 0 < huge <= (1 << 30)
