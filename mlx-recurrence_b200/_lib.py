"""ctypes binding of ``libmlrec.so`` (declared in ``include/mlrec.h``).

The library is built in-tree by ``csrc/build.py`` (``__graft_entry__.build()``
runs it). There is no fallback: if the library or a CUDA sm_100 device is
missing, every scan raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmlrec.so")

MR_OK = 0
MR_E_SHAPE = 1
MR_E_DTYPE = 2
MR_E_ALIGN = 3
MR_E_LAUNCH = 4
MR_E_WORKSPACE = 5
MR_E_DEVICE = 6

MR_F32, MR_BF16, MR_F16 = 0, 1, 2
DTYPE_CODE = {torch.float32: MR_F32, torch.bfloat16: MR_BF16, torch.float16: MR_F16}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t

# argument signatures, in declaration order of include/mlrec.h
SIGNATURES = {
    "mr_abi_version": (_int, []),
    "mr_last_error": (ctypes.c_char_p, []),
    "mr_launch_count": (ctypes.c_uint64, []),
    "mr_device_error_status": (_int, [_int]),
    "mr_selftest_umma": (_int, [_p, _p, _p, _p, _p, _p, _p, _p]),
    "mr_selftest_wait_timeout": (_int, [_int, ctypes.c_uint64, _p, _p]),
    "mr_check_segment_shape": (_int, [_i64, _i64, _i64, ctypes.c_char_p]),
    "mr_ssd_fwd": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _int, _i64, _i64, _i64, _i64, _i64, _i64,
                          _p, _p, _p]),
    "mr_ssd_preferred_seg": (_i64, [_int, _i64, _i64, _i64, _i64, _i64]),
    "mr_ssd_bwd_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "mr_ssd_bwd": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _int, _i64, _i64, _i64, _i64,
                          _i64, _i64, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "mr_ssd_bwd_noalloc": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _int, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _p, _p, _p, _p, _p, _p]),
    "mr_gla_fwd": (_int, [_p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "mr_gla_preferred_seg": (_i64, [_int, _i64, _i64, _i64]),
    "mr_gla_bwd_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64, _i64]),
    "mr_gla_bwd": (_int, [_p, _p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _i64, _p, _p, _p,
                          _p, _p, _sz, _p]),
    "mr_rglru_fwd": (_int, [_p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "mr_rglru_bwd_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64]),
    "mr_rglru_bwd": (_int, [_p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _sz, _p]),
    "mr_rotlru_fwd": (_int, [_p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "mr_rotlru_bwd_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64]),
    "mr_rotlru_bwd": (_int, [_p, _p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _p,
                             _p, _sz, _p]),
    # initial-state variants: (h0) before the stream (forward), (h0, grad_h0) backward
    "mr_ssd_fwd_h0": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _int, _i64, _i64, _i64, _i64, _i64, _i64,
                             _p, _p, _p, _p]),
    "mr_ssd_bwd_h0": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _int, _i64, _i64, _i64, _i64,
                             _i64, _i64, _p, _p, _p, _p, _p, _p, _sz, _p, _p, _p]),
    "mr_gla_fwd_h0": (_int, [_p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "mr_gla_bwd_h0": (_int, [_p, _p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _i64, _p, _p, _p,
                             _p, _p, _sz, _p, _p, _p]),
    "mr_rglru_fwd_h0": (_int, [_p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "mr_rglru_bwd_h0": (_int, [_p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _sz, _p, _p,
                               _p]),
    "mr_rotlru_fwd_h0": (_int, [_p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "mr_rotlru_bwd_h0": (_int, [_p, _p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _p,
                                _p, _sz, _p, _p, _p]),
    # the RG-LRU scan with its input gating folded in
    "mr_rglru_gated_fwd": (_int, [_p, _p, _p, _p, ctypes.c_float, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "mr_rglru_gated_bwd_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64]),
    "mr_rglru_gated_bwd": (_int, [_p, _p, _p, _p, _p, _p, _p, ctypes.c_float, _int, _i64, _i64, _i64, _i64, _p,
                                  _p, _p, _p, _p, _sz, _p, _p, _p]),
    # the rotLRU scan taking the rotation angle (cos, sin formed in the kernels)
    "mr_rotlru_angle_fwd": (_int, [_p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "mr_rotlru_angle_bwd": (_int, [_p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _sz,
                                   _p, _p, _p]),
    # Gated DeltaNet (per-step form, segment checkpoints)
    "mr_gdn_fwd": (_int, [_p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _sz, _p]),
    "mr_gdn_fwd_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64, _i64]),
    "mr_gdn_bwd_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _i64, _i64]),
    "mr_gdn_step": (_int, [_p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _p, _p, _p]),
    "mr_gdn_bwd": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _int, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p,
                          _p, _sz, _p, _p, _p]),
    # one-token decode steps (state advanced in place)
    "mr_ssd_step": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _int, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "mr_gla_step": (_int, [_p, _p, _p, _p, _int, _i64, _i64, _i64, _p, _p, _p]),
    "mr_rglru_step": (_int, [_p, _p, _int, _i64, _i64, _p, _p, _p]),
    "mr_rotlru_step": (_int, [_p, _p, _p, _p, _int, _i64, _i64, _p, _p, _p]),
}

_lib = None
_lock = threading.Lock()


class MrError(RuntimeError):
    """A libmlrec entry point returned a nonzero status."""

    def __init__(self, code, msg):
        super().__init__(f"libmlrec error {code}: {msg}")
        self.code = code


def load():
    """Load (once) and return the ctypes handle of libmlrec.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python {_HERE}/csrc/build.py` "
                    "(or __graft_entry__.build())")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name, *args):
    """Call an entry point; raise ValueError for shape errors (the reference's
    exception type, ``_chassis.py:104-115``) and MrError otherwise."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != MR_OK:
        msg = lib.mr_last_error().decode()
        if rc == MR_E_SHAPE:
            raise ValueError(msg)
        raise MrError(rc, msg)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    """The scans run only on CUDA tensors of one sm_100 device."""
    dev = tensors[0].device
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise RuntimeError("mlx-recurrence_b200 scans need CUDA tensors on a B200 (sm_100); "
                               "there is no CPU path")
        if t.device != dev:
            raise RuntimeError("all scan inputs must be on the same CUDA device")
    major, _ = torch.cuda.get_device_capability(dev)
    if major != 10:
        raise RuntimeError(f"libmlrec is built for sm_100a; device {dev} is sm_{major}x")
    return dev
