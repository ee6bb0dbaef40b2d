"""mlx-recurrence for NVIDIA B200: the four v2 linear-recurrence scan plug-ins
of mlx-recurrence v0.3.0 (``mlx_recurrence/__init__.py:21-90``), rebuilt as
torch.autograd.Functions over a C-ABI library of sm_100a CUDA kernels
(``libmlrec.so``, ABI in ``include/mlrec.h``).

    ssd     - Mamba-2-style head-wise SSD selective scan
    gla     - gated linear attention recurrence
    rglru   - RG-LRU diagonal recurrence
    rotlru  - rotational LRU (complex-diagonal over interleaved pairs)

Beyond the reference: an optional initial state ``h0=`` on every scan
(chunked prefill), one-token decode steps ``*_step`` on a state cache,
``rglru_scan_gated`` with the RG-LRU input gating inside the kernels,
``rotlru_scan_angle`` taking the rotation angle, and
``gated_deltanet_scan``, the recurrence the reference carries as a design
(``docs/DESIGN_gated_deltanet.md``).

Import with ``importlib.import_module("mlx-recurrence_b200")`` (the directory
name carries a hyphen); after that the package is also registered as
``mlx_recurrence_b200``.
"""

import sys as _sys

from ._chassis import DEFAULT_SEG, check_segment_shape, get_or_build_kernel, parity_check
from .gdn import (gated_deltanet_scan, gated_deltanet_scan_reference, gated_deltanet_scan_with_state,
                  gated_deltanet_step)
from .gla import gla_scan, gla_scan_reference, gla_scan_with_state, gla_step
from .rglru import (rglru_scan, rglru_scan_gated, rglru_scan_gated_with_state, rglru_scan_reference,
                    rglru_scan_with_state, rglru_step)
from .rotlru import (rotlru_scan, rotlru_scan_angle, rotlru_scan_angle_with_state, rotlru_scan_reference,
                     rotlru_scan_with_state, rotlru_step)
from .ssd import ssd_scan, ssd_scan_reference, ssd_scan_with_state, ssd_step

__all__ = [
    "ssd_scan",
    "ssd_scan_with_state",
    "ssd_scan_reference",
    "gla_scan",
    "gla_scan_with_state",
    "gla_scan_reference",
    "rglru_scan",
    "rglru_scan_with_state",
    "rglru_scan_reference",
    "rotlru_scan",
    "rotlru_scan_with_state",
    "rotlru_scan_reference",
    "rotlru_scan_angle",
    "rotlru_scan_angle_with_state",
    # the RG-LRU scan with its input gating in the kernels (not in the reference)
    "rglru_scan_gated",
    "rglru_scan_gated_with_state",
    # Gated DeltaNet (a design only in the reference)
    "gated_deltanet_scan",
    "gated_deltanet_scan_with_state",
    "gated_deltanet_scan_reference",
    # one-token decode steps on a float32 state cache (not in the reference)
    "ssd_step",
    "gla_step",
    "rglru_step",
    "rotlru_step",
    "gated_deltanet_step",
    "DEFAULT_SEG",
    "get_or_build_kernel",
    "check_segment_shape",
    "parity_check",
]

__version__ = "0.3.0+b200.1"

_sys.modules.setdefault("mlx_recurrence_b200", _sys.modules[__name__])
