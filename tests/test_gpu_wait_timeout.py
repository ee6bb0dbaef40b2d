"""Bounded waits give up, report, and leave the context usable.

The chunked kernels wait on shared-memory barriers for their TMA copies. A
wait that runs out records a device error word and returns; once the word is
set, every later wait gives up at once, so a kernel whose copies stopped
arriving ends after about one time limit. The self-test kernel waits on a
barrier that nothing completes (no copy is in flight, nothing faults), first
with a short limit, then with the standard 2 s limit, in many CTAs at once.
"""

import importlib

import numpy as np
import pytest
import torch

import _cases as K

pytestmark = pytest.mark.gpu


def test_wait_runs_out_sets_the_error_word_and_later_waits_fail_fast(mr, cuda_dev):
    L = importlib.import_module("mlx-recurrence_b200._lib")
    lib = L.load()
    torch.cuda.synchronize()
    assert lib.mr_device_error_status(1) == 0
    ctas, limit_ns = 296, 20_000_000
    out = torch.zeros(2 * ctas, dtype=torch.int64, device=cuda_dev)
    L.call("mr_selftest_wait_timeout", ctas, limit_ns, L.ptr(out), L.stream_of(cuda_dev))
    torch.cuda.synchronize()
    ns = out.cpu().numpy().reshape(ctas, 2)
    first, second = ns[:, 0], ns[:, 1]
    # some wait ran out its own limit; none ran much past it
    assert first.max() >= 0.9 * limit_ns
    assert first.max() < limit_ns + 200_000_000
    # every wait after the word was set gave up at once, far inside its 2 s limit
    assert second.max() < 20_000_000, second.max()
    assert lib.mr_device_error_status(1) == 1
    assert lib.mr_device_error_status(0) == 0
    # the context is still usable: a scan runs and matches the oracle
    rng = np.random.default_rng(3)
    a = rng.uniform(-0.99, 0.99, (2, 64, 64))
    x = rng.standard_normal((2, 64, 64))
    y = mr.rglru_scan(torch.tensor(a, dtype=torch.float32, device=cuda_dev),
                      torch.tensor(x, dtype=torch.float32, device=cuda_dev))
    yo, _ = K.oracle_fwd("rglru", [a.astype(np.float32).astype(np.float64), x.astype(np.float32).astype(np.float64)])
    assert K.rel_err(y.double().cpu().numpy(), yo) < 1e-5
    assert lib.mr_device_error_status(1) == 0
