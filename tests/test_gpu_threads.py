"""Entry points called from a host thread that has made no CUDA call yet (as
torch's autograd worker threads can be, when every allocation they make is
served from the caching allocator): the tensor-map encoder needs the thread's
device context, which the library binds itself."""

import importlib
import threading

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_rglru_from_fresh_thread(cuda_dev):
    Lm = importlib.import_module("mlx-recurrence_b200._lib")
    g = torch.Generator().manual_seed(5)
    Bt, L, D, seg = 2, 512, 256, 64
    a = torch.rand(Bt, L, D, generator=g).mul(0.5).add(0.45).to(torch.bfloat16).to(cuda_dev)
    x = torch.randn(Bt, L, D, generator=g).to(torch.bfloat16).to(cuda_dev)
    outs = {}
    for name in ("main", "thread"):
        outs[name] = (torch.full((Bt, L, D), float("nan"), device=cuda_dev),
                      torch.full((Bt, L // seg, D), float("nan"), device=cuda_dev))
    stream = Lm.stream_of(cuda_dev)
    torch.cuda.synchronize()

    def run(name):
        y, ck = outs[name]
        Lm.call("mr_rglru_fwd", Lm.ptr(a), Lm.ptr(x), 1, Bt, L, D, seg, Lm.ptr(y), Lm.ptr(ck), stream)

    run("main")
    errors = []

    def worker():
        try:
            run("thread")
        except Exception as e:  # reported below, on the test's thread
            errors.append(e)

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert not errors, errors
    torch.cuda.synchronize()
    assert torch.equal(outs["main"][0], outs["thread"][0])
    assert torch.equal(outs["main"][1], outs["thread"][1])
