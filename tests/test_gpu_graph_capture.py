"""A forward+backward step of the plug-ins captured in a CUDA graph and replayed.

For shapes as small as BASELINE's c0 and c1 the step is bound by host work
(Python, autograd, driver calls), which a caller removes by capturing the step
once and replaying it. Every call the wrappers make must then be legal under
stream capture: kernel launches and copies on the capturing stream, workspaces
from the graph's memory pool, no synchronisation. Each case here captures the
step through the public API, replays it on new inputs copied into the static
buffers, and compares the outputs and every gradient with an eager step on the
same inputs, bit for bit (the same kernels in the same order).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cases(mr, dev):
    g = torch.Generator(device="cpu").manual_seed(3)

    def rnd(*shape, dtype=torch.bfloat16, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dtype).to(dev)

    def gla():
        Bt, L, H, Dh = 2, 256, 4, 64
        q, k, v = (rnd(Bt, L, H, Dh, scale=Dh ** -0.5) for _ in range(3))
        gates = torch.sigmoid(torch.randn(Bt, L, H, generator=g) + 2.0).to(torch.bfloat16).to(dev)
        return (q, k, v, gates), lambda q, k, v, gt: mr.gla_scan(q, k, v, gt, seg=32)

    def ssd_chunk():
        Bt, L, H, Dh, N = 1, 256, 2, 64, 128
        u, Bm, Cm = rnd(Bt, L, H, Dh), rnd(Bt, L, H, N), rnd(Bt, L, H, N)
        delta = (torch.randn(Bt, L, H, generator=g).abs() * 0.1 + 0.01).to(torch.bfloat16).to(dev)
        A = (-torch.exp(torch.randn(H, generator=g) * 0.5)).to(dev)
        return (u, delta, Bm, Cm, A), lambda u, d, b, c, a: mr.ssd_scan(u, d, b, c, a[:, None].expand(-1, N), seg=32)

    def ssd_fp32():  # the per-step kernels
        Bt, L, H, Dh, N = 2, 128, 3, 64, 16
        f = torch.float32
        u, Bm, Cm = rnd(Bt, L, H, Dh, dtype=f), rnd(Bt, L, H, N, dtype=f), rnd(Bt, L, H, N, dtype=f)
        delta = (torch.randn(Bt, L, H, generator=g).abs() * 0.1 + 0.01).to(dev)
        A = (-torch.exp(torch.randn(H, N, generator=g) * 0.5)).to(dev)
        return (u, delta, Bm, Cm, A), lambda u, d, b, c, a: mr.ssd_scan(u, d, b, c, a, seg=32)

    def rglru():
        Bt, L, D = 2, 256, 128
        a = torch.sigmoid(torch.randn(Bt, L, D, generator=g) + 3.0).to(torch.bfloat16).to(dev)
        x = rnd(Bt, L, D)
        return (a, x), lambda a, x: mr.rglru_scan(a, x, seg=32)

    return {"gla": gla, "ssd_chunk": ssd_chunk, "ssd_fp32": ssd_fp32, "rglru": rglru}


@pytest.mark.parametrize("name", ["gla", "ssd_chunk", "ssd_fp32", "rglru"])
def test_step_replays_from_a_cuda_graph(mr, cuda_dev, name):
    ins, fn = _cases(mr, cuda_dev)[name]()
    gy = torch.randn(fn(*ins).shape, device=cuda_dev)

    def step(xs):
        leaves = [x.detach().requires_grad_(x.is_floating_point()) for x in xs]
        y = fn(*leaves)
        grads = torch.autograd.grad(y, [l for l in leaves if l.requires_grad], gy)
        return [y.detach()] + list(grads)

    static = [x.clone() for x in ins]
    side = torch.cuda.Stream(cuda_dev)
    side.wait_stream(torch.cuda.current_stream(cuda_dev))
    with torch.cuda.stream(side):  # warm-up outside the capture, as torch.cuda.graphs asks
        for _ in range(2):
            step(static)
    torch.cuda.current_stream(cuda_dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = step(static)
    # new inputs through the static buffers, then one replay
    fresh = [x.roll(1, dims=1) if x.dim() >= 2 and x.shape[1] > 1 else x for x in ins]
    for s, x in zip(static, fresh):
        s.copy_(x)
    graph.replay()
    torch.cuda.synchronize()
    ref = step(fresh)
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(outs, ref)):
        assert torch.equal(a, b), f"{name}: output {i} differs between the replay and an eager step"
