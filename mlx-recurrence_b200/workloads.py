"""Seeded synthetic inputs for the benchmark configurations c0-c4.

The reference measures on no public dataset; these generators draw inputs
with the shapes and value distributions of its published configurations
(from the reference's own test inputs and
``docs/validation``). A rank's shard is a contiguous batch range
(``shard_batch``) generated with its own seed and ``batch=`` its size.
"""

from __future__ import annotations

import math

import torch

from .sharding import block_of, shard_batch  # noqa: F401  (re-exported for bench.py)

CONFIGS = {
    "c0": dict(kind="ssd", B=3, L=512, H=12, Dh=64, N=16, seg=32, dtype=torch.float32),
    "c1": dict(kind="gla", B=3, L=512, H=12, Dh=64, seg=32, dtype=torch.bfloat16),
    "c2": dict(kind="rglru", B=8, L=4096, D=2560, seg=32, dtype=torch.bfloat16),
    "c3": dict(kind="rotlru", B=16, L=8192, Dp=1024, seg=32, dtype=torch.bfloat16),
    "c4": dict(kind="ssd", B=32, L=16384, H=32, Dh=64, N=128, seg=32, dtype=torch.bfloat16),
    # c4 with a dense per-(head, state) decay A_neg [H, N] (the reference's general contract,
    # ssd.py:62, 96): the float32 per-step kernels
    "c4d": dict(kind="ssd", B=32, L=16384, H=32, Dh=64, N=128, seg=32, dtype=torch.bfloat16, dense_a=True),
    # the GLA shape of the target (SSD/GLA fwd+bwd at B=32, L=16384, H=32, Dh=64)
    "c5": dict(kind="gla", B=32, L=16384, H=32, Dh=64, seg=32, dtype=torch.bfloat16),
    # c2 with the RG-LRU input gating inside the kernels (x, r, i, lam in; c = 8)
    "c2g": dict(kind="rglru_gated", B=8, L=4096, D=2560, seg=32, dtype=torch.bfloat16),
    # c3 with the rotation angle in place of cos/sin (cos, sin formed in the kernels)
    "c3a": dict(kind="rotlru_angle", B=16, L=8192, Dp=1024, seg=32, dtype=torch.bfloat16),
    # Gated DeltaNet (a design only in the reference) at the unit count of c5
    "c6": dict(kind="gdn", B=32, L=2048, H=32, Dh=64, seg=64, dtype=torch.bfloat16),
}

DESCRIPTION = {
    "c0": "ssd_scan fp32 B=3 L=512 H=12 Dh=64 N=16 seg=32",
    "c1": "gla_scan bf16 B=3 L=512 H=12 Dh=64 seg=32",
    "c2": "rglru_scan bf16 B=8 L=4096 D=2560 seg=32",
    "c3": "rotlru_scan bf16 B=16 L=8192 D=2048 seg=32",
    "c4": "ssd_scan bf16 B=32 L=16384 H=32 Dh=64 N=128 seg=32",
    "c4d": "ssd_scan bf16 B=32 L=16384 H=32 Dh=64 N=128 seg=32, dense A_neg [H, N]",
    "c5": "gla_scan bf16 B=32 L=16384 H=32 Dh=64 seg=32",
    "c2g": "rglru_scan_gated bf16 B=8 L=4096 D=2560 seg=32 (gating in the kernels, c=8)",
    "c3a": "rotlru_scan_angle bf16 B=16 L=8192 D=2048 seg=32 (cos, sin formed in the kernels)",
    "c6": "gated_deltanet_scan bf16 B=32 L=2048 H=32 Dh=64 seg=64",
}

GATE_C = 8.0  # the RG-LRU gate exponent scale of c2 / c2g


# The independent units of each kind: batch rows times this axis of the
# config, split across ranks in multiples of the quantum (the scans' lane rule).
UNIT_AXIS = {"ssd": ("H", 1), "gla": ("H", 1), "gdn": ("H", 1), "rglru": ("D", 32), "rglru_gated": ("D", 32),
             "rotlru": ("Dp", 16), "rotlru_angle": ("Dp", 16)}


def tokens(cfg):
    return cfg["B"] * cfg["L"]


def rank_block(name, rank, world, batch=None):
    """(b0, b1, u0, u1): the rank's batch rows and heads / channels / pairs."""
    cfg = CONFIGS[name]
    ax, q = UNIT_AXIS[cfg["kind"]]
    return block_of(batch or cfg["B"], cfg[ax], rank, world, q)


def local_config(name, block=None, batch=None):
    """The config restricted to a block (or with its batch overridden)."""
    cfg = dict(CONFIGS[name])
    if batch is not None:
        cfg["B"] = batch
    if block is not None:
        b0, b1, u0, u1 = block
        ax, _ = UNIT_AXIS[cfg["kind"]]
        cfg["B"], cfg[ax] = b1 - b0, u1 - u0
    return cfg


def make_inputs(name, device, seed=0, batch=None, block=None):
    """Primal inputs of config ``name`` (tuple, in kernel order) on ``device``.

    ``batch`` overrides B; ``block`` = (b0, b1, u0, u1) restricts the inputs to
    a rank's batch rows and heads / channels / pairs (the shared parameters are
    the slice [u0, u1) of their full draw). Values are drawn in float32 from a
    generator on ``device`` and then cast to the config dtype.
    """
    full = dict(CONFIGS[name])
    cfg = local_config(name, block, batch)
    ax, _ = UNIT_AXIS[cfg["kind"]]
    u0, u1 = (0, full[ax]) if block is None else block[2:]
    g = torch.Generator(device=device).manual_seed(seed)
    f32 = dict(dtype=torch.float32, device=device, generator=g)
    # parameters every rank shares (SSD's A, RG-LRU's Lambda) come from a fixed seed
    rep = dict(dtype=torch.float32, device=device, generator=torch.Generator(device=device).manual_seed(4242))
    dt = cfg["dtype"]
    B, L = cfg["B"], cfg["L"]
    if cfg["kind"] == "ssd":
        H, Dh, N = cfg["H"], cfg["Dh"], cfg["N"]
        u = torch.randn((B, L, H, Dh), **f32)
        delta = torch.randn((B, L, H), **f32).abs_().mul_(0.1).add_(0.01)
        Bm = torch.randn((B, L, H, N), **f32)
        Cm = torch.randn((B, L, H, N), **f32)
        if cfg.get("dense_a"):  # one rate per (head, state column)
            A_neg = -torch.exp(torch.randn((full["H"], N), **rep) * 0.5)[u0:u1].contiguous()
        else:
            A = -torch.exp(torch.randn((full["H"],), **rep) * 0.5)[u0:u1]
            A_neg = A[:, None].expand(H, N)  # one rate per head, broadcast over N
        return (u.to(dt), delta.to(dt), Bm.to(dt), Cm.to(dt), A_neg)
    if cfg["kind"] == "gla":
        H, Dh = cfg["H"], cfg["Dh"]
        s = 1.0 / math.sqrt(Dh)
        q = torch.randn((B, L, H, Dh), **f32) * s
        k = torch.randn((B, L, H, Dh), **f32) * s
        v = torch.randn((B, L, H, Dh), **f32) * s
        g_ = torch.sigmoid(torch.randn((B, L, H), **f32) + 2.0)
        return tuple(t.to(dt) for t in (q, k, v, g_))
    if cfg["kind"] == "gdn":
        H, Dh = cfg["H"], cfg["Dh"]
        q = torch.nn.functional.normalize(torch.randn((B, L, H, Dh), **f32), dim=-1)
        k = torch.nn.functional.normalize(torch.randn((B, L, H, Dh), **f32), dim=-1)
        v = torch.randn((B, L, H, Dh), **f32)
        alpha = torch.exp(-torch.nn.functional.softplus(torch.randn((B, L, H), **f32) - 3.0))
        beta = torch.sigmoid(torch.randn((B, L, H), **f32))
        return tuple(t.to(dt) for t in (q, k, v, alpha, beta))
    if cfg["kind"] in ("rglru", "rglru_gated"):
        D = cfg["D"]
        x = torch.randn((B, L, D), **f32)
        r = torch.sigmoid(torch.randn((B, L, D), **f32))
        i = torch.sigmoid(torch.randn((B, L, D), **f32))
        lam = (torch.rand((full["D"],), **rep) * (6.9 - 2.2) + 2.2)[u0:u1]
        if cfg["kind"] == "rglru_gated":
            return (x.to(dt), r.to(dt), i.to(dt), lam)
        a = torch.sigmoid(lam) ** (GATE_C * r)
        b = torch.sqrt(1.0 - a * a) * (i * x)
        return (a.to(dt), b.to(dt))
    if cfg["kind"] in ("rotlru", "rotlru_angle"):
        Dp = cfg["Dp"]
        x = torch.randn((B, L, 2 * Dp), **f32)
        a = torch.sigmoid(torch.randn((B, L, Dp), **f32) + 3.0)
        th = (torch.rand((B, L, Dp), **f32) * 2.0 - 1.0) * (math.pi / 16)
        if cfg["kind"] == "rotlru_angle":
            return (a.to(dt), th.to(dt), x.to(dt))
        return (a.to(dt), torch.cos(th).to(dt), torch.sin(th).to(dt), x.to(dt))
    raise KeyError(name)


def output_shape(name, batch=None, block=None):
    cfg = local_config(name, block, batch)
    B = cfg["B"]
    if cfg["kind"] in ("ssd", "gla", "gdn"):
        return (B, cfg["L"], cfg["H"], cfg["Dh"])
    if cfg["kind"] in ("rglru", "rglru_gated"):
        return (B, cfg["L"], cfg["D"])
    return (B, cfg["L"], 2 * cfg["Dp"])


def scan_fn(pkg, name):
    kind = CONFIGS[name]["kind"]
    seg = CONFIGS[name]["seg"]
    if kind == "rglru_gated":
        return lambda *xs: pkg.rglru_scan_gated(*xs, GATE_C, seg=seg)
    if kind == "rotlru_angle":
        return lambda *xs: pkg.rotlru_scan_angle(*xs, seg=seg)
    if kind == "gdn":
        return lambda *xs: pkg.gated_deltanet_scan(*xs, seg=seg)
    f = getattr(pkg, f"{kind}_scan")
    return lambda *xs: f(*xs, seg=seg)


def gated_to_plain(x, r, i, lam):
    """numpy (x, r, i, lam) of c2g -> the (a, b) the plain RG-LRU scan takes
    (the host-side prologue of rglru.py:8-27), for the CPU baselines."""
    import numpy as np
    ls = -np.logaddexp(0.0, -lam)
    a = np.exp(GATE_C * r * ls)
    b = np.sqrt(np.maximum(1.0 - a * a, 0.0)) * i * x
    return a.astype(np.float32), b.astype(np.float32)


def angle_to_plain(a, theta, x):
    """numpy (a, theta, x) of c3a -> the (a, cs, sn, x) the plain rotLRU scan
    takes (the host-side cos/sin of rotlru.py:18-22), for the CPU baselines."""
    import numpy as np
    return a, np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32), x
