"""Multi-rank host logic on CPU with the gloo backend (world size 2): batch
sharding covers every row exactly once, each rank computes its shard with no
exchange, gathering the shards reproduces the single-process result, and the
timing reduction takes the maximum over ranks."""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ORACLE, ROOT, import_pkg


def test_shards_cover_every_row_once():
    import importlib
    import_pkg()
    S = importlib.import_module("mlx-recurrence_b200.sharding")
    for B in (1, 3, 8, 32, 33):
        for world in (1, 2, 3, 4, 8):
            rows = []
            for r in range(world):
                b0, b1 = S.shard_batch(B, r, world)
                assert b1 - b0 in (B // world, B // world + 1)
                rows += list(range(b0, b1))
            assert rows == list(range(B))
    with pytest.raises(ValueError):
        S.shard_batch(4, 2, 2)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_blocks_cover_every_unit_once_for_every_config(world):
    """Every configuration splits over 1-8 ranks into nonempty rectangular
    blocks of (batch row, head / channel / pair) units that cover each unit
    exactly once and keep the scans' lane rule on the channel axis."""
    import importlib
    import_pkg()
    W = importlib.import_module("mlx-recurrence_b200.workloads")
    for name, cfg in W.CONFIGS.items():
        ax, q = W.UNIT_AXIS[cfg["kind"]]
        B, U = cfg["B"], cfg[ax]
        seen = np.zeros((B, U), dtype=int)
        sizes = []
        for r in range(world):
            b0, b1, u0, u1 = W.rank_block(name, r, world)
            assert b1 > b0 and u1 > u0, (name, world, r)
            assert u0 % q == 0 and u1 % q == 0
            seen[b0:b1, u0:u1] += 1
            sizes.append((b1 - b0) * (u1 - u0))
        assert np.all(seen == 1), (name, world)
        if B % world == 0:  # whole batch ranges, balanced
            assert all(W.rank_block(name, r, world)[2:] == (0, U) for r in range(world))
            assert len(set(sizes)) == 1
    # c0 / c1 (B = 3) at 4 and 8 ranks: split by heads, every rank busy
    assert [W.rank_block("c0", r, 4) for r in range(4)] == [(0, 3, 0, 3), (0, 3, 3, 6), (0, 3, 6, 9), (0, 3, 9, 12)]
    with pytest.raises(ValueError):
        import importlib as il
        il.import_module("mlx-recurrence_b200.sharding").block_of(2, 3, 0, 8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    sys.path[:0] = [ROOT, ORACLE]
    import importlib
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        S = importlib.import_module("mlx-recurrence_b200.sharding")
        import c_oracle
        B, L, D = 5, 64, 64
        g = torch.Generator().manual_seed(0)  # the global problem, sliced per rank
        a = torch.rand(B, L, D, generator=g) * 1.8 - 0.9
        x = torch.randn(B, L, D, generator=g)
        gy = torch.randn(B, L, D, generator=g)
        b0, b1 = S.shard_batch(B, rank, world)
        out = c_oracle.run("rglru", [a[b0:b1].numpy(), x[b0:b1].numpy()], 16, gy=gy[b0:b1].numpy())
        y = S.gather_rows(torch.from_numpy(out["y"]), B)
        ga = S.gather_rows(torch.from_numpy(out["grads"][0]), B)
        t = S.max_over_ranks([float(rank + 1), 10.0 - rank])
        if rank == 0:
            ref = c_oracle.run("rglru", [a.numpy(), x.numpy()], 16, gy=gy.numpy())
            np.save(os.path.join(out_dir, "y.npy"), y.numpy())
            np.save(os.path.join(out_dir, "ref.npy"), ref["y"])
            np.save(os.path.join(out_dir, "ga.npy"), ga.numpy())
            np.save(os.path.join(out_dir, "ga_ref.npy"), ref["grads"][0])
            np.save(os.path.join(out_dir, "t.npy"), np.array(t))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_compute_and_gather(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    assert np.array_equal(np.load(tmp_path / "y.npy"), np.load(tmp_path / "ref.npy"))
    assert np.array_equal(np.load(tmp_path / "ga.npy"), np.load(tmp_path / "ga_ref.npy"))
    assert list(np.load(tmp_path / "t.npy")) == [2.0, 10.0]


def _blocks_main(rank, world, port, out_dir):
    sys.path[:0] = [ROOT, ORACLE]
    import importlib
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        S = importlib.import_module("mlx-recurrence_b200.sharding")
        import ref_loops as R
        # SSD units (batch row, head): B = 3 rows over 2 or 3 ranks with heads split too
        B, L, H, Dh, N = 3, 24, 4, 4, 3
        g = torch.Generator().manual_seed(1)
        u = torch.randn(B, L, H, Dh, generator=g, dtype=torch.float64)
        d = torch.rand(B, L, H, generator=g, dtype=torch.float64) * 0.2 + 0.01
        Bm = torch.randn(B, L, H, N, generator=g, dtype=torch.float64)
        Cm = torch.randn(B, L, H, N, generator=g, dtype=torch.float64)
        A = -torch.rand(H, N, generator=g, dtype=torch.float64) - 0.1
        gy = torch.randn(B, L, H, Dh, generator=g, dtype=torch.float64)
        b0, b1, h0, h1 = S.block_of(B, H, rank, world)
        sl = lambda t: t[b0:b1, :, h0:h1]
        y, _ = R.ssd_forward(sl(u).numpy(), sl(d).numpy(), sl(Bm).numpy(), sl(Cm).numpy(), A[h0:h1].numpy())
        gr = R.ssd_backward(sl(u).numpy(), sl(d).numpy(), sl(Bm).numpy(), sl(Cm).numpy(), A[h0:h1].numpy(),
                            sl(gy).numpy())
        y_all = S.gather_blocks(torch.from_numpy(y), B, H)
        gu_all = S.gather_blocks(torch.from_numpy(gr[0]), B, H)
        gd_all = S.gather_blocks(torch.from_numpy(gr[1]), B, H)
        gA_all = S.sum_unit_param(torch.from_numpy(gr[4]), B, H)
        if rank == 0:
            yo, _ = R.ssd_forward(u.numpy(), d.numpy(), Bm.numpy(), Cm.numpy(), A.numpy())
            ro = R.ssd_backward(u.numpy(), d.numpy(), Bm.numpy(), Cm.numpy(), A.numpy(), gy.numpy())
            np.save(os.path.join(out_dir, "errs.npy"), np.array([
                np.max(np.abs(y_all.numpy() - yo)), np.max(np.abs(gu_all.numpy() - ro[0])),
                np.max(np.abs(gd_all.numpy() - ro[1])), np.max(np.abs(gA_all.numpy() - ro[4]))]))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_on_batch_head_blocks(tmp_path, world):
    """B = 3 does not split evenly: the ranks take (batch row x head) blocks,
    compute them with no exchange, and the gathered outputs and gradients (the
    shared A's as a sum over ranks) equal the single-process result."""
    mp.start_processes(_blocks_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    errs = np.load(tmp_path / "errs.npy")
    assert np.all(errs[:3] == 0.0), errs
    assert errs[3] < 1e-12, errs
