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
