"""Multi-GPU host logic on CPU: two gloo ranks shard a batch, run a per-sample
stand-in for the forward, gather the outputs to rank 0 and take the slowest
rank's time, exactly as bench.py does over NCCL."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from nnc_cuda import shard as S


def test_shard_ranges_cover_the_batch_in_order():
    for world in (1, 2, 4, 8):
        got = [S.shard_range(1024, world, r) for r in range(world)]
        assert got[0][0] == 0 and all(c == 1024 // world for _, c in got)
        assert all(got[i][0] + got[i][1] == got[i + 1][0] for i in range(world - 1))


@pytest.mark.parametrize("args", [(1000, 3, 0), (8, 2, 2), (8, 0, 0)])
def test_shard_range_rejects_uneven_or_out_of_range(args):
    with pytest.raises(ValueError):
        S.shard_range(*args)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _forward(x):
    # Per-sample stand-in for the model: depends on each sample only.
    return x.reshape(x.shape[0], -1).sum(1, keepdim=True) * 2.0 + x[:, :1, 0, 0]


def _rank_main(rank, world, port, out_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = torch.from_numpy(np.random.default_rng(1).standard_normal((8, 3, 4, 4)).astype(np.float32))
        first, count = S.shard_range(full.shape[0], world, rank)
        local = _forward(full[first:first + count])
        gathered = S.gather_to_rank0(local, world, dist)
        slowest = S.max_over_ranks(float(rank + 1) * 1.5, world, dist)
        if rank == 0:
            np.savez(out_path, gathered=gathered.numpy(), want=_forward(full).numpy(), slowest=slowest)
        else:
            assert gathered is None
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_in_batch_order(tmp_path):
    import torch.multiprocessing as mp

    out = tmp_path / "r0.npz"
    mp.start_processes(_rank_main, args=(2, _free_port(), str(out)), nprocs=2, start_method="spawn", join=True)
    r = np.load(out)
    np.testing.assert_array_equal(r["gathered"], r["want"])
    assert float(r["slowest"]) == 3.0
