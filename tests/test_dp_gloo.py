"""Data-parallel host logic with two gloo ranks on the CPU: the sequence shards cover
every sequence once, the timed region reports the slowest rank, and rank 0 gathers the
generated tokens in sequence order.  The per-rank 'generation' is a deterministic stand-in
(no GPU); the device path it stands for is covered by the GPU tests."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import load_package


def test_shard_partitions_every_count():
    dp = load_package().dp
    for n in [0, 1, 7, 64, 65]:
        for world in [1, 2, 3, 8]:
            got = [i for r in range(world) for i in dp.shard(n, r, world)]
            assert got == list(range(n))
            sizes = [len(dp.shard(n, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        dp.shard(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_seq, n_gen, out_q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    pkg = load_package()
    dp = pkg.dp.DataParallel.from_env(timeout_s=60, backend="gloo")
    mine = pkg.dp.shard(n_seq, dp.rank, dp.world)
    # stand-in for ctx.generate on this rank's sequences: token = seq * 1000 + position
    rows = np.array([[s * 1000 + j for j in range(n_gen)] for s in mine], np.int32).reshape(len(mine), n_gen)
    dp.barrier()
    slowest = dp.max_over_ranks(10.0 + rank)
    total = dp.sum_over_ranks(len(mine))
    gathered = dp.gather_rows(rows, n_seq)
    # rank 0's bytes (the tensor-parallel NCCL id under bench.py --tp) reach every rank
    shared = dp.broadcast_bytes(bytes(range(128)) if rank == 0 else b"")
    out_q.put((rank, slowest, total, None if gathered is None else gathered.tolist(), shared))
    dp.close()


@pytest.mark.parametrize("n_seq", [5, 64])
def test_two_rank_gloo_sharding(n_seq):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world, n_gen = _free_port(), 2, 4
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n_seq, n_gen, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, slowest, total, gathered, shared = q.get(timeout=120)
        res[rank] = (slowest, total, gathered)
        assert shared == bytes(range(128))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][0] == 10.0 + world - 1  # max over ranks
        assert res[r][1] == n_seq             # every sequence generated once
    assert res[1][2] is None
    expect = [[s * 1000 + j for j in range(n_gen)] for s in range(n_seq)]
    assert res[0][2] == expect
