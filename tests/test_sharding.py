"""Sharding of the MatMul node across ranks, on CPU: the partition rules,
their agreement with the C ABI, and a two-rank gloo run in which each rank
computes its column block with the oracle, the blocks are all-gathered, and
the assembled result equals the unsharded one bit for bit."""
import os
import socket

import numpy as np
import pytest

from momiru_b200 import shard_columns
from momiru_b200.sharding import GatherLayout, batch_shards, column_shards


@pytest.mark.parametrize("n,world", [(8192, 1), (8192, 2), (8192, 8), (11008, 8), (11008, 3), (100, 4), (0, 2),
                                     (257, 2)])
def test_column_shards_cover_once_and_match_abi(n, world):
    sh = column_shards(n, world)
    assert sh[0][0] == 0 and sh[-1][1] == n
    for (a0, a1), (b0, b1) in zip(sh, sh[1:]):
        assert a1 == b0 and a0 <= a1
    for c0, _ in sh:
        assert c0 % 256 == 0 or c0 == n
    for r in range(world):
        assert shard_columns(n, world, r, 256) == sh[r]
    widths = [c1 - c0 for c0, c1 in sh]
    assert max(widths) - min(widths) <= 256


def test_c4_shards_are_whole_tiles():
    # 11008 = 43 tiles of 256 over 8 ranks: 6 x 6 tiles, 2 x 5 tiles
    sh = column_shards(11008, 8)
    assert [c1 - c0 for c0, c1 in sh] == [1536, 1536, 1536, 1280, 1280, 1280, 1280, 1280]


def test_batch_shards():
    assert batch_shards(512, 8) == [(64 * r, 64 * (r + 1)) for r in range(8)]
    assert batch_shards(5, 2) == [(0, 3), (3, 5)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, m, k, n, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ok = False
    try:
        from momiru_b200 import rng
        from oracle import oracle as O
        a = rng.randu((m, k), 1)
        b = rng.randu((k, n), 2)
        bias = rng.randn((n,), 3, 0.1)
        lay = GatherLayout.make(m, n, world)
        c0, c1 = lay.shards[rank]
        block = np.zeros((m, lay.width), np.float32)
        if c1 > c0:
            block[:, :c1 - c0] = O.matmul(a, b[:, c0:c1], bias=bias[c0:c1], epilogue=O.EPI_BIAS_RELU, nthreads=2)
        gathered = torch.empty((world * m, lay.width), dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, torch.from_numpy(block))
        full = lay.assemble(gathered.view(world, m, lay.width).numpy())
        ref = O.matmul(a, b, bias=bias, epilogue=O.EPI_BIAS_RELU, nthreads=2)
        ok = bool(np.array_equal(full.view(np.uint32), ref.view(np.uint32)))
    finally:
        q.put((rank, ok))
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [768, 700])
def test_two_rank_gloo_column_shard_allgather(n):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, 64, 96, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(results) == [(0, True), (1, True)]
