"""Sharding of the MatMul node across ranks, on CPU: the partition rules,
their agreement with the C ABI, and two-rank gloo runs of the shipped
replicated-output protocol. Each rank narrows the whole node with the
library's own host-only narrowing (mmr_shard_local_desc, the code
mmr_sharded_gemm_bind runs), validates its narrowed node, exchanges its
replica handles through the bind-time exchange the GPU path uses, computes
its column block with the oracle by reading exactly the views the narrowed
descriptor names, and stores the block into every rank's replica at the
offset the library gives (the stores the GEMM epilogue makes over NVLink,
here carried by gloo). Every replica must equal the unsharded oracle result
bit for bit."""
import os
import socket

import numpy as np
import pytest

from momiru_b200 import shard_columns
from momiru_b200.sharding import batch_shards, column_shards


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


def _host_view(arr, base_elems=0, dims=None, strides=None):
    """An mmr_view over a host numpy buffer (validation never touches a GPU)."""
    from momiru_b200 import _abi
    v = _abi.MmrView()
    v.address = arr.ctypes.data
    v.bytes = arr.nbytes
    v.base_offset_bytes = 4 * base_elems
    dims = arr.shape if dims is None else dims
    strides = tuple(st // 4 for st in arr.strides) if strides is None else strides
    v.rank = len(dims)
    v.device_ordinal = 0
    for i, (d, st) in enumerate(zip(dims, strides)):
        v.dims[i] = d
        v.strides[i] = st
    v.allocation_id = arr.ctypes.data
    return v


def _read_view(v, buf):
    """The numpy view an mmr_view names inside `buf` (same address)."""
    assert v.address == buf.ctypes.data and v.base_offset_bytes % 4 == 0
    flat = buf.reshape(-1)
    dims = tuple(v.dims[i] for i in range(v.rank))
    strides = tuple(4 * v.strides[i] for i in range(v.rank))
    return np.lib.stride_tricks.as_strided(flat[v.base_offset_bytes // 4:], shape=dims, strides=strides)


def _protocol_rank(rank, world, port, m, k, n, transpose_rhs, q):
    import ctypes

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ok, why = False, ""
    try:
        from momiru_b200 import _abi, rng
        from momiru_b200.execution import _check
        from momiru_b200.sharding import exchange_replica_handles, local_shard
        from oracle import oracle as O
        lib = _abi.load()
        a = rng.randu((m, k), 1)
        b = rng.randu((k, n), 2)
        rhs = np.ascontiguousarray(b.T) if transpose_rhs else b   # [n, k] buffer read transposed
        bias = rng.randn((n,), 3, 0.1)
        pitch = (n + 3) // 4 * 4 + 4                               # padded output rows
        replica = np.full((m, pitch), np.nan, np.float32)          # this rank's whole output replica
        d = _abi.MmrMatmulDesc()
        d.lhs, d.rhs, d.bias = _host_view(a), _host_view(rhs), _host_view(bias)
        d.out = _host_view(replica, 0, (m, n), (pitch, 1))
        d.transpose_rhs = int(transpose_rhs)
        d.math_mode = _abi.MATH_STRICT_FP32
        d.epilogue = _abi.EPI_BIAS_RELU
        local, c0, c1, off = local_shard(d, rank, world)
        assert (c0, c1) == column_shards(n, world)[rank], (c0, c1)
        assert off == 4 * c0, off
        info = _abi.MmrGemmInfo()
        _check(lib.mmr_gemm_validate(ctypes.byref(local), ctypes.byref(info)))
        assert (info.m, info.n, info.k) == (m, c1 - c0, k), (info.m, info.n, info.k)
        # Bind-time exchange of (replica, signal) handles, in the shape the GPU
        # path sends: rank-specific stand-ins for the 64-byte IPC handles.
        mine = ((bytes([rank]) * 64, 0), (bytes([rank + 100]) * 64, 8 * rank))
        everyone = exchange_replica_handles(mine)
        assert everyone == [((bytes([r]) * 64, 0), (bytes([r + 100]) * 64, 8 * r)) for r in range(world)]
        # This rank's block, read through the narrowed descriptor's views.
        block = np.zeros((m, 0), np.float32)
        if c1 > c0:
            bv = _read_view(local.rhs, rhs)
            block = O.matmul(a, bv.T if transpose_rhs else bv, bias=_read_view(local.bias, bias),
                             epilogue=O.EPI_BIAS_RELU, nthreads=2)
        # Peer stores: every rank writes every block at its offset in its replica.
        stores = [None] * world
        dist.all_gather_object(stores, (off, block))
        for o, blk in stores:
            if blk.shape[1]:
                dst = replica.reshape(-1)[o // 4:]
                np.lib.stride_tricks.as_strided(dst, shape=blk.shape, strides=(4 * pitch, 4))[...] = blk
        ref = O.matmul(a, b, bias=bias, epilogue=O.EPI_BIAS_RELU, nthreads=2)
        ok = bool(np.array_equal(replica[:, :n].view(np.uint32), ref.view(np.uint32)))
        ok = ok and bool(np.all(np.isnan(replica[:, n:])))  # the pad columns are never written
        why = "" if ok else "replica differs from the unsharded oracle result"
    except Exception as e:  # reported through the queue
        why = repr(e)
    finally:
        q.put((rank, ok, why))
        dist.destroy_process_group()


@pytest.mark.parametrize("n,transpose_rhs", [(768, False), (700, False), (600, True)])
def test_two_rank_gloo_replicated_column_protocol(n, transpose_rhs):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_protocol_rank, args=(r, 2, port, 64, 96, n, transpose_rhs, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [(r, ok) for r, ok, _ in results] == [(0, True), (1, True)], results


def test_local_shard_rejects_bad_ranks():
    from momiru_b200 import _abi
    from momiru_b200.execution import InvalidArgument, InvalidShape
    from momiru_b200.sharding import local_shard
    a = np.zeros((8, 8), np.float32)
    d = _abi.MmrMatmulDesc()
    d.lhs, d.rhs, d.out = _host_view(a), _host_view(a), _host_view(np.zeros((8, 8), np.float32))
    with pytest.raises(InvalidArgument):
        local_shard(d, 2, 2)
    with pytest.raises(InvalidArgument):
        local_shard(d, 0, 9)
    v = np.zeros(8, np.float32)
    d.rhs = _host_view(v)
    d.out = _host_view(np.zeros(8, np.float32))
    with pytest.raises(InvalidShape):
        local_shard(d, 0, 2)  # a vector rhs has no columns to shard


def test_column_block_views_match_the_library_narrowing():
    """The C4 projection shape (A = X^T view, B = a column slice of a wider
    buffer) split over 8 ranks with the output kept sharded: every rank's
    views are the library's narrowing (mmr_shard_local_desc), and the blocks
    tile the 11008 output columns in 256-column units. Host only."""
    from momiru_b200 import DeviceBuffer, DeviceView, MatMulNode
    from momiru_b200.sharding import column_block_views, column_shards
    g = 1 << 32
    x = DeviceView.contiguous(DeviceBuffer(1 * g, 4 * 4096 * 4096, 0), (4096, 4096))
    w = DeviceView.contiguous(DeviceBuffer(2 * g, 4 * 4096 * 12288, 0), (4096, 12288))
    out = DeviceView.contiguous(DeviceBuffer(3 * g, 4 * 4096 * 11008, 0), (4096, 11008))
    blocks = []
    for rank in range(8):
        rb, ob, bb, c0, c1 = column_block_views(MatMulNode(), x.transpose(), w.narrow(1, 0, 11008), out,
                                                None, rank, 8)
        assert bb is None and (c0, c1) == column_shards(11008, 8)[rank]
        assert rb.dims == (4096, c1 - c0) and rb.strides == (12288, 1) and rb.offset == c0
        assert ob.dims == (4096, c1 - c0) and ob.strides == (11008, 1) and ob.offset == c0
        blocks.append((c0, c1))
    assert blocks[0][0] == 0 and blocks[-1][1] == 11008
    assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
    # transpose_rhs: the rhs buffer is [n, k] and its rows are the columns being dealt
    wt = DeviceView.contiguous(DeviceBuffer(4 * g, 4 * 1024 * 512, 0), (1024, 512))
    o2 = DeviceView.contiguous(DeviceBuffer(5 * g, 4 * 300 * 1024, 0), (300, 1024))
    a2 = DeviceView.contiguous(DeviceBuffer(6 * g, 4 * 300 * 512, 0), (300, 512))
    rb, ob, _, c0, c1 = column_block_views(MatMulNode(transpose_rhs=True), a2, wt, o2, None, 1, 2)
    assert (c0, c1) == (512, 1024) and rb.dims == (512, 512) and rb.offset == 512 * 512
