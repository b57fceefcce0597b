"""Column-block and batch sharding of the MatMul node across ranks.

The reference IR names the collectives a sharded node would need
(CollectiveSpec, src/momiru/tensor_light/execution/ir.rs:1140-1154) but
rejects AllGather today (ir.rs:1773-1779). The GPU path uses two partitions:

  * columns: rank r owns output columns [c0, c1) in whole 256-column tile
    units (mmr_shard_columns) and binds the ordinary GEMM on the zero-copy
    views B[:, c0:c1], bias[c0:c1], C[:, c0:c1] (mmr_shard_local_desc). When
    the output is replicated, the GEMM's own epilogue stores every finished
    tile into each rank's replica over NVLink (mmr_sharded_gemm_bind): the
    all-gather is fused into the GEMM and no collective runs on the data path.
    The only host exchange is the one-time swap of IPC handles at bind.
  * batch: rank r owns batch entries [b0, b1); no collective.

The partition arithmetic is plain Python so it runs (and is tested) on CPU
ranks; `local_shard` calls the library's host-only narrowing, the same code
mmr_sharded_gemm_bind runs.
"""
from __future__ import annotations

TILE_N = 256


def column_shards(n: int, world: int, align: int = TILE_N) -> list[tuple[int, int]]:
    """[c0, c1) per rank: whole `align` units dealt as evenly as possible, the
    first (units % world) ranks taking one extra (same rule as the C ABI's
    mmr_shard_columns)."""
    if world < 1 or n < 0 or align < 1:
        raise ValueError("bad shard request")
    units = (n + align - 1) // align
    base, extra = divmod(units, world)
    out = []
    for r in range(world):
        u0 = r * base + min(r, extra)
        u1 = u0 + base + (1 if r < extra else 0)
        out.append((min(n, u0 * align), min(n, u1 * align)))
    return out


def batch_shards(batch: int, world: int) -> list[tuple[int, int]]:
    base, extra = divmod(batch, world)
    out = []
    for r in range(world):
        b0 = r * base + min(r, extra)
        out.append((b0, b0 + base + (1 if r < extra else 0)))
    return out


def local_shard(desc, rank: int, world: int):
    """The node rank `rank` binds in a column-sharded run: `desc` (a whole
    mmr_matmul_desc) narrowed to the rank's column block. Returns
    (local_desc, c0, c1, out_offset_bytes), out_offset_bytes being where the
    block starts in every output replica. Host only (mmr_shard_local_desc)."""
    import ctypes

    from . import _abi, execution
    lib = _abi.load()
    local = _abi.MmrMatmulDesc()
    c0, c1, off = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_uint64()
    execution._check(lib.mmr_shard_local_desc(ctypes.byref(desc), rank, world, ctypes.byref(local),
                                              ctypes.byref(c0), ctypes.byref(c1), ctypes.byref(off)))
    return local, c0.value, c1.value, off.value


def column_block_views(node, lhs, rhs, out, bias=None, rank: int = 0, world: int = 1):
    """Rank `rank`'s share of a column-sharded node whose output stays
    sharded: each rank computes and keeps out[..., c0:c1], so no collective
    runs (the C4 projection shape across GPUs). Returns (rhs_block,
    out_block, bias_block, c0, c1): zero-copy views narrowed to the rank's
    column block, exactly the ones the library's host-only narrowing
    (mmr_shard_local_desc) produces, which is checked here."""
    from . import _abi, execution
    local, c0, c1, _ = local_shard(execution._desc(node, lhs, rhs, out, bias, None), rank, world)
    n = c1 - c0
    rb = rhs.narrow(-2 if node.transpose_rhs else -1, c0, n)
    ob = out.narrow(-1, c0, n)
    bb = bias.narrow(-1, c0, n) if bias is not None else None
    for mine, theirs in ((rb, local.rhs), (ob, local.out)):
        v = mine.to_abi()
        same = (v.address + v.base_offset_bytes == theirs.address + theirs.base_offset_bytes
                and list(v.dims[:v.rank]) == list(theirs.dims[:theirs.rank])
                and list(v.strides[:v.rank]) == list(theirs.strides[:theirs.rank]))
        if not same:
            raise execution.InvalidArgument("column block disagrees with mmr_shard_local_desc",
                                            _abi.ERR_INVALID_ARGUMENT)
    return rb, ob, bb, c0, c1


def exchange_replica_handles(mine, group=None) -> list:
    """Bind-time exchange: every rank contributes the IPC handles of its output
    replica and its completion-signal array, as ((handle bytes, offset),
    (handle bytes, offset)); every rank receives all ranks' pairs in rank order.
    The only collective of the replicated GEMM, run once at bind."""
    import torch.distributed as dist
    everyone = [None] * dist.get_world_size(group)
    dist.all_gather_object(everyone, mine, group=group)
    return everyone


class ReplicatedColumnGemm:
    """Column-sharded GEMM whose output is replicated on every rank.

    One process per GPU, `torch.distributed` initialised (any backend: it only
    carries the 72-byte IPC handles at bind time). Each rank passes the full
    lhs, rhs, bias views and a full output replica of its own; the node is
    bound with mmr_sharded_gemm_bind, whose GEMM epilogue stores every finished
    output tile into all replicas over NVLink, followed by a bounded
    completion handshake. No collective runs on the data path.
    """

    def __init__(self, node, lhs, rhs, out, bias=None, stream=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _abi, execution
        self._lib = _abi.load()
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        if self.world > 8:
            raise execution.InvalidArgument("at most 8 ranks", _abi.ERR_INVALID_ARGUMENT)
        dev = out.buffer.device_ordinal
        self._views = (lhs, rhs, out, bias)
        self._signal = torch.zeros(8, dtype=torch.int64, device=f"cuda:{dev}")
        torch.cuda.synchronize(dev)

        def export(addr):
            h = _abi.MmrIpcHandle()
            execution._check(self._lib.mmr_ipc_export(addr, ctypes.byref(h)))
            return bytes(h.bytes), int(h.offset)

        mine = (export(out.buffer.address), export(self._signal.data_ptr()))
        everyone = exchange_replica_handles(mine)
        self._imported = []
        d = _abi.MmrShardedDesc()
        d.local = execution._desc(node, lhs, rhs, out, bias, stream)
        d.rank = self.rank
        d.nranks = self.world
        d.signal = self._signal.data_ptr()
        for r, ((ob, oo), (sb, so)) in enumerate(everyone):
            if r == self.rank:
                d.peer_out[r] = out.buffer.address
                d.peer_signal[r] = self._signal.data_ptr()
                continue
            for i, (b, off) in enumerate(((ob, oo), (sb, so))):
                h = _abi.MmrIpcHandle()
                ctypes.memmove(h.bytes, b, 64)
                h.offset = off
                addr = ctypes.c_uint64()
                execution._check(self._lib.mmr_ipc_import(ctypes.byref(h), dev, ctypes.byref(addr)))
                self._imported.append((addr.value, h))
                if i == 0:
                    d.peer_out[r] = addr.value
                else:
                    d.peer_signal[r] = addr.value
        self._handle = ctypes.c_void_p()
        execution._check(self._lib.mmr_sharded_gemm_bind(ctypes.byref(d), ctypes.byref(self._handle)))
        info = _abi.MmrGemmInfo()
        execution._check(self._lib.mmr_gemm_query(self._handle, ctypes.byref(info)))
        self.info = info.as_dict()
        self.columns = column_shards(out.dims[-1], self.world)[self.rank]

    def replay(self):
        from . import execution
        execution._check(self._lib.mmr_gemm_run(self._handle))

    def quiesce_or_abort(self, timeout_s: float = 60.0):
        from . import execution
        execution._check(self._lib.mmr_gemm_quiesce(self._handle, int(timeout_s * 1e9)))

    def close(self):
        import ctypes
        if self._handle:
            self._lib.mmr_gemm_destroy(self._handle)
            self._handle = ctypes.c_void_p()
        for addr, h in self._imported:
            self._lib.mmr_ipc_release(addr, ctypes.byref(h))
        self._imported = []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
