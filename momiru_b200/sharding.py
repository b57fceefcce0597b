"""Column-block and batch sharding of the MatMul node across ranks.

The reference IR names the collectives a sharded node would need
(CollectiveSpec, src/momiru/tensor_light/execution/ir.rs:1140-1154) but
rejects AllGather today (ir.rs:1773-1779); this module is the host-side plan
for the two partitions the GPU path uses:

  * columns: rank r owns output columns [c0, c1) in whole 256-column tile
    units (mmr_shard_columns); it binds the ordinary GEMM on the zero-copy
    views B[:, c0:c1], bias[c0:c1], C[:, c0:c1]; replicating C then needs an
    all-gather of the column blocks.
  * batch: rank r owns batch entries [b0, b1); no collective.

The arithmetic here is plain Python so it runs (and is tested) on CPU ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

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


@dataclass(frozen=True)
class GatherLayout:
    """Where each rank's column block lands in the gathered buffer.

    All-gather moves equal-sized blocks, so each rank's block is padded to
    the widest shard: gathered[r] is an [m, width] block whose first
    (c1 - c0) columns are rank r's output columns c0..c1-1."""
    m: int
    n: int
    width: int
    shards: tuple

    @staticmethod
    def make(m: int, n: int, world: int, align: int = TILE_N) -> "GatherLayout":
        shards = tuple(column_shards(n, world, align))
        width = max(c1 - c0 for c0, c1 in shards) if shards else 0
        return GatherLayout(m, n, max(width, 1), shards)

    def assemble(self, gathered):
        """gathered: array-like [world, m, width] (numpy or torch) -> [m, n]."""
        import numpy as np
        is_np = isinstance(gathered, np.ndarray)
        if is_np:
            out = np.empty((self.m, self.n), dtype=gathered.dtype)
        else:
            import torch
            out = torch.empty((self.m, self.n), dtype=gathered.dtype, device=gathered.device)
        for r, (c0, c1) in enumerate(self.shards):
            out[:, c0:c1] = gathered[r][:, :c1 - c0]
        return out
