"""Multi-GPU partitioning of the tiled GEMM / batched conv (one process per GPU).

The reference shards a matmul across Tensix cores by output rows
(tests/test_matmul_2core.cpp:43-63: core c owns A rows and C rows
[c*Mt_pc, (c+1)*Mt_pc)), every core reading the whole B.  Across B200s the
same split is done in tile rows: a tile row of a tile-layout matrix is one
contiguous run of Nt*2 KiB, so each rank's C shard is a contiguous slice and
concatenating the shards in rank order (an all-gather) rebuilds the global
tile-layout C exactly.  Convolutions shard the batch: NHWC images are
contiguous, so no halo is exchanged.
"""


def split_rows(total, world, rank):
    """Contiguous [begin, end) share of `total` units (tile rows or images) for
    `rank`; the first `total % world` ranks take one extra unit."""
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_bytes(Mt_shard, Nt):
    """Bytes of a C shard of Mt_shard tile rows."""
    return Mt_shard * Nt * 2048


def gather_tiles(shards):
    """Host-side reassembly: concatenating per-rank tile-row shards in rank
    order gives the global tile-layout matrix (what ncclAllGather produces
    on the device)."""
    import numpy as np
    return np.concatenate([s.reshape(-1) for s in shards])
