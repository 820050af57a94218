"""Multi-rank host logic on CPU (gloo, world size 2 and 3): the M-shard of the
tiled GEMM and the batch shard of the NHWC conv, reassembled with an
all-gather, equal the unsharded result; the row shard of a 'same'
convolution with its halo exchange (shard.conv2d_nhwc_h_sharded, the oracle
as the local convolution) gives every rank exactly its rows of the unsharded
output.  The GPU path (bench.py under torchrun) uses the same split_rows /
contiguous-shard layout with NCCL.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def worker(rank, world, port, q):
    import sys
    import torch
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "tt-foil_b200")]
    from oracle import oracle
    from ttfoil import shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # GEMM: 7 tile rows over `world` ranks (uneven split), Kt = 3, Nt = 2.
        Mt, Kt, Nt = 7, 3, 2
        a = oracle.rand_bf16((Mt * 32, Kt * 32), 1)
        b = oracle.rand_bf16((Kt * 32, Nt * 32), 2)
        r0, r1 = shard.split_rows(Mt, world, rank)
        a_tiles = oracle.tilize(a)
        mine = a_tiles[r0 * Kt * 1024:r1 * Kt * 1024]
        c_part = oracle.matmul_tiles(mine, oracle.tilize(b), r1 - r0, Kt, Nt) if r1 > r0 else \
            np.zeros(0, np.uint16)
        # all-gather of uneven shards: pad to the largest share
        # gloo has no 16-bit integer collectives: move bf16 bits as int32 pairs
        cap = shard.shard_bytes(-(-Mt // world), Nt) // 2
        buf = np.zeros(cap, np.uint16)
        buf[:c_part.size] = c_part
        parts = [torch.zeros(cap // 2, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(buf.view(np.int32)))
        shards = []
        for r in range(world):
            s0, s1 = shard.split_rows(Mt, world, r)
            shards.append(parts[r].numpy().view(np.uint16)[:(s1 - s0) * Nt * 1024])
        c_all = shard.gather_tiles(shards)
        ok_gemm = np.array_equal(c_all, oracle.matmul_tiles(a_tiles, oracle.tilize(b), Mt, Kt, Nt))

        # conv: batch 4 split over ranks, NHWC images are contiguous.
        x = oracle.rand_bf16((4, 6, 6, 8), 3)
        w = oracle.randn_bf16((16, 3, 3, 8), 4, 0.2)
        bias = oracle.rand_bf16((16,), 5, -0.1, 0.1)
        n0, n1 = shard.split_rows(4, world, rank)
        y_part = oracle.conv_nhwc(x[n0:n1], w, bias, 2, 1, relu=True)
        per = y_part[0].size if n1 > n0 else 3 * 3 * 16
        cap = -(-4 // world) * per
        buf = np.zeros(cap, np.uint16)
        buf[:y_part.size] = y_part.reshape(-1)
        parts = [torch.zeros(cap // 2, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(buf.view(np.int32)))
        ys = []
        for r in range(world):
            s0, s1 = shard.split_rows(4, world, r)
            ys.append(parts[r].numpy().view(np.uint16)[:(s1 - s0) * per])
        y_all = np.concatenate(ys).reshape(4, 3, 3, 16)
        ok_conv = np.array_equal(y_all, oracle.conv_nhwc(x, w, bias, 2, 1, relu=True))

        # row shard with halos: 2 images of 11 rows (uneven split), 3x3 and 5x5.
        ok_rows = True
        for K, pad in ((3, 1), (5, 2)):
            H, W, Cin, Cout = 11, 7, 16, 16
            xi = oracle.rand_bf16((2, H, W, Cin), 10 + K)
            wk = oracle.randn_bf16((Cout, K, K, Cin), 11 + K, 0.1)
            bk = oracle.rand_bf16((Cout,), 12 + K, -0.1, 0.1)
            h0, h1 = shard.split_rows(H, world, rank)

            def oracle_conv(ext, w_, b_, N_, H_, W_, Cin_, Cout_, K_, pad_, relu_):
                y = oracle.conv_nhwc(ext.numpy().view(np.uint16), w_, b_, 1, pad_, relu=relu_)
                return torch.from_numpy(y.view(np.int16))

            xs = torch.from_numpy(np.ascontiguousarray(xi[:, h0:h1]).view(np.int16))
            ys = shard.conv2d_nhwc_h_sharded(xs, wk, bk, 2, h1 - h0, W, Cin, Cout, K, pad, relu=True,
                                            conv=oracle_conv)
            full = oracle.conv_nhwc(xi, wk, bk, 1, pad, relu=True)
            ok_rows &= np.array_equal(ys.numpy().view(np.uint16), full[:, h0:h1])
        q.put((rank, bool(ok_gemm), bool(ok_conv and ok_rows)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_results_reassemble(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(g and c for _, g, c in res), res


def test_split_rows_covers_range():
    from ttfoil import shard
    for total in [0, 1, 7, 64, 65]:
        for world in [1, 2, 3, 8]:
            spans = [shard.split_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1


def gathered_worker(rank, world, port, q, fail_open_on=None):
    """GatheredTiles' host logic on CPU: the peer buffers are POSIX shared
    memory segments (a handle = the segment name), the fused GEMM a stand-in
    that writes this rank's oracle rows into its own and every peer segment
    at the addresses GatheredTiles computes, the fence a gloo barrier.  With
    `fail_open_on`, that rank fails to open a peer buffer: every rank must
    then raise from the constructor (none left waiting in a collective) and
    release what it allocated."""
    import sys
    from multiprocessing import shared_memory
    import torch
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "tt-foil_b200")]
    from oracle import oracle
    import ttfoil
    from ttfoil import shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    segs = {}            # fake device address -> (segment, size)
    calls = {"close": 0, "free": 0}

    def resolve(addr):
        for base, (seg, size) in segs.items():
            if base <= addr < base + size:
                return seg, addr - base
        raise AssertionError(f"address {addr:#x} outside every buffer")

    def peer_alloc(device, nbytes):
        seg = shared_memory.SharedMemory(create=True, size=nbytes)
        base = (rank + 1) << 40
        segs[base] = (seg, nbytes)
        return base, seg.name.encode().ljust(64, b"\0")

    def peer_open(device, handle):
        if rank == fail_open_on:
            raise ttfoil.FoilError(4, "injected: cudaIpcOpenMemHandle failed")
        seg = shared_memory.SharedMemory(name=handle.rstrip(b"\0").decode())
        base = (len(segs) + 1) << 44
        segs[base] = (seg, seg.size)
        return base

    def matmul_tiles_gather(a, b, c, peer_c, Mt, Kt, Nt, bias=None, relu=False, stream=None):
        rows = oracle.matmul_tiles(a, b, Mt, Kt, Nt).view(np.uint8)
        for addr in [c] + list(peer_c):
            seg, off = resolve(addr)
            assert off % 2048 == 0 and off + rows.size <= seg.size
            seg.buf[off:off + rows.size] = rows.tobytes()

    def peer_close(device, ptr):
        calls["close"] += 1

    def peer_free(device, ptr):
        calls["free"] += 1
        seg = segs[ptr][0]
        seg.close()
        seg.unlink()

    ttfoil.peer_alloc, ttfoil.peer_open = peer_alloc, peer_open
    ttfoil.matmul_tiles_gather, ttfoil.peer_close, ttfoil.peer_free = (matmul_tiles_gather, peer_close,
                                                                      peer_free)
    torch.cuda.synchronize = lambda *a, **k: None
    ok = True
    try:
        if fail_open_on is not None:
            try:
                shard.GatheredTiles(7, 2, device=0)
                ok = False
            except RuntimeError as e:
                ok = "injected" in str(e) and calls["free"] == 1
            dist.barrier()
            q.put((rank, bool(ok)))
            return
        Mt, Kt, Nt = 7, 3, 2
        a = oracle.tilize(oracle.rand_bf16((Mt * 32, Kt * 32), 1))
        b = oracle.tilize(oracle.rand_bf16((Kt * 32, Nt * 32), 2))
        g = shard.GatheredTiles(Mt, Nt, device=0)
        g.fence = dist.barrier
        r0, r1 = g.rows
        ok &= (r0, r1) == shard.split_rows(Mt, world, rank)
        g.matmul(a[r0 * Kt * 1024:r1 * Kt * 1024], b, Kt)
        g.fence()
        mine = np.frombuffer(segs[g.ptr][0].buf, dtype=np.uint16, count=Mt * Nt * 1024).copy()
        ok &= np.array_equal(mine, oracle.matmul_tiles(a, b, Mt, Kt, Nt))
        g.close()
        ok &= calls == {"close": world - 1, "free": 1}
        dist.barrier()
        for base, (seg, _) in segs.items():
            if base != g.ptr:
                seg.close()
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,fail_open_on", [(2, None), (3, None), (3, 1)])
def test_gathered_tiles_host_logic(world, fail_open_on):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=gathered_worker, args=(r, world, port, q, fail_open_on)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok in res), res
