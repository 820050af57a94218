"""Two-GPU paths (skipped with fewer GPUs):

* row-sharded 'same' convolution (NCCL point-to-point halo exchange, then the
  implicit-GEMM kernel on each GPU): every rank's output rows equal the
  oracle's rows of the unsharded convolution;
* the row-sharded GEMM whose kernel is its own all-gather (every output tile
  stored to both GPUs' copies of C over NVLink, by the epilogue or by pusher
  warps): after the fence, both copies equal the per-rank results of the
  plain GEMM concatenated (bit for bit, same kernels), and the oracle on
  sampled rows; likewise with the GEMM in row chunks whose finished chunks
  the copy engines push to the peer ("ce"), and with every tile stored once
  through an NVLink multicast address (skipped without multicast support).
"""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def worker(rank, world, port, q):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "tt-foil_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    from oracle import oracle
    from ttfoil import shard
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = True
    try:
        for (N, H, W, Cin, Cout, K, pad) in ((2, 57, 40, 64, 128, 3, 1), (1, 30, 33, 32, 64, 5, 2)):
            x = oracle.rand_bf16((N, H, W, Cin), 20 + K)
            w = oracle.randn_bf16((Cout, K, K, Cin), 21 + K, np.sqrt(2.0 / (K * K * Cin)))
            b = oracle.rand_bf16((Cout,), 22 + K, -0.1, 0.1)
            h0, h1 = shard.split_rows(H, world, rank)
            dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()
            y = shard.conv2d_nhwc_h_sharded(dev(x[:, h0:h1]), dev(w), dev(b), N, h1 - h0, W, Cin, Cout, K, pad,
                                            relu=True)
            torch.cuda.synchronize()
            got = y.cpu().numpy().view(np.uint16)
            exp = oracle.conv_nhwc(x, w, b, 1, pad, relu=True, threads=8)[:, h0:h1]
            ok &= oracle.compare(got, exp)[0] == 0
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def gather_worker(rank, world, port, q):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "tt-foil_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    from oracle import oracle
    import ttfoil
    from ttfoil import shard
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = []
    try:
        # Mt odd -> uneven row split; Nt 8 (256-column kernel, the epilogue
        # stores to the peer) and 24 (512-column kernel, pusher warps copy
        # finished tiles to the peer).  Both are the plain GEMM's kernels.
        # "ce": the same GEMM in row chunks, copy engines push each chunk.
        cases = [(Mt, Kt, Nt, m, ch) for (Mt, Kt, Nt) in ((25, 16, 8), (19, 12, 24))
                 for (m, ch) in (("fused", 0), ("ce", 1), ("ce", 3))] + [(40, 4, 24, "ce", 64)]
        for (Mt, Kt, Nt, method, chunks) in cases:
            a_all = oracle.rand_bf16(Mt * Kt * 1024, 40 + Nt)
            b = oracle.rand_bf16(Kt * Nt * 1024, 41 + Nt)
            dev = lambda arr: torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda()
            g = shard.GatheredTiles(Mt, Nt)
            m0, m1 = g.rows
            a_r = dev(a_all[m0 * Kt * 1024:m1 * Kt * 1024])
            b_d = dev(b)
            g.tensor().fill_(0x7fff)
            torch.cuda.synchronize()
            dist.barrier()          # no rank's GEMM may land before every fill
            g.matmul(a_r, b_d, Kt, method=method, chunks=max(1, chunks))
            g.fence()
            torch.cuda.synchronize()
            full = g.tensor().cpu().numpy().view(np.uint16).copy()
            # the plain GEMM of this rank's rows, gathered on the host
            c_r = torch.empty((m1 - m0) * Nt * 1024, dtype=torch.int16, device="cuda")
            ttfoil.matmul_tiles(a_r, b_d, c_r, m1 - m0, Kt, Nt)
            torch.cuda.synchronize()
            parts = [None] * world
            dist.all_gather_object(parts, c_r.cpu().numpy().view(np.uint16))
            ref = np.concatenate(parts)
            ok.append(bool(np.array_equal(full, ref)))
            a_rm = oracle.untilize(a_all, Mt * 32, Kt * 32)
            b_rm = oracle.untilize(b, Kt * 32, Nt * 32)
            got = oracle.untilize(full, Mt * 32, Nt * 32)
            rows = [0, 31, 32 * m1 - 1, 32 * Mt - 1]
            exp = oracle.matmul(a_rm[rows], b_rm)
            ok.append(oracle.compare(got[rows], exp)[0] == 0)
            ok.append(ttfoil.device_error() == 0)
            g.close()
        # C copies only 16-byte aligned (base + 16 bytes): the 128-bit store
        # path (the 256-column kernel's epilogue writes the peer itself).
        Mt, Kt, Nt = 9, 4, 12
        a_all = oracle.rand_bf16(Mt * Kt * 1024, 60)
        b = oracle.rand_bf16(Kt * Nt * 1024, 61)
        dev = lambda arr: torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda()
        g = shard.GatheredTiles(Mt + 1, Nt)          # one spare tile row of room
        m0, m1 = shard.split_rows(Mt, world, rank)
        a_r, b_d = dev(a_all[m0 * Kt * 1024:m1 * Kt * 1024]), dev(b)
        torch.cuda.synchronize()
        dist.barrier()
        off = 16 + m0 * Nt * 2048
        peers = [g.bases[r] + off for r in range(world) if r != rank]
        ttfoil.matmul_tiles_gather(a_r, b_d, g.ptr + off, peers, m1 - m0, Kt, Nt)
        g.fence()
        torch.cuda.synchronize()
        full = g.tensor()[8:8 + Mt * Nt * 1024].cpu().numpy().view(np.uint16).copy()
        got = oracle.untilize(full, Mt * 32, Nt * 32)
        exp = oracle.matmul(oracle.untilize(a_all, Mt * 32, Kt * 32), oracle.untilize(b, Kt * 32, Nt * 32),
                            threads=4)
        ok.append(oracle.compare(got, exp)[0] == 0)
        ok.append(ttfoil.device_error() == 0)
        g.close()
        q.put((rank, all(ok), ok))
    finally:
        dist.destroy_process_group()


def mc_worker(rank, world, port, q):
    """MulticastTiles: the tiles stored once through the NVLink multicast
    address equal the plain GEMM's shards on both GPUs, bit for bit."""
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "tt-foil_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    from oracle import oracle
    import ttfoil
    from ttfoil import shard
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = []
    try:
        for (Mt, Kt, Nt) in ((25, 16, 8), (19, 12, 24), (3, 4, 24)):
            a_all = oracle.rand_bf16(Mt * Kt * 1024, 80 + Nt + Mt)
            b = oracle.rand_bf16(Kt * Nt * 1024, 81 + Nt + Mt)
            dev = lambda arr: torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda()
            try:
                g = shard.MulticastTiles(Mt, Nt)
            except RuntimeError as e:
                q.put((rank, True, ["skip: " + str(e)[:200]]))
                return
            m0, m1 = g.rows
            a_r = dev(a_all[m0 * Kt * 1024:m1 * Kt * 1024])
            b_d = dev(b)
            g.tensor().fill_(0x7fff)
            torch.cuda.synchronize()
            dist.barrier()
            g.matmul(a_r, b_d, Kt)
            g.fence()
            torch.cuda.synchronize()
            full = g.tensor().cpu().numpy().view(np.uint16).copy()
            c_r = torch.empty((m1 - m0) * Nt * 1024, dtype=torch.int16, device="cuda")
            ttfoil.matmul_tiles(a_r, b_d, c_r, m1 - m0, Kt, Nt)
            torch.cuda.synchronize()
            parts = [None] * world
            dist.all_gather_object(parts, c_r.cpu().numpy().view(np.uint16))
            ok.append(bool(np.array_equal(full, np.concatenate(parts))))
            ok.append(ttfoil.device_error() == 0)
            g.close()
        q.put((rank, all(ok), ok))
    finally:
        dist.destroy_process_group()


def run_two(target):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def test_gemm_is_its_own_allgather_two_gpus():
    res = run_two(gather_worker)
    assert all(r[1] for r in res), res


def test_gemm_allgather_through_multicast_two_gpus():
    res = run_two(mc_worker)
    assert all(r[1] for r in res), res
    skipped = [r for r in res if r[2] and str(r[2][0]).startswith("skip")]
    if skipped:
        pytest.skip(skipped[0][2][0])


def test_row_sharded_conv_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok in res), res
