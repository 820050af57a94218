"""Row-sharded 'same' convolution across 2 GPUs (NCCL point-to-point halo
exchange, then the implicit-GEMM kernel on each GPU): every rank's output
rows equal the oracle's rows of the unsharded convolution.  Needs 2 GPUs;
skipped otherwise."""
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
