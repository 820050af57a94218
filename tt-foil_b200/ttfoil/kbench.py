"""Per-kernel micro-benchmark of libfoil (CUDA events, operands resident in HBM).

    python -m ttfoil.kbench gemm    --m 8192 --n 8192 --k 8192 [--iters 20]
    python -m ttfoil.kbench tilize  --rows 16384 --cols 16384
    python -m ttfoil.kbench untilize --rows 16384 --cols 16384
    python -m ttfoil.kbench add     --n 268435456
    python -m ttfoil.kbench relu    --n 268435456
    python -m ttfoil.kbench bias    --rows 16384 --cols 16384
    python -m ttfoil.kbench copy    --bytes 1073741824
    python -m ttfoil.kbench conv    --batch 32 --hw 112 --cin 64 --cout 128 --ksize 3 --stride 2

Prints one JSON line: mean time per launch, TFLOP/s or GB/s of algorithmic
traffic.  Used for the secondary numbers of bench.py and as the command line
of the ncu captures summarised under profiles/.
"""
import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import ttfoil  # noqa: E402


_FLUSH = None


def _time(torch, fn, iters, warmup=3):
    """Mean ms per launch: back to back, or with --flush L2 flushed before
    each launch (256 MiB written, another 256 MiB read, outside the timing)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if _FLUSH is None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters
    evs = []
    for _ in range(iters):
        _FLUSH[0].add_(1)
        _FLUSH[1].sum()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / iters


def run(kind, args):
    import torch
    global _FLUSH
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    if args.flush:
        _FLUSH = (torch.zeros(1 << 26, dtype=torch.int32, device=dev),
                  torch.ones(1 << 26, dtype=torch.int32, device=dev))
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(n):
        return (torch.rand(n, device=dev, generator=g) * 2 - 1).to(torch.bfloat16)

    res = {"kernel": kind, "l2": "flushed" if args.flush else "back-to-back"}
    if kind == "gemm":
        M, N, K = args.m, args.n, args.k
        a, b = rnd(M * K), rnd(K * N)
        c = torch.empty(M * N, dtype=torch.bfloat16, device=dev)
        bias = rnd(N) if args.bias else None
        ms = _time(torch, lambda: ttfoil.matmul_tiles(a, b, c, M // 32, K // 32, N // 32, bias=bias,
                                                       relu=args.relu), args.iters)
        res.update(M=M, N=N, K=K, ms=ms, tflops=2.0 * M * N * K / ms / 1e9)
    elif kind in ("tilize", "untilize", "bias"):
        R, C = args.rows, args.cols
        x, y = rnd(R * C), torch.empty(R * C, dtype=torch.bfloat16, device=dev)
        if kind == "tilize":
            fn = lambda: ttfoil.tilize(x, y, R, C)
            nbytes = 4 * R * C
        elif kind == "untilize":
            fn = lambda: ttfoil.untilize(x, y, R, C)
            nbytes = 4 * R * C
        else:
            band = rnd(32 * C)
            fn = lambda: ttfoil.bias_add_tiles(x, band, y, R, C)
            nbytes = 4 * R * C
        ms = _time(torch, fn, args.iters)
        res.update(rows=R, cols=C, ms=ms, gbs=nbytes / ms / 1e6)
    elif kind in ("add", "relu"):
        n = args.n
        x, y, o = rnd(n), rnd(n) if kind == "add" else None, torch.empty(n, dtype=torch.bfloat16, device=dev)
        if kind == "add":
            fn = lambda: ttfoil.add_tiles(x, y, o, n)
            nbytes = 6 * n
        else:
            fn = lambda: ttfoil.relu_tiles(x, o, n)
            nbytes = 4 * n
        ms = _time(torch, fn, args.iters)
        res.update(n=n, ms=ms, gbs=nbytes / ms / 1e6)
    elif kind == "conv":
        N, H, W, Cin, Cout, KH, stride, pad = (args.batch, args.hw, args.hw, args.cin, args.cout,
                                               args.ksize, args.stride, args.pad)
        Ho = (H + 2 * pad - KH) // stride + 1
        Wo = (W + 2 * pad - KH) // stride + 1
        x = rnd(N * H * W * Cin)
        w = rnd(Cout * KH * KH * Cin) * 0.05
        bias = rnd(Cout) * 0.1
        y = torch.empty(N * Ho * Wo * Cout, dtype=torch.bfloat16, device=dev)
        ms = _time(torch, lambda: ttfoil.conv2d_nhwc(x, w, bias, y, N, H, W, Cin, Cout, KH, KH,
                                                       stride, pad, relu=True), args.iters)
        flops = 2.0 * N * Ho * Wo * Cout * KH * KH * Cin
        nbytes = 2.0 * (N * H * W * Cin + Cout * KH * KH * Cin + N * Ho * Wo * Cout)
        res.update(N=N, H=H, W=W, Cin=Cin, Cout=Cout, k=KH, stride=stride, pad=pad, ms=ms,
                   tflops=flops / ms / 1e9, gbs=nbytes / ms / 1e6)
    elif kind == "copy":
        nb = args.bytes
        x = torch.empty(nb // 2, dtype=torch.int16, device=dev).random_()
        y = torch.empty_like(x)
        ms = _time(torch, lambda: ttfoil.tile_copy(x, y, nb), args.iters)
        res.update(bytes=nb, ms=ms, gbs=2 * nb / ms / 1e6)
    else:
        raise SystemExit(f"unknown kernel {kind}")
    assert ttfoil.device_error() == 0
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel")
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--cols", type=int, default=16384)
    ap.add_argument("--bytes", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--bias", action="store_true")
    ap.add_argument("--relu", action="store_true")
    ap.add_argument("--flush", action="store_true", help="flush L2 before each timed launch")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--hw", type=int, default=56)
    ap.add_argument("--cin", type=int, default=64)
    ap.add_argument("--cout", type=int, default=64)
    ap.add_argument("--ksize", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--pad", type=int, default=1)
    args = ap.parse_args()
    if args.kernel in ("add", "relu") and args.n == 8192:
        args.n = 1 << 28
    print(json.dumps(run(args.kernel, args)))


if __name__ == "__main__":
    main()
