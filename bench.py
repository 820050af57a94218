"""Benchmark of the B200 tt-foil hot path: the tiled bf16 GEMM at 8192^3.

One step = one C (8192 x 8192) = A (8192 x 8192) . B (8192 x 8192) product per
GPU on 32x32-tile-layout bf16 operands with fp32 accumulation (the tt-foil
matmul_dram program at Mt = Kt = Nt = 256), run by the sm_100a tcgen05 kernel
of libfoil.  With N GPUs (torchrun, one process per GPU) every rank computes
its own 8192-row shard of an (8192 N) x 8192 x 8192 product (weak scaling, no
collective inside the step).  Reassembling the global tile-layout C is timed
separately under "allgather": ncclAllGather after the GEMM; ("fused") the
GEMM kernel that stores every C tile into all ranks' copies over NVLink
itself; and ("copy_engines") the GEMM in row chunks whose finished chunks the
copy engines send to the peers while the next chunk computes; the last two
followed by a one-element all-reduce.

value      TFLOP/s over all ranks, operands resident in HBM, CUDA events on the
           launching stream, max over ranks.
value_with_gather  (N > 1) the same step with the global C reassembled on every
           rank: the best of GEMM + ncclAllGather, the fused GEMM that stores
           each tile to every rank's copy over NVLink (per peer; with
           --gather-multicast also once through an NVLink multicast
           address), and the GEMM in row
           chunks whose finished chunks the copy engines send to the peers
           while the next chunk computes, with the achieved NVLink GB/s
           against the link floor.
e2e        TFLOP/s of the same GEMM on host buffers through the public entry
           point foil_matmul_tiles_host (pinned A, B in; C out; copies of
           chunk i+1 and read-back of chunk i-1 overlap the GEMM of chunk i)
           every step, host timer around the blocking call, max over ranks.
           "runtime_api" inside it: the same through the tt-foil runtime API
           (write_buffer A and B, execute matmul_dram, read_buffer C), the
           reference's blocking sequence.
roofline   GEMM FLOPs per launch / mean launch time against the measured bf16
           peak (MEASURED_PEAKS.json): the burst figure, or the sustained one
           when the clock samples of the timed region show the power cap
           holding the SM clock below 95 % of its maximum; both fractions are
           in the line.
cpu_baseline  the oracle (the reference golden's loop nest, oracle/golden.cpp)
           on a bounded sample of output rows, all host threads, rank 0, N=1.
secondary  the other parts of the metric, each on every rank with CUDA events
           (max over ranks; values summed over ranks):
           conv   3x3 s1 56^2x64->64 (N=1) and the batch-32 pair 3x3 s2
                  112^2x64->128 + 1x1 56^2x128->256, bias+relu, batch sharded
                  over ranks; TFLOP/s and algorithmic HBM GB/s against the
                  measured HBM peak (both convolutions are HBM-bound: the
                  working set is below L2, so L2 is flushed before each timed
                  launch: a 256 MiB buffer written, then another read);
           gemm   4096^3 and 16384^3 per rank, 65536x8192x8192 M-sharded;
           eltwise tilize / untilize 16384^2, add_tiles / bias_add / relu on
                  2^28 elements, tile_copy of 1 GiB: GB/s of algorithmic
                  traffic against the measured HBM peak;
           cpu    the oracle restatements of the conv and elementwise goldens
                  on bounded samples (rank 0, N=1).

--impl reference times the reference's CPU golden implementation of the same
workload on the same sample as cpu_baseline (one whole 32-row block of the
8192^3 product per host thread, each timed step) and prints its line.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "tt-foil_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "bf16 tile-GEMM TFLOP/s & % peak @8192³; conv TFLOP/s; eltwise HBM GB/s"
M_PER_GPU = N_DIM = K_DIM = 8192
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gather-chunks", type=int, default=8,
                    help="row chunks of the copy-engine reassembly path (N > 1)")
    ap.add_argument("--gather-multicast", action="store_true",
                    help="also time the NVLink-multicast reassembly path (N > 1; measured slower: "
                         "2.77 against 1.68 ms per step at 8 GPUs)")
    return ap.parse_args()


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


# ------------------------------------------------------------ distributed ---
class Dist:
    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x):
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------- clocks ---
def smi_id(cuda_index):
    """nvidia-smi identifier of a CUDA device: its UUID (CUDA ordinals and
    nvidia-smi indices differ when visible devices are remapped)."""
    import torch
    try:
        u = str(torch.cuda.get_device_properties(cuda_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(cuda_index)



class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.idx)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.15)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9:
                    rows.append(p)
        os.unlink(self.path)
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        under_load = [s for s in sm if s > 600] or sm
        return {"sm_mhz": statistics.median(under_load) if under_load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()),
                                   default=None)}


# ----------------------------------------------------------- CPU baseline ---
def _run_blocks(fn, a_blocks, b, n_blocks, threads):
    """n_blocks calls fn(a_blocks[i % len], b) spread over `threads` Python
    threads (the ctypes call releases the GIL); returns the elapsed seconds."""
    import threading
    todo = list(range(n_blocks))
    lock = threading.Lock()

    def worker():
        while True:
            with lock:
                if not todo:
                    return
                i = todo.pop()
            fn(a_blocks[i % len(a_blocks)], b)

    ts = [threading.Thread(target=worker) for _ in range(max(1, min(threads, n_blocks)))]
    t0 = time.perf_counter()
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    return time.perf_counter() - t0


def cpu_gemm_baseline(seconds, threads):
    """The reference's own golden matmul (tests/test_matmul_mnk.cpp:62-76,
    compiled from the reference sources into oracle/_ref) on whole 32-row
    blocks of the 8192^3 workload, one block per host thread (at most 32)
    in parallel: the same sample as one step of --impl reference.  Falls
    back to the oracle port (same loop nest, bit-equal results) for
    `seconds` when oracle/_ref is absent."""
    import numpy as np
    from oracle import oracle
    K = N = 8192
    ref = oracle.ref_matmul_8192(N)
    if ref is not None:
        t = max(1, min(threads, 32))
        a_blocks = [oracle.rand_bf16((32, K), 91 + i) for i in range(t)]
        b = oracle.rand_bf16((K, N), 92)
        el = _run_blocks(ref, a_blocks, b, t, t)
        flops = 2.0 * 32 * t * N * K
        return {"value": flops / el / 1e12, "unit": "TFLOP/s", "cores": t, "kind": "reference",
                "sample": f"{t} blocks of 32 output rows x 8192 cols (K=8192) of the 8192^3 product, "
                          f"one per thread, {el:.1f} s; the reference's golden loop compiled from its "
                          f"sources"}
    rows = max(threads, 1)
    a = oracle.rand_bf16((rows, K), 91)
    b = oracle.rand_bf16((K, N), 92)
    done_rows = 0
    t0 = time.perf_counter()
    while True:
        oracle.matmul(a, b, rows=(0, rows), threads=threads)
        done_rows += rows
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    flops = 2.0 * done_rows * N * K
    return {"value": flops / el / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{done_rows} output rows x 8192 cols (K=8192) of the 8192^3 product, "
                      f"{el:.1f} s"}


def gemm_config(world):
    return {"workload": "tiled bf16 GEMM 8192x8192x8192 per GPU "
                        "(tt-foil 32x32 tile / 16x16 face layout, fp32 accumulate)",
            "M_per_gpu": M_PER_GPU, "N": N_DIM, "K": K_DIM, "global_M": M_PER_GPU * world,
            "parallelism": f"M-shard x{world}",
            "l2": "operands 384 MiB per GPU > 126 MB L2, no flush"}


# ------------------------------------------------------------- reference ---
def run_reference(args, dist):
    """The reference's CPU implementation of the path: its golden matmul
    (tests/test_matmul_mnk.cpp:62-76, compiled from its sources into
    oracle/_ref; the bit-identical oracle port when that is absent) on rank 0
    with one thread per host core (at most 32).  Each timed step is the same
    sample as cpu_baseline: one whole 32-row block (32 x 8192 outputs,
    K = 8192) of the 8192^3 product per thread, in parallel.  The warm-up
    steps are untimed single 32 x 32 output tiles: the loop needs no warm-up
    beyond its first touch of the operands, and a whole block takes ~18 s."""
    if dist.rank != 0:
        return
    import numpy as np
    threads = host_threads()
    from oracle import oracle
    K = N = 8192
    t = max(1, min(threads, 32))
    a_blocks = [oracle.rand_bf16((32, K), 91 + i) for i in range(t)]
    b = oracle.rand_bf16((K, N), 92)
    fn, kind = oracle.ref_matmul_8192(N), "reference"
    if fn is None:
        kind = "port"
        fn = lambda a, bb: oracle.matmul(a, bb, threads=1)
    tile = oracle.ref_matmul_8192(32)
    if tile is not None:
        b_tile = np.ascontiguousarray(b[:, :32])
        for _ in range(args.warmup):
            tile(a_blocks[0], b_tile)
    el = 0.0
    for _ in range(args.steps):
        el += _run_blocks(fn, a_blocks, b, t, t)
    flops = 2.0 * 32 * N * K * t * args.steps
    v = flops / el / 1e12
    sample = (f"{t} blocks of 32 output rows x 8192 cols (K=8192) of the 8192^3 product per step, "
              f"one per thread; the reference's golden loop" +
              (" compiled from its sources" if kind == "reference" else " (oracle port)"))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic seeded U(-1,1) bf16",
            "config": gemm_config(dist.world),
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": t, "kind": kind,
                             "sample": sample},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours ---
def run_ours(args, dist):
    import numpy as np
    import torch
    import ttfoil

    torch.cuda.set_device(dist.local)
    dev = torch.device("cuda", dist.local)
    Mt, Kt, Nt = M_PER_GPU // 32, K_DIM // 32, N_DIM // 32
    flops = 2.0 * M_PER_GPU * N_DIM * K_DIM

    # Synthetic operands (seeded U(-1,1) bf16), tile layout; B identical on
    # every rank, A is this rank's row shard.
    g = torch.Generator(device=dev).manual_seed(1234 + dist.rank)
    gb = torch.Generator(device=dev).manual_seed(99)
    a_rm = (torch.rand(M_PER_GPU, K_DIM, device=dev, generator=g) * 2 - 1).to(torch.bfloat16)
    b_rm = (torch.rand(K_DIM, N_DIM, device=dev, generator=gb) * 2 - 1).to(torch.bfloat16)
    a = torch.empty(M_PER_GPU * K_DIM, dtype=torch.bfloat16, device=dev)
    b = torch.empty(K_DIM * N_DIM, dtype=torch.bfloat16, device=dev)
    c = torch.empty(M_PER_GPU * N_DIM, dtype=torch.bfloat16, device=dev)
    ttfoil.tilize(a_rm, a, M_PER_GPU, K_DIM)
    ttfoil.tilize(b_rm, b, K_DIM, N_DIM)
    torch.cuda.synchronize()
    del a_rm, b_rm

    stream = torch.cuda.current_stream()

    def step():
        ttfoil.matmul_tiles(a, b, c, Mt, Kt, Nt, stream=stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    assert ttfoil.device_error(stream) == 0

    clocks = ClockSampler(smi_id(dist.local))
    clocks.start()
    launches0 = ttfoil.launch_count()
    dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    launches = ttfoil.launch_count() - launches0
    clk = clocks.stop()
    ms_local = ev0.elapsed_time(ev1)
    ms = dist.max(ms_local)
    assert ttfoil.device_error(stream) == 0
    value = dist.world * flops * args.steps / (ms / 1e3) / 1e12

    # Spot-check a few output rows of this rank against the oracle.
    check = spot_check(ttfoil, a, b, c, Mt, Kt, Nt) if dist.rank == 0 else None

    # Roofline of the dominant (only) kernel: FLOPs per launch / launch time.
    pk, pk_kind = peaks()
    per_launch_ms = ms_local / args.steps
    achieved = flops / (per_launch_ms / 1e3) / 1e12
    traffic = read_traffic()
    peak, capped = roofline_peak(pk, clk)
    burst, sustained = pk["bf16_tflops"], pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak,
                "frac_of_burst": achieved / burst, "frac_of_sustained": achieved / sustained,
                "peak_kind": f"{pk_kind} {'sustained (power-capped clocks in the timed region)' if capped else 'burst'}"
                             " cuBLAS bf16",
                "traffic": traffic,
                "algorithmic_bytes": 2.0 * (M_PER_GPU * K_DIM + K_DIM * N_DIM + M_PER_GPU * N_DIM)}

    # All-gather of the C shards (reassembly of the global tile-layout C), and
    # the headline with it: the better of GEMM + ncclAllGather and the fused
    # GEMM that stores every tile to all ranks' copies itself.
    allgather = None
    with_gather = None
    if dist.world > 1:
        allgather = time_allgather(dist, c, ms / args.steps, flops)
        methods = [("fused", "fused"), ("copy_engines", "ce")]
        if args.gather_multicast:
            methods.append(("multicast", "multicast"))
        for key, method in methods:
            try:
                allgather[key] = time_fused_gather(dist, a, b, Mt, Kt, Nt, flops, method=method,
                                                   chunks=args.gather_chunks)
            except RuntimeError as e:  # raised on every rank alike (see GatheredTiles)
                allgather[key] = {"unavailable": str(e)[:300]}
        shard_bytes = M_PER_GPU * N_DIM * 2
        recv = (dist.world - 1) * shard_bytes  # C bytes every GPU must receive per step
        link_gbs = 770.0  # measured peer copy per direction per GPU on this pool
        nccl_ms = ms / args.steps + allgather["ms"]
        step_of = lambda k: allgather.get(k, {}).get("ms_per_step")
        fused_ms, ce_ms, mc_ms = step_of("fused"), step_of("copy_engines"), step_of("multicast")
        paths = {"ncclAllGather": nccl_ms, "fused": fused_ms, "multicast": mc_ms, "copy_engines": ce_ms}
        best = best_path(paths)
        step_ms = paths[best]
        with_gather = {
            "value": dist.world * flops / (step_ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": step_ms,
            "path": best, "nccl_ms_per_step": nccl_ms, "fused_ms_per_step": fused_ms,
            "copy_engines_ms_per_step": ce_ms, "multicast_ms_per_step": mc_ms,
            "nvlink_GBps_multicast": recv / (mc_ms / 1e3) / 1e9 if mc_ms else None,
            "received_bytes_per_gpu": recv,
            "nvlink_GBps_fused": recv / (fused_ms / 1e3) / 1e9 if fused_ms else None,
            "nvlink_GBps_copy_engines": recv / (ce_ms / 1e3) / 1e9 if ce_ms else None,
            "allgather_busbw_GBps": allgather["busbw_GBps"],
            "link_floor_ms": recv / (link_gbs * 1e9) * 1e3,
            "compute_floor_ms": ms / args.steps,
            "note": "per step: the GEMM of every rank's 8192-row shard plus reassembly of the whole C on "
                    "every rank; floor = max(compute, received bytes at 770 GB/s per direction)"}

    e2e = None if args.no_e2e else run_e2e(args, dist, flops)

    secondary = None if args.no_secondary else run_secondary(dist, pk)

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_gemm_baseline(args.cpu_seconds, host_threads())
        if secondary is not None:
            secondary["cpu"] = cpu_secondary_baseline(host_threads())

    if dist.rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": dist.world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic seeded U(-1,1) bf16, 32x32 tile layout",
                "config": gemm_config(dist.world),
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
                "gpu_launches": launches, "parity_spot_check": check, "secondary": secondary}
        if allgather:
            line["allgather"] = allgather
            line["value_with_gather"] = with_gather
        print(json.dumps(line), flush=True)


def roofline_peak(pk, clk):
    """(peak TFLOP/s, capped) for the GEMM roofline: the burst cuBLAS figure
    while the SM clock held its maximum in the timed region, the sustained
    (power-capped) one when the clock samples show the power cap holding the
    median SM clock below 95 % of its maximum, as in a long run of steps."""
    burst, sustained = pk["bf16_tflops"], pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    capped = bool(clk and clk.get("sm_mhz") and clk.get("sm_max_mhz") and
                  clk["sm_mhz"] < 0.95 * clk["sm_max_mhz"] and "sw_power_cap" in clk.get("reasons", []))
    return (sustained if capped else burst), capped


def best_path(paths):
    """Name of the fastest reassembly path: `paths` maps names to ms per
    step, None for a path that did not run."""
    return min((v, k) for k, v in paths.items() if v is not None)[1]


def _timed(torch, fn, iters, flush=None, warmup=3):
    """Mean device time (ms) of fn over `iters` launches on the current
    stream: back to back between one pair of events, or with `flush` (two
    256 MiB buffers) one event pair per launch, and before each launch,
    outside the timed interval, one buffer rewritten and the other read, so
    that no operand starts in L2 and the rewrite's dirty lines have been
    written back before the timed launch."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if flush is None:
        # Back-to-back launches between one pair of events (operands > L2).
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
        flush[0].add_(1)
        flush[1].sum()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in evs)


def run_secondary(dist, pk):
    """Conv, GEMM-sweep and memory-bound numbers of the metric (see the module
    docstring).  Every rank runs the same launches; times are max over ranks."""
    import torch
    import ttfoil

    dev = torch.device("cuda", dist.local)
    g = torch.Generator(device=dev).manual_seed(777 + dist.rank)
    hbm = pk["hbm_gbs"]

    def rnd(n, scale=1.0):
        return ((torch.rand(n, device=dev, generator=g) * 2 - 1) * scale).to(torch.bfloat16)

    flush = (torch.zeros(256 << 18, dtype=torch.int32, device=dev),   # 2 x 256 MiB > L2
             torch.ones(256 << 18, dtype=torch.int32, device=dev))
    out = {}

    # ---- memory-bound sweep (config 5), first: measured right after the dense
    # GEMM sweep (the part at its power cap) these kernels ran ~10 % slower.
    elt = {}
    R = C = 16384
    x, y = rnd(R * C), torch.empty(R * C, dtype=torch.bfloat16, device=dev)
    for name, fn in (("tilize_16384^2", lambda: ttfoil.tilize(x, y, R, C)),
                     ("untilize_16384^2", lambda: ttfoil.untilize(x, y, R, C))):
        ms = dist.max(_timed(torch, fn, 20))
        elt[name] = 4.0 * R * C / (ms / 1e3) / 1e9
    band = rnd(32 * C)
    ms = dist.max(_timed(torch, lambda: ttfoil.bias_add_tiles(x, band, y, R, C), 20))
    elt["bias_add_2^28"] = (4.0 * R * C + 64.0 * C) / (ms / 1e3) / 1e9
    n = 1 << 28
    z = rnd(n)
    ms = dist.max(_timed(torch, lambda: ttfoil.add_tiles(x, z, y, n), 20))
    elt["add_tiles_2^28"] = 6.0 * n / (ms / 1e3) / 1e9
    ms = dist.max(_timed(torch, lambda: ttfoil.relu_tiles(x, y, n), 20))
    elt["relu_2^28"] = 4.0 * n / (ms / 1e3) / 1e9
    del x, y, z, band
    nbytes = 1 << 30
    src = torch.empty(nbytes // 2, dtype=torch.int16, device=dev).random_(generator=g)
    dst = torch.empty_like(src)
    ms = dist.max(_timed(torch, lambda: ttfoil.tile_copy(src, dst, nbytes), 20))
    elt["tile_copy_1GiB"] = 2.0 * nbytes / (ms / 1e3) / 1e9
    del src, dst
    out["eltwise_GBps_per_gpu"] = elt
    out["eltwise_frac_of_hbm"] = {k: v / hbm for k, v in elt.items()}

    # ---- conv (configs: 3x3 s1 N=1, and the batch-32 pair sharded by batch)
    # The per-launch figure brackets one launch with events after an L2
    # flush; that method reads ~6 us even for an empty kernel (launch_floor).
    # "stream" also times back-to-back launches that cycle through `sets`
    # copies of the operands, together more than twice L2, so every launch
    # reads inputs that other launches have evicted and the outputs' write-
    # backs land inside the timed interval.
    tiny = torch.zeros(1, dtype=torch.int32, device=dev)
    floor_ms = dist.max(_timed(torch, lambda: tiny.add_(1), 20, flush))
    l2_bytes = 126 * 2 ** 20

    def conv_case(N, H, Cin, Cout, k, stride, pad, x=None, stream=False):
        Ho = (H + 2 * pad - k) // stride + 1
        x = rnd(N * H * H * Cin) if x is None else x
        w = rnd(Cout * k * k * Cin, (2.0 / (k * k * Cin)) ** 0.5)
        b = rnd(Cout, 0.1)
        y = torch.empty(N * Ho * Ho * Cout, dtype=torch.bfloat16, device=dev)
        fn = lambda: ttfoil.conv2d_nhwc(x, w, b, y, N, H, H, Cin, Cout, k, k, stride, pad, relu=True)
        ms = dist.max(_timed(torch, fn, 20, flush))
        flops = 2.0 * N * Ho * Ho * Cout * k * k * Cin
        nbytes = 2.0 * (N * H * H * Cin + Cout * k * k * Cin + Cout + N * Ho * Ho * Cout)
        gbs = dist.world * nbytes / (ms / 1e3) / 1e9
        res = {"us": ms * 1e3, "TFLOPs": dist.world * flops / (ms / 1e3) / 1e12,
               "hbm_GBps": gbs, "hbm_frac": gbs / (dist.world * hbm), "bound": "hbm",
               "algorithmic_bytes_per_rank": nbytes, "flops_per_rank": flops}
        if stream:
            sets = max(2, int(-(-2 * l2_bytes // nbytes)))
            ops = [(x, y)] + [(rnd(N * H * H * Cin), torch.empty_like(y)) for _ in range(sets - 1)]
            it = iter(range(1 << 30))

            def nxt():
                xi, yi = ops[next(it) % sets]
                ttfoil.conv2d_nhwc(xi, w, b, yi, N, H, H, Cin, Cout, k, k, stride, pad, relu=True)
            sms = dist.max(_timed(torch, nxt, 10 * sets, warmup=sets))
            sg = dist.world * nbytes / (sms / 1e3) / 1e9
            res["stream"] = {"us": sms * 1e3, "hbm_GBps": sg, "hbm_frac": sg / (dist.world * hbm),
                             "operand_sets": sets, "footprint_bytes": sets * nbytes}
            del ops
        return y, res

    _, c2 = conv_case(1, 56, 64, 64, 3, 1, 1)
    nb = max(1, 32 // dist.world)
    y1, c3a = conv_case(nb, 112, 64, 128, 3, 2, 1, stream=True)
    _, c3b = conv_case(nb, 56, 128, 256, 1, 1, 0, x=y1, stream=True)
    pair_us = c3a["us"] + c3b["us"]
    pair_flops = dist.world * (c3a["flops_per_rank"] + c3b["flops_per_rank"])
    out["conv"] = {"conv3x3_s1_56x56x64_n1": c2,
                   "conv3x3_s2_112x112x64to128": dict(c3a, batch_per_rank=nb),
                   "conv1x1_56x56x128to256": dict(c3b, batch_per_rank=nb),
                   "pair_TFLOPs": pair_flops / (pair_us / 1e6) / 1e12,
                   "pair_us": pair_us, "global_batch": nb * dist.world,
                   "launch_floor_us": floor_ms * 1e3,
                   "l2": "flushed before each timed launch (256 MiB written, another 256 MiB read); "
                         "launch_floor_us: a one-element torch kernel timed the same way; 'stream': "
                         "back-to-back launches over operand copies totalling more than twice L2"}

    # ---- GEMM sweep (config 4): square per rank, tall M-sharded
    sweep = {}
    for name, (M, K, N) in {"4096^3": (4096, 4096, 4096), "16384^3": (16384, 16384, 16384),
                            "65536x8192x8192": (65536 // dist.world, 8192, 8192)}.items():
        a, b = rnd(M * K), rnd(K * N)
        c = torch.empty(M * N, dtype=torch.bfloat16, device=dev)
        fn = lambda: ttfoil.matmul_tiles(a, b, c, M // 32, K // 32, N // 32)
        small = 2 * (M * K + K * N + M * N) < (128 << 20)
        ms = dist.max(_timed(torch, fn, 10 if M * N * K > 2 ** 40 else 30, flush if small else None))
        t = dist.world * 2.0 * M * N * K / (ms / 1e3) / 1e12
        sweep[name] = {"M_per_rank": M, "N": N, "K": K, "ms": ms, "TFLOPs": t,
                       "frac_of_peak": t / (dist.world * pk["bf16_tflops"])}
        del a, b, c
    out["gemm_sweep"] = sweep

    assert ttfoil.device_error() == 0
    return out


def cpu_secondary_baseline(threads):
    """Oracle restatements of the conv and elementwise goldens on bounded
    samples: one image of the 3x3 s2 conv, a 4096^2 tilize, 2^24-element add."""
    from oracle import oracle
    res = {"cores": threads, "kind": "port"}
    x = oracle.rand_bf16((1, 112, 112, 64), 3)
    w = oracle.randn_bf16((128, 3, 3, 64), 31, (2.0 / 576) ** 0.5)
    b = oracle.rand_bf16((128,), 32, -0.1, 0.1)
    t0 = time.perf_counter()
    oracle.conv_nhwc(x, w, b, 2, 1, relu=True, threads=threads)
    el = time.perf_counter() - t0
    res["conv3x3_s2_TFLOPs"] = 2.0 * 56 * 56 * 128 * 576 / el / 1e12
    res["conv_sample"] = f"1 image of 112^2x64->128 3x3 s2, {el:.2f} s"
    m = oracle.rand_bf16((4096, 4096), 5)
    t0 = time.perf_counter()
    oracle.tilize(m)
    el = time.perf_counter() - t0
    res["tilize_GBps"] = 4.0 * 4096 * 4096 / el / 1e9
    a = oracle.rand_bf16((1 << 24,), 6)
    c = oracle.rand_bf16((1 << 24,), 7)
    t0 = time.perf_counter()
    oracle.add(a, c)
    el = time.perf_counter() - t0
    res["add_GBps"] = 6.0 * (1 << 24) / el / 1e9
    res["eltwise_sample"] = "4096^2 tilize, 2^24-element add_tiles (single-threaded golden loops)"
    return res


def bits(t):
    """bf16 CUDA tensor -> numpy uint16 bit patterns."""
    import numpy as np
    import torch
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def spot_check(ttfoil, a, b, c, Mt, Kt, Nt):
    """Three output rows of the timed product against the oracle."""
    from oracle import oracle
    rows = [0, 4097, 8191]
    K, N = Kt * 32, Nt * 32
    b_h = oracle.untilize(bits(b), K, N)
    a_h, c_h = bits(a), bits(c)
    worst = 0.0
    for r in rows:
        mt, r0 = divmod(r, 32)
        a_row = oracle.untilize(a_h[mt * Kt * 1024:(mt + 1) * Kt * 1024], 32, K)[r0:r0 + 1]
        c_row = oracle.untilize(c_h[mt * Nt * 1024:(mt + 1) * Nt * 1024], 32, N)[r0:r0 + 1]
        exp = oracle.matmul(a_row, b_h, threads=8)
        worst = max(worst, oracle.normalized_error(c_row, exp, K, 1.0, 1.0))
    return {"rows": rows, "normalized_error": worst, "tolerance": 1e-2, "ok": worst <= 1e-2}


def read_traffic():
    """DRAM bytes per GEMM launch from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "gemm_tc_8192.md")
    if os.path.exists(path):
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch"):
                    return float(line.split("=")[1])
    return None


def time_allgather(dist, c, compute_ms, flops):
    import torch
    out = torch.empty(c.numel() * dist.world, dtype=c.dtype, device=c.device)
    for _ in range(3):
        dist.pg.all_gather_into_tensor(out, c)
    torch.cuda.synchronize()
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    it = 10
    e0.record()
    for _ in range(it):
        dist.pg.all_gather_into_tensor(out, c)
    e1.record()
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1)) / it
    nbytes = c.numel() * c.element_size()
    busbw = nbytes * (dist.world - 1) / (ms / 1e3) / 1e9
    return {"ms": ms, "bytes_per_rank": nbytes, "busbw_GBps": busbw,
            "value_with_gather_TFLOPs": dist.world * flops / ((compute_ms + ms) / 1e3) / 1e12,
            "note": "ncclAllGather of the C shards after the step, timed separately"}


def time_fused_gather(dist, a, b, Mt, Kt, Nt, flops, method="fused", chunks=8):
    """The same per-rank GEMM with its own all-gather into all ranks' copies
    of the global C over NVLink (ttfoil.shard.GatheredTiles), then a
    one-element all-reduce orders the ranks' launches.  method "fused": one
    kernel per rank whose pusher warps store every tile to the peers; "ce":
    the GEMM in `chunks` row chunks, each finished chunk copied to the peers
    by the copy engines while the next computes.  Time per step = GEMM +
    transfer + fence, max over ranks."""
    import torch
    import ttfoil
    from ttfoil import shard
    if method == "multicast":
        g = shard.MulticastTiles(Mt * dist.world, Nt)
        mm = lambda: g.matmul(a, b, Kt)
    else:
        g = shard.GatheredTiles(Mt * dist.world, Nt)
        mm = lambda: g.matmul(a, b, Kt, method=method, chunks=chunks)
    try:
        assert g.rows == (dist.rank * Mt, (dist.rank + 1) * Mt)

        def step():
            mm()
            g.fence()

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        it = 10
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(it):
            step()
        e1.record()
        torch.cuda.synchronize()
        ms = dist.max(e0.elapsed_time(e1)) / it
        assert ttfoil.device_error() == 0
        # every rank's copy holds the whole C: compare a checksum of each
        # rank's own rows in its copy with that slice in rank 0's copy
        full = g.tensor()
        sums = torch.stack([full[r * Mt * Nt * 1024:(r + 1) * Mt * Nt * 1024].float().sum()
                            for r in range(dist.world)]).double()
        ref = sums.clone()
        dist.pg.broadcast(ref, 0)
        consistent = bool(torch.equal(sums, ref))
    finally:
        g.close()
    note = {"fused": "one GEMM kernel per rank that also stores each C tile to every peer GPU's copy "
                     "over NVLink (256x512 pair tiles; four pusher warps copy finished tiles to the peers "
                     "while later tiles compute), plus a one-element all-reduce",
            "multicast": "the same kernel whose pusher warps store each C tile once through an NVLink "
                         "multicast address (PyTorch symmetric memory); the NVSwitch writes it into every "
                         "GPU's copy; plus a one-element all-reduce",
            "ce": f"the GEMM as {chunks} row-chunk launches per rank; one copy stream per peer copies each "
                  "finished chunk over NVLink (copy engines) while the next chunk computes, plus a "
                  "one-element all-reduce"}[method]
    out = {"ms_per_step": ms, "value_TFLOPs": dist.world * flops / (ms / 1e3) / 1e12,
           "copies_consistent": consistent, "note": note}
    if method == "ce":
        out["chunks"] = chunks
    return out


def run_e2e(args, dist, flops):
    """Same GEMM with host buffers: the pipelined entry point, and the
    reference's blocking write / execute / read sequence through the runtime."""
    import torch
    import ttfoil

    Mt, Kt, Nt = M_PER_GPU // 32, K_DIM // 32, N_DIM // 32
    a_bytes, b_bytes, c_bytes = Mt * Kt * 2048, Kt * Nt * 2048, Mt * Nt * 2048
    pin = lambda n: torch.empty(n // 2, dtype=torch.int16, pin_memory=True)
    a_h, b_h, c_h = pin(a_bytes), pin(b_bytes), pin(c_bytes)
    # Seeded U(-1,1) rounded to bf16, as the config states (i.i.d., so the
    # tile order of the stream does not matter).
    g = torch.Generator().manual_seed(5 + dist.rank)
    for h in (a_h, b_h):
        h.copy_((torch.rand(h.numel(), generator=g) * 2 - 1).to(torch.bfloat16).view(torch.int16))

    def pipelined():
        ttfoil.matmul_tiles_host(dist.local, a_h, b_h, c_h, Mt, Kt, Nt)

    for _ in range(3):
        pipelined()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        pipelined()
    el_p = dist.max(time.perf_counter() - t0)
    dist.barrier()
    ttfoil.host_pipeline_release(dist.local)

    with ttfoil.Device(dist.local) as d:
        ba = d.allocate(ttfoil.LOC_DRAM, a_bytes)
        bb = d.allocate(ttfoil.LOC_DRAM, b_bytes)
        bc = d.allocate(ttfoil.LOC_DRAM, c_bytes)
        k = d.load_program("matmul_dram")
        an, bn, cn = (d.noc_dram_addr(x.device_addr) for x in (ba, bb, bc))
        d.set_runtime_args(k, ttfoil.BRISC, [ttfoil.lo(an), ttfoil.hi(an), ttfoil.lo(bn),
                                             ttfoil.hi(bn), Mt, Kt, Nt])
        d.set_runtime_args(k, ttfoil.NCRISC, [ttfoil.lo(cn), ttfoil.hi(cn), Mt * Nt])

        def blocking():
            d.write(ba, a_h.data_ptr(), a_bytes)
            d.write(bb, b_h.data_ptr(), b_bytes)
            d.execute(k)
            d.read(bc, c_h.data_ptr(), c_bytes)

        for _ in range(3):
            blocking()
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            blocking()
        el_b = time.perf_counter() - t0
        dist.barrier()
    el_b = dist.max(el_b)
    return {"value": dist.world * flops * args.e2e_steps / el_p / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": a_bytes + b_bytes, "d2h_bytes_per_step": c_bytes,
            "steps": args.e2e_steps, "ms_per_step": el_p / args.e2e_steps * 1e3,
            "path": "ttfoil.matmul_tiles_host -> foil_matmul_tiles_host (pinned host A, B, C; "
                    "B first, then ~32 chunks of A / GEMM / C overlapped on 3 streams)",
            "timer": "host perf_counter around the blocking call",
            "runtime_api": {"value": dist.world * flops * args.e2e_steps / el_b / 1e12,
                            "ms_per_step": el_b / args.e2e_steps * 1e3,
                            "path": "ttfoil.Device write_buffer x2 (pinned) + execute(matmul_dram) + "
                                    "read_buffer"}}


def main():
    args = parse()
    dist = Dist(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, dist)
        else:
            run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
