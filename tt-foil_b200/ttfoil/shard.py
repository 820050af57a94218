"""Multi-GPU partitioning of the tiled GEMM / batched conv (one process per GPU).

The reference shards a matmul across Tensix cores by output rows
(tests/test_matmul_2core.cpp:43-63: core c owns A rows and C rows
[c*Mt_pc, (c+1)*Mt_pc)), every core reading the whole B.  Across B200s the
same split is done in tile rows: a tile row of a tile-layout matrix is one
contiguous run of Nt*2 KiB, so each rank's C shard is a contiguous slice and
concatenating the shards in rank order (an all-gather) rebuilds the global
tile-layout C exactly.  Convolutions shard the batch: NHWC images are
contiguous, so no halo is exchanged.  A convolution of few large images can
instead shard the image rows (conv2d_nhwc_h_sharded), as the reference splits
one image's rows over two cores with a one-row halo each
(tests/test_conv_3x3_2core.cpp:6-16, 114-133): neighbouring ranks exchange
their border rows with point-to-point sends (NCCL between GPUs) into local
memory before the local convolution.
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


def _device_conv(ext, w, bias, N, H, W, Cin, Cout, K, pad, relu):
    """Implicit-GEMM conv of the extended shard on its CUDA device."""
    import torch
    from . import conv2d_nhwc
    y = torch.empty(N * H * W * Cout, dtype=ext.dtype, device=ext.device)
    conv2d_nhwc(ext, w, bias, y, N, H, W, Cin, Cout, K, K, 1, pad, relu=relu)
    return y.view(N, H, W, Cout)


def conv2d_nhwc_h_sharded(x, w, bias, N, H_local, W, Cin, Cout, K, pad, relu=False, conv=None):
    """Stride-1 'same' convolution (K = 2 pad + 1) of N images whose rows are
    split over the ranks of the default process group in rank order: `x`
    holds this rank's H_local rows of every image, (N, H_local, W, Cin) bf16
    bits (int16 or bfloat16 tensor).  Returns this rank's output rows,
    (N, H_local, W, Cout).

    The rank sends its first `pad` rows to rank - 1 and its last `pad` rows to
    rank + 1 and receives theirs (torch.distributed batched point-to-point:
    NCCL over NVLink between GPUs, gloo on CPU), places them above and below
    its own rows, and runs the convolution on those H_local + 2 pad rows with
    the ordinary zero padding; of the H_local + 2 pad output rows, rows
    pad .. pad + H_local - 1 are exactly the global output rows of this shard
    (the first and last rank receive nothing: their outer halo stays zero, the
    image's own padding).  Halos move as 32-bit words (gloo has no 16-bit
    point-to-point types).  `conv(ext, w, bias, N, H, W, Cin, Cout, K, pad,
    relu)` defaults to the implicit-GEMM kernel on the tensors' CUDA device."""
    import torch
    import torch.distributed as dist
    if K != 2 * pad + 1:
        raise ValueError("conv2d_nhwc_h_sharded: only stride-1 'same' convolutions (K = 2 pad + 1)")
    rank, world = dist.get_rank(), dist.get_world_size()
    if world > 1 and H_local < pad:
        raise ValueError("conv2d_nhwc_h_sharded: every shard needs at least `pad` rows")
    xv = x.view(N, H_local, W, Cin)
    p = pad
    ext = torch.zeros((N, H_local + 2 * p, W, Cin), dtype=x.dtype, device=x.device)
    ext[:, p:p + H_local] = xv
    if p and world > 1:
        top_send, bot_send = xv[:, :p].contiguous(), xv[:, H_local - p:].contiguous()
        top_recv, bot_recv = torch.empty_like(top_send), torch.empty_like(bot_send)
        w32 = lambda t: t.view(torch.int32)
        ops = []
        if rank > 0:
            ops += [dist.P2POp(dist.isend, w32(top_send), rank - 1),
                    dist.P2POp(dist.irecv, w32(top_recv), rank - 1)]
        if rank < world - 1:
            ops += [dist.P2POp(dist.isend, w32(bot_send), rank + 1),
                    dist.P2POp(dist.irecv, w32(bot_recv), rank + 1)]
        for req in dist.batch_isend_irecv(ops):
            req.wait()
        if rank > 0:
            ext[:, :p] = top_recv
        if rank < world - 1:
            ext[:, p + H_local:] = bot_recv
    y_ext = (conv or _device_conv)(ext, w, bias, N, H_local + 2 * p, W, Cin, Cout, K, p, relu)
    return y_ext[:, p:p + H_local].contiguous()


class _DeviceArray:
    """Minimal __cuda_array_interface__ exporter (int16 elements) so that a
    raw device address can be viewed as a torch tensor."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i2", "data": (ptr, False),
                                         "version": 3, "strides": None}


class GatheredTiles:
    """A tile-layout matrix of Mt x Nt tiles held in full on every rank of the
    default process group (one process per GPU of a node).

    Rank r owns the tile rows split_rows(Mt, world, r) (the reference's
    per-core row split, tests/test_matmul_2core.cpp:43-63).  `matmul` runs
    this rank's rows as ONE kernel launch whose epilogue stores every output
    tile both into this GPU's copy and, over NVLink, into every other rank's
    copy (foil_matmul_tiles_gather_dev), so the GEMM is its own all-gather:
    no separate collective moves C.  `fence` (a one-element all-reduce on the
    launch stream) orders every rank's launch before later reads; after it,
    `tensor()` is the whole C on every rank.

    Ordering rules.  Rank A's matmul writes into rank B's copy over NVLink,
    so two orderings are needed: (1) fence after a matmul before any rank
    reads C; (2) fence after the last read of a result and before the next
    matmul that overwrites it (otherwise rank A's next launch may store into
    B's copy while B still reads the previous C).  A loop of matmul, fence,
    matmul, fence with no reads in between needs nothing more.  Pass fence
    the stream the matmul was issued on (and the one the reads run on)
    when that is not torch's current stream.

    The copies are plain device buffers shared through CUDA IPC handles
    (foil_peer_alloc / foil_peer_open), exchanged once here."""

    def __init__(self, Mt, Nt, device=None):
        import torch
        import torch.distributed as dist
        from . import peer_alloc, peer_open
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.Mt, self.Nt = Mt, Nt
        self.nbytes = Mt * Nt * 2048
        self.rows = split_rows(Mt, self.world, self.rank)
        # Every step is collective and a failure anywhere fails every rank at
        # the same point (no rank is left waiting in a collective).
        from . import FoilError, peer_close, peer_free
        self.ptr, handle, why = None, None, ""
        try:
            self.ptr, handle = peer_alloc(self.device, self.nbytes)
        except FoilError as e:
            why = f"rank {self.rank}: {e}"
        handles = [None] * self.world
        dist.all_gather_object(handles, (handle, why))
        errors = [w for _, w in handles if w]
        self.bases = []
        if not errors:
            for r, (h, _) in enumerate(handles):
                try:
                    self.bases.append(self.ptr if r == self.rank else peer_open(self.device, h))
                except FoilError as e:
                    why = f"rank {self.rank} opening rank {r}'s buffer: {e}"
                    break
            states = [None] * self.world
            dist.all_gather_object(states, why)
            errors = [w for w in states if w]
        if errors:
            for r, p in enumerate(self.bases):
                if r != self.rank:
                    peer_close(self.device, p)
            dist.barrier()
            if self.ptr is not None:
                peer_free(self.device, self.ptr)
            raise RuntimeError("GatheredTiles: " + "; ".join(errors))
        self._one = None
        self._closed = False

    def tensor(self):
        """This rank's copy of C as an int16 CUDA tensor (bf16 bits, tile layout)."""
        import torch
        return torch.as_tensor(_DeviceArray(self.ptr, self.nbytes // 2), device=torch.device("cuda", self.device))

    def matmul(self, a, b, Kt, bias=None, relu=False, stream=None, method="fused", chunks=8):
        """C[rows of this rank] = A_r . B: `a` holds this rank's tile rows of A
        (tile layout, rows[1] - rows[0] tile rows x Kt), `b` all of B.
        method "fused": one kernel whose pusher warps store every tile to the
        peers; "ce": the GEMM in `chunks` row chunks, each chunk copied to
        the peers by the copy engines while the next one computes."""
        from . import matmul_tiles_gather, matmul_tiles_gather_ce
        m0, m1 = self.rows
        off = m0 * self.Nt * 2048
        peers = [self.bases[r] + off for r in range(self.world) if r != self.rank]
        if method == "ce":
            matmul_tiles_gather_ce(a, b, self.ptr + off, peers, m1 - m0, Kt, self.Nt, bias=bias, relu=relu,
                                   chunks=chunks, stream=stream)
        elif method == "fused":
            matmul_tiles_gather(a, b, self.ptr + off, peers, m1 - m0, Kt, self.Nt, bias=bias, relu=relu,
                                stream=stream)
        else:
            raise ValueError(f"GatheredTiles.matmul: unknown method {method!r}")

    def fence(self, stream=None):
        """Stream-ordered completion of every rank's work issued so far on
        `stream` (torch's current stream when None): a one-element
        all-reduce that work on `stream` after it waits for, on every rank.
        Needed after a matmul before C is read, and after the last read of
        C before the next matmul (see the class docstring)."""
        import torch
        import torch.distributed as dist
        if self._one is None:
            self._one = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", self.device))
        s = torch.cuda.current_stream(self.device) if stream is None else stream
        with torch.cuda.stream(s):
            dist.all_reduce(self._one)

    def close(self):
        """Unmap the peers' copies and free this rank's (collective)."""
        if self._closed:
            return
        import torch
        import torch.distributed as dist
        from . import peer_close, peer_free
        torch.cuda.synchronize(self.device)
        dist.barrier()
        for r, p in enumerate(self.bases):
            if r != self.rank:
                peer_close(self.device, p)
        torch.cuda.synchronize(self.device)
        dist.barrier()
        peer_free(self.device, self.ptr)
        self._closed = True


class MulticastTiles:
    """GatheredTiles over an NVLink multicast object: every rank's copy of
    the Mt x Nt tile-layout C lives in PyTorch symmetric memory, bound to one
    multicast object (NVSwitch), and `matmul` stores each output tile once
    through the multicast address; the switch writes it into every GPU's
    copy (foil_matmul_tiles_gather_mc_dev).  Same row split, same ordering
    rules and the same `fence` as GatheredTiles.  Raises RuntimeError on
    every rank alike when a rank has no multicast support."""

    def __init__(self, Mt, Nt, device=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.Mt, self.Nt = Mt, Nt
        self.nbytes = Mt * Nt * 2048
        self.rows = split_rows(Mt, self.world, self.rank)
        why = ""
        self.buf, self.handle = None, None
        try:
            if not symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, self.device):
                why = f"rank {self.rank}: no NVLink multicast support on device {self.device}"
        except Exception as e:  # noqa: BLE001 - reported on every rank below
            why = f"rank {self.rank}: {e}"
        states = [None] * self.world
        dist.all_gather_object(states, why)
        errors = [w for w in states if w]
        if not errors:
            try:
                self.buf = symm.empty(Mt * Nt * 1024, dtype=torch.int16,
                                      device=torch.device("cuda", self.device))
                self.handle = symm.rendezvous(self.buf, dist.group.WORLD)
                mc = int(self.handle.multicast_ptr)
                if mc == 0:
                    why = f"rank {self.rank}: the symmetric buffer has no multicast address"
                else:
                    # the multicast mapping mirrors this rank's buffer base
                    base = int(self.handle.buffer_ptrs[self.rank])
                    self.mc = mc + (self.buf.data_ptr() - base)
            except Exception as e:  # noqa: BLE001
                why = f"rank {self.rank}: {e}"
            states = [None] * self.world
            dist.all_gather_object(states, why)
            errors = [w for w in states if w]
        if errors:
            self.handle, self.buf = None, None
            raise RuntimeError("MulticastTiles: " + "; ".join(errors))
        self.ptr = self.buf.data_ptr()
        self._one = None
        self._closed = False

    def tensor(self):
        """This rank's copy of C as an int16 CUDA tensor (bf16 bits, tile layout)."""
        return self.buf

    def matmul(self, a, b, Kt, bias=None, relu=False, stream=None):
        """C[rows of this rank] = A_r . B, stored through the multicast
        address into every rank's copy (see GatheredTiles.matmul)."""
        from . import matmul_tiles_gather_mc
        m0, m1 = self.rows
        off = m0 * self.Nt * 2048
        matmul_tiles_gather_mc(a, b, self.ptr + off, self.mc + off, m1 - m0, Kt, self.Nt, bias=bias, relu=relu,
                               stream=stream)

    fence = GatheredTiles.fence

    def close(self):
        """Release the symmetric buffer (collective)."""
        if self._closed:
            return
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier()
        self.handle, self.buf = None, None
        self._closed = True
