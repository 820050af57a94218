"""Python binding of the B200 tt-foil C-ABI (include/foil_c.h, lib/libfoil.so).

Two layers, matching the C header:

* ``Device`` / ``Kernel`` / ``Buffer`` mirror tt-foil's host API
  (open_device, allocate_buffer, write/read_buffer, load_kernel,
  set_runtime_args, register_cbs, execute, make_noc_*_addr); every failure
  raises :class:`FoilError` with the library's message, as the reference
  raises std::runtime_error.
* ``tilize`` / ``untilize`` / ``tile_copy`` / ``add_tiles`` / ``relu_tiles`` /
  ``bias_add_tiles`` / ``matmul_tiles`` run the CUDA kernels on tensors that
  already live on the GPU (torch CUDA tensors or raw device pointers), on the
  current torch stream.

There is no fallback: if lib/libfoil.so is missing or was built for another
GPU, importing or calling this module raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(_HERE)
LIB_DIR = os.path.join(ROOT, "lib")
PROGRAMS_DIR = os.path.join(ROOT, "programs")
LIB_PATH = os.path.join(LIB_DIR, "libfoil.so")

FOIL_OK = 0
STATUS_NAMES = {1: "INVALID", 2: "OOM", 3: "NOT_FOUND", 4: "CUDA", 5: "TIMEOUT",
                6: "UNSUPPORTED", 7: "DEVICE"}
LOC_L1, LOC_DRAM = 0, 1
BRISC, NCRISC, TRISC0, TRISC1, TRISC2 = range(5)


class FoilError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(message)
        self.status = status


class foil_core(ctypes.Structure):
    _fields_ = [("x", ctypes.c_uint32), ("y", ctypes.c_uint32)]


class foil_buffer(ctypes.Structure):
    _fields_ = [("location", ctypes.c_int32), ("reserved", ctypes.c_uint32),
                ("device_addr", ctypes.c_uint64), ("size_bytes", ctypes.c_uint64),
                ("core", foil_core)]


class foil_risc_binary(ctypes.Structure):
    _fields_ = [("risc", ctypes.c_int32), ("elf_path", ctypes.c_char_p)]


class foil_cb_config(ctypes.Structure):
    _fields_ = [("cb_index", ctypes.c_uint8), ("fifo_addr", ctypes.c_uint64),
                ("fifo_size", ctypes.c_uint32), ("num_pages", ctypes.c_uint32),
                ("page_size", ctypes.c_uint32)]


# Exported C-ABI symbols with their signatures (restype, argtypes).
_P = ctypes.c_void_p
_U16P = ctypes.c_void_p
SIGNATURES = {
    "foil_last_error": (ctypes.c_char_p, []),
    "foil_version": (ctypes.c_char_p, []),
    "foil_open_device": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(foil_core),
                                        ctypes.c_size_t, ctypes.POINTER(_P)]),
    "foil_close_device": (ctypes.c_int, [_P]),
    "foil_allocate_buffer": (ctypes.c_int, [_P, ctypes.c_int32, ctypes.c_uint64, foil_core,
                                            ctypes.POINTER(foil_buffer)]),
    "foil_free_buffer": (ctypes.c_int, [_P, ctypes.POINTER(foil_buffer)]),
    "foil_write_buffer": (ctypes.c_int, [_P, ctypes.POINTER(foil_buffer), _P, ctypes.c_uint64]),
    "foil_read_buffer": (ctypes.c_int, [_P, ctypes.POINTER(foil_buffer), _P, ctypes.c_uint64]),
    "foil_load_kernel": (ctypes.c_int, [_P, ctypes.POINTER(foil_risc_binary), ctypes.c_size_t,
                                        foil_core, ctypes.POINTER(_P)]),
    "foil_release_kernel": (ctypes.c_int, [_P]),
    "foil_set_runtime_args": (ctypes.c_int, [_P, _P, ctypes.c_int32,
                                             ctypes.POINTER(ctypes.c_uint32), ctypes.c_size_t]),
    "foil_register_cbs": (ctypes.c_int, [_P, _P, ctypes.POINTER(foil_cb_config), ctypes.c_size_t]),
    "foil_execute": (ctypes.c_int, [_P, ctypes.POINTER(_P), ctypes.c_size_t, ctypes.c_int32]),
    "foil_make_noc_unicast_addr": (ctypes.c_int, [_P, foil_core, ctypes.c_uint64,
                                                  ctypes.POINTER(ctypes.c_uint64)]),
    "foil_make_noc_dram_addr": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "foil_buffer_device_ptr": (ctypes.c_int, [_P, ctypes.POINTER(foil_buffer), ctypes.POINTER(_P)]),
    "foil_launch_count": (ctypes.c_uint64, []),
    "foil_tilize_dev": (ctypes.c_int, [_U16P, _U16P, ctypes.c_uint32, ctypes.c_uint32, _P]),
    "foil_untilize_dev": (ctypes.c_int, [_U16P, _U16P, ctypes.c_uint32, ctypes.c_uint32, _P]),
    "foil_tile_copy_dev": (ctypes.c_int, [_P, _P, ctypes.c_uint64, _P]),
    "foil_add_tiles_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, ctypes.c_uint64, _P]),
    "foil_relu_tiles_dev": (ctypes.c_int, [_U16P, _U16P, ctypes.c_uint64, _P]),
    "foil_bias_add_tiles_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, ctypes.c_uint32,
                                               ctypes.c_uint32, _P]),
    "foil_matmul_tiles_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, ctypes.c_uint32, ctypes.c_uint32,
                                             ctypes.c_uint32, _U16P, ctypes.c_int32, _P]),
    "foil_device_error_dev": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint32)]),
    "foil_conv2d_nhwc_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, _U16P] + [ctypes.c_uint32] * 9 +
                             [ctypes.c_int32, _P]),
    "foil_matmul_tiles_noalloc_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, ctypes.c_uint32,
                                                     ctypes.c_uint32, ctypes.c_uint32, _U16P,
                                                     ctypes.c_int32, _P,
                                                     ctypes.POINTER(ctypes.c_uint32)]),
    "foil_matmul_tiles_host": (ctypes.c_int, [ctypes.c_int32, _U16P, _U16P, _U16P, ctypes.c_uint32,
                                              ctypes.c_uint32, ctypes.c_uint32, _U16P, ctypes.c_int32,
                                              ctypes.c_uint32]),
    "foil_conv2d_nhwc_host": (ctypes.c_int, [ctypes.c_int32, _U16P, _U16P, _U16P, _U16P] +
                              [ctypes.c_uint32] * 9 + [ctypes.c_int32, ctypes.c_uint32]),
    "foil_host_pipeline_release": (ctypes.c_int, [ctypes.c_int32]),
    "foil_matmul_tiles_gather_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, ctypes.POINTER(_P), ctypes.c_uint32,
                                                    ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, _U16P,
                                                    ctypes.c_int32, _P]),
    "foil_matmul_tiles_gather_mc_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, _U16P, ctypes.c_uint32, ctypes.c_uint32,
                                                       ctypes.c_uint32, _U16P, ctypes.c_int32, _P]),
    "foil_matmul_tiles_gather_ce_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, ctypes.POINTER(_P), ctypes.c_uint32,
                                                       ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, _U16P,
                                                       ctypes.c_int32, ctypes.c_uint32, _P]),
    "foil_peer_alloc": (ctypes.c_int, [ctypes.c_int32, ctypes.c_uint64, ctypes.POINTER(_P),
                                       ctypes.POINTER(ctypes.c_uint8)]),
    "foil_peer_open": (ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(_P)]),
    "foil_peer_close": (ctypes.c_int, [ctypes.c_int32, _P]),
    "foil_peer_free": (ctypes.c_int, [ctypes.c_int32, _P]),
    "foil_set_wait_limit_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "foil_conv2d_chw_dev": (ctypes.c_int, [_U16P, _U16P, _U16P, _U16P] + [ctypes.c_uint32] * 9 +
                            [ctypes.c_int32, _P]),
}

# Bits of the device error word (include/foil_c.h FOIL_DEVERR_*).
DEVERR_WAIT_TIMEOUT, DEVERR_BAD_SHAPE, DEVERR_CONFIG = 1, 2, 4

_lib = None


def lib():
    """Load lib/libfoil.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FoilError(4, f"libfoil.so not built: {LIB_PATH} (run make -C tt-foil_b200)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc):
    if rc != FOIL_OK:
        msg = lib().foil_last_error().decode(errors="replace")
        raise FoilError(rc, msg)


def launch_count():
    return int(lib().foil_launch_count())


def set_wait_limit_ns(ns):
    """Wall-time limit of every bounded device-side wait for the launches
    that follow (0 = the default 2 s); returns the previous limit."""
    return int(lib().foil_set_wait_limit_ns(int(ns)))


# ------------------------------------------------------------ device layer ---

def _ptr(t):
    """Device pointer of a torch tensor or an int."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def tilize(row_major, tiles, rows, cols, stream=None):
    check(lib().foil_tilize_dev(_ptr(row_major), _ptr(tiles), rows, cols, _stream(stream)))


def untilize(tiles, row_major, rows, cols, stream=None):
    check(lib().foil_untilize_dev(_ptr(tiles), _ptr(row_major), rows, cols, _stream(stream)))


def tile_copy(src, dst, nbytes, stream=None):
    check(lib().foil_tile_copy_dev(_ptr(src), _ptr(dst), nbytes, _stream(stream)))


def add_tiles(a, b, out, n, stream=None):
    check(lib().foil_add_tiles_dev(_ptr(a), _ptr(b), _ptr(out), n, _stream(stream)))


def relu_tiles(x, out, n, stream=None):
    check(lib().foil_relu_tiles_dev(_ptr(x), _ptr(out), n, _stream(stream)))


def bias_add_tiles(x, bias_tiles, out, rows, cols, stream=None):
    check(lib().foil_bias_add_tiles_dev(_ptr(x), _ptr(bias_tiles), _ptr(out), rows, cols,
                                        _stream(stream)))


def matmul_tiles(a, b, c, Mt, Kt, Nt, bias=None, relu=False, stream=None):
    check(lib().foil_matmul_tiles_dev(_ptr(a), _ptr(b), _ptr(c), Mt, Kt, Nt, _ptr(bias),
                                      1 if relu else 0, _stream(stream)))


def matmul_tiles_gather(a, b, c, peer_c, Mt, Kt, Nt, bias=None, relu=False, stream=None):
    """matmul_tiles that also stores every output tile to the peer buffers
    `peer_c` (device addresses as ints, other GPUs' memory opened with
    peer_open, offset like c): C = A . B lands in c and in every peer copy."""
    arr = (_P * max(1, len(peer_c)))(*[int(x) for x in peer_c])
    check(lib().foil_matmul_tiles_gather_dev(_ptr(a), _ptr(b), _ptr(c), arr, len(peer_c), Mt, Kt, Nt,
                                             _ptr(bias), 1 if relu else 0, _stream(stream)))


def matmul_tiles_gather_mc(a, b, c, mc_c, Mt, Kt, Nt, bias=None, relu=False, stream=None):
    """matmul_tiles whose output tiles are stored through the NVLink
    multicast address `mc_c` (an int: c's offset in a multicast object bound
    on every GPU), so C lands in every GPU's copy."""
    check(lib().foil_matmul_tiles_gather_mc_dev(_ptr(a), _ptr(b), _ptr(c), _P(int(mc_c)), Mt, Kt, Nt, _ptr(bias),
                                                1 if relu else 0, _stream(stream)))


def matmul_tiles_gather_ce(a, b, c, peer_c, Mt, Kt, Nt, bias=None, relu=False, chunks=8, stream=None):
    """matmul_tiles_gather with the transfer on the copy engines: the GEMM
    runs in `chunks` row chunks and each finished chunk is copied to every
    peer buffer while the next one computes; `stream` continues after the
    last copy."""
    arr = (_P * max(1, len(peer_c)))(*[int(x) for x in peer_c])
    check(lib().foil_matmul_tiles_gather_ce_dev(_ptr(a), _ptr(b), _ptr(c), arr, len(peer_c), Mt, Kt, Nt,
                                                _ptr(bias), 1 if relu else 0, int(chunks), _stream(stream)))


PEER_HANDLE_BYTES = 64


def peer_alloc(device, nbytes):
    """Device buffer on CUDA device `device` shareable with the node's other
    processes: returns (device address, 64-byte export handle)."""
    ptr = _P()
    h = (ctypes.c_uint8 * PEER_HANDLE_BYTES)()
    check(lib().foil_peer_alloc(device, nbytes, ctypes.byref(ptr), h))
    return int(ptr.value), bytes(h)


def peer_open(device, handle):
    """Open another process's peer_alloc buffer on CUDA device `device`;
    returns its device address there."""
    if len(handle) != PEER_HANDLE_BYTES:
        raise FoilError(1, "peer_open: handle must be 64 bytes")
    ptr = _P()
    h = (ctypes.c_uint8 * PEER_HANDLE_BYTES).from_buffer_copy(handle)
    check(lib().foil_peer_open(device, h, ctypes.byref(ptr)))
    return int(ptr.value)


def peer_close(device, ptr):
    check(lib().foil_peer_close(device, ptr))


def peer_free(device, ptr):
    check(lib().foil_peer_free(device, ptr))


def conv2d_nhwc(x, w, bias, y, N, H, W, Cin, Cout, KH, KW, stride, pad, relu=False, stream=None):
    """y (N,Ho,Wo,Cout) = relu?(conv(x (N,H,W,Cin), w (Cout,KH,KW,Cin)) + bias)."""
    check(lib().foil_conv2d_nhwc_dev(_ptr(x), _ptr(w), _ptr(bias), _ptr(y), N, H, W, Cin, Cout, KH,
                                     KW, stride, pad, 1 if relu else 0, _stream(stream)))


def conv2d_chw(x, w, bias, y, N, Cin, H, W, Cout, KH, KW, stride, pad, relu=False, stream=None):
    """The reference's convention: y (N,Cout,Ho,Wo) = relu?(conv(x (N,Cin,H,W),
    w (Cout, Cin*KH*KW)) + bias), operands re-laid on the device."""
    check(lib().foil_conv2d_chw_dev(_ptr(x), _ptr(w), _ptr(bias), _ptr(y), N, Cin, H, W, Cout, KH, KW, stride,
                                    pad, 1 if relu else 0, _stream(stream)))


def matmul_tiles_host(device, a, b, c, Mt, Kt, Nt, bias=None, relu=False, chunk_rows=0):
    """Pipelined C = A . B (+bias, relu) on host tile streams (pinned CPU
    tensors, numpy arrays or host addresses): copies, GEMM chunks and
    read-back overlap; returns when C is in host memory."""
    check(lib().foil_matmul_tiles_host(device, _hptr(a), _hptr(b), _hptr(c), Mt, Kt, Nt, _hptr(bias),
                                       1 if relu else 0, chunk_rows))


def conv2d_nhwc_host(device, x, w, bias, y, N, H, W, Cin, Cout, KH, KW, stride, pad, relu=False,
                     chunk_images=0):
    """Pipelined NHWC convolution on host buffers (see matmul_tiles_host)."""
    check(lib().foil_conv2d_nhwc_host(device, _hptr(x), _hptr(w), _hptr(bias), _hptr(y), N, H, W, Cin,
                                      Cout, KH, KW, stride, pad, 1 if relu else 0, chunk_images))


def host_pipeline_release(device):
    check(lib().foil_host_pipeline_release(device))


def _hptr(t):
    """Host address of a CPU torch tensor, a numpy array or an int (None -> NULL)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    assert not t.is_cuda, "host pipeline entry points take host memory"
    return t.data_ptr()


def device_error(stream=None):
    """Read and clear the device-side error word (synchronizes the stream)."""
    v = ctypes.c_uint32(0)
    check(lib().foil_device_error_dev(_stream(stream), ctypes.byref(v)))
    return v.value


# ----------------------------------------------------------- runtime layer ---

class Buffer:
    def __init__(self, c):
        self.c = c

    @property
    def device_addr(self):
        return int(self.c.device_addr)

    @property
    def size_bytes(self):
        return int(self.c.size_bytes)


class Kernel:
    def __init__(self, device, handle):
        self.device = device
        self.handle = handle

    def __del__(self):
        if self.handle and _lib is not None:
            _lib.foil_release_kernel(self.handle)
            self.handle = None


class Device:
    """tt-foil device (open_device ... close_device) over the C-ABI."""

    def __init__(self, index=0, cores=((0, 0),), firmware_dir=""):
        arr = (foil_core * len(cores))(*[foil_core(x, y) for x, y in cores])
        h = ctypes.c_void_p()
        check(lib().foil_open_device(index, firmware_dir.encode(), arr, len(cores), ctypes.byref(h)))
        self.handle = h

    def close(self):
        if self.handle:
            h, self.handle = self.handle, None
            check(lib().foil_close_device(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def allocate(self, loc, size, core=(0, 0)):
        b = foil_buffer()
        check(lib().foil_allocate_buffer(self.handle, loc, size, foil_core(*core), ctypes.byref(b)))
        return Buffer(b)

    def write(self, buf, src_ptr, nbytes):
        check(lib().foil_write_buffer(self.handle, ctypes.byref(buf.c), src_ptr, nbytes))

    def read(self, buf, dst_ptr, nbytes):
        check(lib().foil_read_buffer(self.handle, ctypes.byref(buf.c), dst_ptr, nbytes))

    def write_array(self, buf, arr):
        import numpy as np
        a = np.ascontiguousarray(arr)
        self.write(buf, a.ctypes.data, a.nbytes)

    def read_array(self, buf, dtype, count):
        import numpy as np
        a = np.empty(count, dtype=dtype)
        self.read(buf, a.ctypes.data, a.nbytes)
        return a

    def device_ptr(self, buf):
        p = ctypes.c_void_p()
        check(lib().foil_buffer_device_ptr(self.handle, ctypes.byref(buf.c), ctypes.byref(p)))
        return int(p.value)

    def load_kernel(self, binaries, core=(0, 0)):
        keep = [(r, p.encode()) for r, p in binaries]
        arr = (foil_risc_binary * len(keep))(*[foil_risc_binary(r, p) for r, p in keep])
        h = ctypes.c_void_p()
        check(lib().foil_load_kernel(self.handle, arr, len(keep), foil_core(*core), ctypes.byref(h)))
        return Kernel(self, h)

    def load_program(self, program, core=(0, 0), reader="reader.brisc.elf"):
        """Load the standard five descriptors of programs/<program>/."""
        d = os.path.join(PROGRAMS_DIR, program)
        bins = [(BRISC, os.path.join(d, reader)), (NCRISC, os.path.join(d, "writer.ncrisc.elf")),
                (TRISC0, os.path.join(d, "compute.trisc0.elf")),
                (TRISC1, os.path.join(d, "compute.trisc1.elf")),
                (TRISC2, os.path.join(d, "compute.trisc2.elf"))]
        return self.load_kernel(bins, core)

    def set_runtime_args(self, kernel, risc, args):
        arr = (ctypes.c_uint32 * len(args))(*[int(a) & 0xffffffff for a in args])
        check(lib().foil_set_runtime_args(self.handle, kernel.handle, risc, arr, len(args)))

    def register_cbs(self, kernel, cbs):
        arr = (foil_cb_config * len(cbs))(*[foil_cb_config(*c) for c in cbs])
        check(lib().foil_register_cbs(self.handle, kernel.handle, arr, len(cbs)))

    def execute(self, kernels, timeout_ms=5000):
        if not isinstance(kernels, (list, tuple)):
            kernels = [kernels]
        arr = (ctypes.c_void_p * len(kernels))(*[k.handle for k in kernels])
        check(lib().foil_execute(self.handle, arr, len(kernels), timeout_ms))

    def noc_unicast_addr(self, core, l1_addr):
        out = ctypes.c_uint64()
        check(lib().foil_make_noc_unicast_addr(self.handle, foil_core(*core), l1_addr, ctypes.byref(out)))
        return int(out.value)

    def noc_dram_addr(self, offset):
        out = ctypes.c_uint64()
        check(lib().foil_make_noc_dram_addr(self.handle, offset, ctypes.byref(out)))
        return int(out.value)


def lo(v):
    return v & 0xffffffff


def hi(v):
    return (v >> 32) & 0xffffffff
