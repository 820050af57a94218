"""ORACLE — test infrastructure only.

numpy binding of the CPU restatement of tt-foil's golden path
(oracle/golden.cpp -> oracle/liboracle.so) and, when it was built, of the
reference's own golden code (oracle/_ref/libref_golden.so).  Imported by
tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg only;
the product (tt-foil_b200) never uses it.

bf16 arrays are numpy uint16 bit patterns.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_golden.so")
DROPTESTS_DIR = os.path.join(HERE, "_ref", "droptests")

_U16 = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_F32 = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u32, _u64, _i = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            import subprocess
            import sys
            subprocess.check_call([sys.executable, os.path.join(HERE, "build.py"), "--reference", "/nonexistent"])
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        L.oracle_bf16_to_f32.restype = ctypes.c_float
        L.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f32_to_bf16_array.argtypes = [_F32, _U16, _u64]
        L.oracle_tilize.argtypes = [_U16, _U16, _u32, _u32]
        L.oracle_untilize.argtypes = [_U16, _U16, _u32, _u32]
        L.oracle_matmul.argtypes = [_U16, _U16, _U16, _u32, _u32, _u32, _u32, _u32, _i]
        L.oracle_matmul_tiles.argtypes = [_U16, _U16, _U16, _u32, _u32, _u32, _i]
        L.oracle_conv_chw.argtypes = [_U16, _U16, _U16] + [_u32] * 8
        L.oracle_im2col_chw.argtypes = [_U16, _U16] + [_u32] * 7
        L.oracle_conv_nhwc.argtypes = [_U16, _U16, ctypes.c_void_p, _U16] + [_u32] * 9 + [_i, _u32, _u32, _i]
        L.oracle_bias_add.argtypes = [_U16, _U16, _U16, _u32, _u32]
        L.oracle_relu.argtypes = [_U16, _U16, _u64]
        L.oracle_add.argtypes = [_U16, _U16, _U16, _u64]
        L.oracle_gen_matmul_inputs.argtypes = [_U16, _U16, _u32, _u32, _u32]
        L.oracle_gen_conv_inputs.argtypes = [_U16, _U16] + [_u32] * 6
        L.oracle_compare.restype = _u64
        L.oracle_compare.argtypes = [_U16, _U16, _u64, ctypes.c_float, ctypes.c_float,
                                     ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)]
        _lib = L
    return _lib


def _c(a):
    return np.ascontiguousarray(a)


# ---------------------------------------------------------------- numbers ---
def f32_to_bf16(x):
    x = _c(np.asarray(x, dtype=np.float32))
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_bf16_array(x.reshape(-1), out.reshape(-1), x.size)
    return out


def bf16_to_f32(b):
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def rand_bf16(shape, seed, lo=-1.0, hi=1.0):
    """Seeded U(lo, hi) rounded to bf16 with the golden's rounding."""
    rng = np.random.default_rng(seed)
    return f32_to_bf16(rng.uniform(lo, hi, size=shape).astype(np.float32))


def randn_bf16(shape, seed, std):
    rng = np.random.default_rng(seed)
    return f32_to_bf16((rng.standard_normal(size=shape) * std).astype(np.float32))


# ----------------------------------------------------------------- layout ---
def tilize(rm):
    rm = _c(rm.astype(np.uint16, copy=False))
    r, c = rm.shape
    out = np.empty(r * c, dtype=np.uint16)
    lib().oracle_tilize(rm.reshape(-1), out, r, c)
    return out


def untilize(tiles, rows, cols):
    out = np.empty((rows, cols), dtype=np.uint16)
    lib().oracle_untilize(_c(tiles.reshape(-1)), out.reshape(-1), rows, cols)
    return out


# ------------------------------------------------------------------- math ---
def matmul(a, b, rows=None, threads=1):
    """bf16 C = A.B with the golden's sequential fp32 accumulation.  `rows`
    (begin, end) limits the computed output rows (others stay 0)."""
    a = _c(a)
    b = _c(b)
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    c = np.zeros((M, N), dtype=np.uint16)
    rb, re = rows if rows is not None else (0, M)
    lib().oracle_matmul(a.reshape(-1), b.reshape(-1), c.reshape(-1), M, N, K, rb, re, threads)
    return c


def matmul_tiles(a_tiles, b_tiles, Mt, Kt, Nt, threads=1):
    c = np.empty(Mt * Nt * 1024, dtype=np.uint16)
    lib().oracle_matmul_tiles(_c(a_tiles.reshape(-1)), _c(b_tiles.reshape(-1)), c, Mt, Kt, Nt, threads)
    return c


def conv_chw(x, w, stride, pad):
    """x (Cin, H, W), w (Cout, Cin, kh, kw) -> y (Cout, Ho, Wo)."""
    Cin, H, W = x.shape
    Cout, Cin2, kh, kw = w.shape
    assert Cin == Cin2
    Ho, Wo = (H + 2 * pad - kh) // stride + 1, (W + 2 * pad - kw) // stride + 1
    y = np.empty((Cout, Ho, Wo), dtype=np.uint16)
    lib().oracle_conv_chw(_c(x).reshape(-1), _c(w).reshape(-1), y.reshape(-1), Cin, H, W, Cout,
                          kh, kw, stride, pad)
    return y


def im2col_chw(x, kh, kw, stride, pad):
    Cin, H, W = x.shape
    Ho, Wo = (H + 2 * pad - kh) // stride + 1, (W + 2 * pad - kw) // stride + 1
    a = np.empty((Cin * kh * kw, Ho * Wo), dtype=np.uint16)
    lib().oracle_im2col_chw(_c(x).reshape(-1), a.reshape(-1), Cin, H, W, kh, kw, stride, pad)
    return a


def conv_nhwc(x, w, bias, stride, pad, relu, images=None, threads=1):
    """x (N, H, W, Cin), w (Cout, kh, kw, Cin), bias (Cout,) or None."""
    N, H, W, Cin = x.shape
    Cout, kh, kw, Cin2 = w.shape
    assert Cin == Cin2
    Ho, Wo = (H + 2 * pad - kh) // stride + 1, (W + 2 * pad - kw) // stride + 1
    y = np.zeros((N, Ho, Wo, Cout), dtype=np.uint16)
    nb, ne = images if images is not None else (0, N)
    bptr = None
    if bias is not None:
        bias = _c(bias.astype(np.uint16))
        bptr = bias.ctypes.data
    lib().oracle_conv_nhwc(_c(x).reshape(-1), _c(w).reshape(-1), bptr, y.reshape(-1), N, H, W, Cin,
                           Cout, kh, kw, stride, pad, 1 if relu else 0, nb, ne, threads)
    return y


def bias_add(x, bias_row):
    x = _c(x)
    r, c = x.shape
    out = np.empty_like(x)
    lib().oracle_bias_add(x.reshape(-1), _c(bias_row.reshape(-1)), out.reshape(-1), r, c)
    return out


def relu(x):
    x = _c(x)
    out = np.empty_like(x)
    lib().oracle_relu(x.reshape(-1), out.reshape(-1), x.size)
    return out


def add(a, b):
    a, b = _c(a), _c(b)
    out = np.empty_like(a)
    lib().oracle_add(a.reshape(-1), b.reshape(-1), out.reshape(-1), a.size)
    return out


def gen_matmul_inputs(M, K, N):
    a = np.empty((M, K), dtype=np.uint16)
    b = np.empty((K, N), dtype=np.uint16)
    lib().oracle_gen_matmul_inputs(a.reshape(-1), b.reshape(-1), M, K, N)
    return a, b


def gen_conv_inputs(Cin, H, W, Cout, kh, kw):
    x = np.empty((Cin, H, W), dtype=np.uint16)
    w = np.empty((Cout, Cin, kh, kw), dtype=np.uint16)
    lib().oracle_gen_conv_inputs(x.reshape(-1), w.reshape(-1), Cin, H, W, Cout, kh, kw)
    return x, w


def compare(got, exp, abs_tol=0.05, rel_tol=0.01):
    """Reference comparator: returns (mismatches, worst_abs, worst_rel)."""
    got, exp = _c(got.reshape(-1)), _c(exp.reshape(-1))
    wa, wr = ctypes.c_float(), ctypes.c_float()
    bad = lib().oracle_compare(got, exp, got.size, abs_tol, rel_tol, ctypes.byref(wa), ctypes.byref(wr))
    return int(bad), wa.value, wr.value


def normalized_error(got, exp, K, amax, bmax):
    """max |got - exp| / (sqrt(K) * max|a| * max|b|) — the GEMM/conv parity
    metric (bound 1e-2)."""
    g = bf16_to_f32(got).astype(np.float64)
    e = bf16_to_f32(exp).astype(np.float64)
    return float(np.max(np.abs(g - e)) / (np.sqrt(K) * amax * bmax))


# ------------------------------------------------ reference-built goldens ---
_ref = None


def ref_lib():
    """The reference's golden code compiled by oracle/build.py, or None."""
    global _ref
    if _ref is None and os.path.exists(REF_LIB_PATH):
        _ref = ctypes.CDLL(REF_LIB_PATH)
    return _ref


def ref_matmul_8192(cols):
    """The reference's own golden matmul (tests/test_matmul_mnk.cpp:62-76)
    compiled for one block of an 8192 x 8192 x 8192 product: 32 output rows
    by `cols` = 8192 (a whole row block, Mt = 1, Kt = Nt = 256) or 32 (one
    output tile, Nt = 1) columns, K = 8192.  Returns f(a, b) -> c with a
    (32, 8192) and b (8192, cols) row-major bf16 bits, or None when
    oracle/_ref was not built.  The call releases the GIL (ctypes), so
    threads run blocks in parallel."""
    tag = {8192: "mnk_1_256_256", 32: "mnk_1_256_1"}[cols]
    L = ref_lib()
    if L is None or not hasattr(L, "ref_matmul_" + tag):
        return None
    fn = getattr(L, "ref_matmul_" + tag)
    fn.restype = None
    fn.argtypes = [_U16, _U16, _U16]

    def run(a, b):
        a, b = _c(a), _c(b)
        assert a.shape == (32, 8192) and b.shape == (8192, cols)
        c = np.empty((32, cols), dtype=np.uint16)
        fn(a, b, c)
        return c
    return run
