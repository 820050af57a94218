"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Runs the reference's golden functions — tests/tile_utils.hpp and the golden
loops of tests/test_matmul_mnk.cpp, test_conv_3x3.cpp, test_conv_3x3_s2.cpp,
test_conv_1x1.cpp, compiled from the reference tree into
oracle/_ref/libref_golden.so by oracle/build.py — on the reference tests'
closed-form inputs and on seeded U(-1,1) / N(0, s) inputs, and stores inputs
and outputs as .npz files.  The CPU tests pin the oracle to these files and
the GPU tests compare the CUDA kernels with them, on machines where the
reference tree is absent.

Usage (needs the reference tree and a built oracle/_ref):
    python oracle/build.py && python tests/golden/make_fixtures.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle  # noqa: E402

U16 = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
F32 = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


def ref():
    L = oracle.ref_lib()
    if L is None:
        raise SystemExit("oracle/_ref/libref_golden.so missing: run python oracle/build.py first")
    return L


def ref_f32_to_bf16(x):
    L = ref()
    L.ref_f32_to_bf16_array.argtypes = [F32, U16, ctypes.c_uint64]
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size, dtype=np.uint16)
    L.ref_f32_to_bf16_array(x, out, x.size)
    return out


def dims(tag, n):
    d = (ctypes.c_uint32 * n)()
    getattr(ref(), f"ref_dims_{tag}")(d)
    return list(d)


def call(name, *arrays):
    fn = getattr(ref(), name)
    fn.argtypes = [U16] * len(arrays)
    fn(*arrays)


def ref_bf16_rand(shape, seed, lo=-1.0, hi=1.0):
    rng = np.random.default_rng(seed)
    return ref_f32_to_bf16(rng.uniform(lo, hi, size=shape).astype(np.float32)).reshape(shape)


def ref_bf16_randn(shape, seed, std):
    rng = np.random.default_rng(seed)
    return ref_f32_to_bf16((rng.standard_normal(size=shape) * std).astype(np.float32)).reshape(shape)


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path}")


def tile_utils_fixture():
    specials = np.array([0.0, -0.0, 1.0, -1.0, 1.00390625, 1.01171875, 3.0e38, -3.0e38, 3.4e38,
                         1e-40, -1e-40, 1.5e-45, 65504.0, 0.1, 0.005, np.inf, -np.inf],
                        dtype=np.float32)
    # Exact halfway cases (round-to-even on both parities) and NaN payloads.
    halfway = np.array([0x3f808000, 0x3f818000, 0xbf808000, 0x7f7f8000, 0x7fc00001, 0xffc00000,
                        0x7fffffff, 0x7f800001], dtype=np.uint32).view(np.float32)
    rng = np.random.default_rng(101)
    rand = rng.standard_normal(4096).astype(np.float32) * np.float32(10.0) ** rng.integers(-30, 30, 4096)
    f = np.concatenate([specials, halfway, rand.astype(np.float32)])
    bf = ref_f32_to_bf16(f)
    block = ref_bf16_rand((32, 32), 102)
    tile = np.empty(1024, dtype=np.uint16)
    call("ref_row_major_to_tile", np.ascontiguousarray(block.reshape(-1)), tile)
    back = np.empty(1024, dtype=np.uint16)
    call("ref_tile_to_row_major", tile, back)
    assert np.array_equal(back, block.reshape(-1))
    save("tile_utils", f32=f.view(np.uint32), bf16=bf, block=block, tile=tile)


def matmul_fixture(tag, inputs):
    Mt, Kt, Nt = dims(tag, 3)
    M, K, N = Mt * 32, Kt * 32, Nt * 32
    if inputs == "formula":
        a, b = oracle.gen_matmul_inputs(M, K, N)  # checked against the test's formula below
    else:
        a, b = ref_bf16_rand((M, K), 200 + Mt), ref_bf16_rand((K, N), 300 + Nt)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    c = np.empty(M * N, dtype=np.uint16)
    call(f"ref_matmul_{tag}", a.reshape(-1), b.reshape(-1), c)
    at = np.empty(M * K, dtype=np.uint16)
    bt = np.empty(K * N, dtype=np.uint16)
    call(f"ref_tile_a_{tag}", a.reshape(-1), at)
    call(f"ref_tile_b_{tag}", b.reshape(-1), bt)
    # Output tiles: inverse of the reference's untile_C_stream.
    ct = oracle.tilize(c.reshape(M, N))
    back = np.empty(M * N, dtype=np.uint16)
    call(f"ref_untile_c_{tag}", ct, back)
    assert np.array_equal(back, c)
    tiles = dict(a_tiles=at, b_tiles=bt, c_tiles=ct) if inputs == "formula" else {}
    save(f"matmul_{tag}", dims=np.array([Mt, Kt, Nt]), a=a, b=b, c=c.reshape(M, N),
         inputs=np.array(inputs), **tiles)


def conv_fixture(tag, kind, inputs, stride, ksize):
    Cin, H, W, Cout = dims(tag, 4)
    pad = 1 if ksize == 3 else 0
    if inputs == "formula":
        x, w = oracle.gen_conv_inputs(Cin, H, W, Cout, ksize, ksize)
    else:
        x = ref_bf16_rand((Cin, H, W), 400 + Cin)
        w = ref_bf16_randn((Cout, Cin, ksize, ksize), 500 + Cout, np.sqrt(2.0 / (Cin * ksize * ksize)))
    x = np.ascontiguousarray(x)
    w = np.ascontiguousarray(w)
    Ho, Wo = (H + 2 * pad - ksize) // stride + 1, (W + 2 * pad - ksize) // stride + 1
    y = np.empty(Cout * Ho * Wo, dtype=np.uint16)
    call(f"ref_conv_{tag}", x.reshape(-1), w.reshape(-1), y)
    extra = {}
    if kind in (2, 3):
        a = np.empty(Cin * 9 * Ho * Wo, dtype=np.uint16)
        call(f"ref_im2col_{tag}", x.reshape(-1), a)
        extra["im2col"] = a.reshape(Cin * 9, Ho * Wo)
    save(f"conv_{tag}", dims=np.array([Cin, H, W, Cout, ksize, stride, pad]), x=x, w=w,
         y=y.reshape(Cout, Ho, Wo), inputs=np.array(inputs), **extra)


def formula_check():
    """The oracle's closed-form input generators equal the reference tests'
    formulas (restated here from tests/test_matmul_mnk.cpp:146-155)."""
    M, K, N = 64, 128, 64
    a, b = oracle.gen_matmul_inputs(M, K, N)
    r = np.arange(M)[:, None]
    k = np.arange(K)[None, :]
    a_ref = ref_f32_to_bf16(np.float32(0.005) * ((r + 1) + (k % 7)).astype(np.float32)).reshape(M, K)
    assert np.array_equal(a, a_ref)


def main():
    formula_check()
    tile_utils_fixture()
    matmul_fixture("mnk_2_4_2", "formula")
    matmul_fixture("mnk_8_8_8", "random")
    matmul_fixture("mnk_3_5_2", "random")
    conv_fixture("conv3_1_9_2", 2, "formula", 1, 3)
    conv_fixture("conv3_2_18_14", 2, "random", 1, 3)
    conv_fixture("conv3s2_1_9_2", 3, "formula", 2, 3)
    conv_fixture("conv3s2_4_18_8", 3, "random", 2, 3)
    conv_fixture("conv1_2_2_2", 4, "formula", 1, 1)
    conv_fixture("conv1_8_4_16", 4, "random", 1, 1)


if __name__ == "__main__":
    main()
