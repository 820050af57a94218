"""Pin the oracle (oracle/golden.cpp) to the reference's own golden code.

The fixtures in tests/golden/ were produced by the reference's functions
(tests/tile_utils.hpp, test_matmul_mnk.cpp, test_conv_*.cpp) compiled from
its sources (tests/golden/make_fixtures.py).  When oracle/_ref is built in
this checkout, the oracle is also compared with that code directly.
"""
import numpy as np
import pytest

from oracle import oracle

MATMUL_TAGS = ["mnk_2_4_2", "mnk_8_8_8", "mnk_3_5_2"]
CONV_TAGS = ["conv3_1_9_2", "conv3_2_18_14", "conv3s2_1_9_2", "conv3s2_4_18_8", "conv1_2_2_2",
             "conv1_8_4_16"]


def test_f32_to_bf16_matches_reference(golden):
    g = golden("tile_utils")
    f = g["f32"].view(np.float32)
    assert np.array_equal(oracle.f32_to_bf16(f), g["bf16"])
    # widening is exact
    assert np.array_equal(oracle.bf16_to_f32(g["bf16"]).view(np.uint32),
                          g["bf16"].astype(np.uint32) << 16)


def test_tile_permutation_matches_reference(golden):
    g = golden("tile_utils")
    assert np.array_equal(oracle.tilize(g["block"]), g["tile"])
    assert np.array_equal(oracle.untilize(g["tile"], 32, 32), g["block"])


@pytest.mark.parametrize("tag", MATMUL_TAGS)
def test_matmul_matches_reference(golden, tag):
    g = golden("matmul_" + tag)
    c = oracle.matmul(g["a"], g["b"])
    assert np.array_equal(c, g["c"]), "oracle matmul must be bit-identical to matmul_reference"
    if "a_tiles" in g:
        assert np.array_equal(oracle.tilize(g["a"]), g["a_tiles"])
        assert np.array_equal(oracle.tilize(g["b"]), g["b_tiles"])
        assert np.array_equal(oracle.untilize(g["c_tiles"], *g["c"].shape), g["c"])
        Mt, Kt, Nt = (int(v) for v in g["dims"])
        ct = oracle.matmul_tiles(g["a_tiles"], g["b_tiles"], Mt, Kt, Nt)
        assert np.array_equal(ct, g["c_tiles"])


def test_matmul_formula_inputs(golden):
    g = golden("matmul_mnk_2_4_2")
    M, K = g["a"].shape
    N = g["b"].shape[1]
    a, b = oracle.gen_matmul_inputs(M, K, N)
    assert np.array_equal(a, g["a"]) and np.array_equal(b, g["b"])


@pytest.mark.parametrize("tag", CONV_TAGS)
def test_conv_matches_reference(golden, tag):
    g = golden("conv_" + tag)
    Cin, H, W, Cout, k, stride, pad = (int(v) for v in g["dims"])
    y = oracle.conv_chw(g["x"], g["w"], stride, pad)
    assert np.array_equal(y, g["y"])
    if "im2col" in g:
        assert np.array_equal(oracle.im2col_chw(g["x"], k, k, stride, pad), g["im2col"])
    # The NHWC conv used for the implicit-GEMM path sums the same products in
    # the same order: bit-identical to the CHW golden after re-indexing.
    x_nhwc = np.ascontiguousarray(g["x"].transpose(1, 2, 0))[None]
    w_nhwc = np.ascontiguousarray(g["w"].transpose(0, 2, 3, 1))
    y_nhwc = oracle.conv_nhwc(x_nhwc, w_nhwc, None, stride, pad, relu=False)
    assert np.array_equal(y_nhwc[0].transpose(2, 0, 1), g["y"])


def test_conv_formula_inputs(golden):
    g = golden("conv_conv3_1_9_2")
    Cin, H, W, Cout, k, _, _ = (int(v) for v in g["dims"])
    x, w = oracle.gen_conv_inputs(Cin, H, W, Cout, k, k)
    assert np.array_equal(x, g["x"]) and np.array_equal(w, g["w"])


def test_conv_as_gemm_equals_direct(golden):
    """Reference strategy (tests/test_conv_3x3.cpp:214-222): Y = W . im2col(X)."""
    g = golden("conv_conv3_1_9_2")
    Cin, H, W, Cout, k, stride, pad = (int(v) for v in g["dims"])
    a = oracle.im2col_chw(g["x"], k, k, stride, pad)
    y = oracle.matmul(g["w"].reshape(Cout, -1), a)
    assert np.array_equal(y.reshape(g["y"].shape), g["y"])


def test_eltwise_semantics():
    # relu: negatives -> +0, -0.0 and NaN unchanged (test_relu.cpp:54-59)
    x = np.array([0x0000, 0x8000, 0x3f80, 0xbf80, 0x7fc0, 0xffc0, 0xff80, 0x7f80, 0x0001, 0x8001],
                 dtype=np.uint16)
    assert list(oracle.relu(x)) == [0x0000, 0x8000, 0x3f80, 0x0000, 0x7fc0, 0xffc0, 0x0000, 0x7f80,
                                    0x0001, 0x0000]
    a = oracle.rand_bf16((64, 64), 1)
    b = oracle.rand_bf16((64, 64), 2)
    s = oracle.add(a, b)
    ref = oracle.f32_to_bf16(oracle.bf16_to_f32(a) + oracle.bf16_to_f32(b))
    assert np.array_equal(s, ref)
    bias = oracle.rand_bf16((64,), 3)
    o = oracle.bias_add(a, bias)
    ref = oracle.f32_to_bf16(oracle.bf16_to_f32(a) + oracle.bf16_to_f32(bias)[None, :])
    assert np.array_equal(o, ref)


def test_add_nan_results_of_the_x86_golden():
    """NaN results of the golden's `f(a) + f(b)` as compiled for x86-64 (the
    device kernels reproduce exactly these): one NaN operand comes out
    quieted, of two the second wins, inf - inf is the default NaN.  Scalar
    and vectorised loops agree (1 and 8 elements)."""
    a = np.array([0x7f83, 0xff8a, 0x7f80, 0x7f80, 0x3f80, 0x7f83, 0x7fc0, 0xff80], dtype=np.uint16)
    b = np.array([0x7f9f, 0xffe1, 0xff80, 0x7f80, 0x7f85, 0x3f80, 0xffc1, 0x7f80], dtype=np.uint16)
    exp = [0x7fdf, 0xffe1, 0xffc0, 0x7f80, 0x7fc5, 0x7fc3, 0xffc1, 0xffc0]
    assert list(oracle.add(a, b)) == exp
    assert [int(oracle.add(a[i:i + 1], b[i:i + 1])[0]) for i in range(8)] == exp
    x = np.full((1, 32), 0x3f80, dtype=np.uint16)
    x[0, :2] = 0x7f83
    bias = np.full(32, 0x3f80, dtype=np.uint16)
    bias[0] = 0x7f9f
    assert list(oracle.bias_add(x, bias)[0, :2]) == [0x7fdf, 0x7fc3]


def test_conv_nhwc_epilogue_is_composition():
    x = oracle.rand_bf16((2, 6, 7, 16), 5)
    w = oracle.randn_bf16((8, 3, 3, 16), 6, 0.1)
    bias = oracle.rand_bf16((8,), 7, -0.1, 0.1)
    y0 = oracle.conv_nhwc(x, w, None, 1, 1, relu=False)
    y = oracle.conv_nhwc(x, w, bias, 1, 1, relu=True)
    comp = oracle.relu(oracle.bias_add(y0.reshape(-1, 8), bias)).reshape(y.shape)
    assert np.array_equal(y, comp)


def test_compare_matches_reference_rule():
    exp = oracle.f32_to_bf16(np.array([10.0, 1.0, 0.0], dtype=np.float32))
    got = oracle.f32_to_bf16(np.array([10.09, 1.04, 0.06], dtype=np.float32))
    bad, wa, wr = oracle.compare(got, exp)
    assert bad == 1  # 0.06 > max(0.05, 0) ; 0.09 <= 0.1 ; 0.04 <= 0.05


@pytest.mark.skipif(oracle.ref_lib() is None, reason="oracle/_ref not built in this checkout")
@pytest.mark.parametrize("tag", ["mnk_3_5_2"])
def test_matmul_against_reference_library(tag):
    import ctypes
    L = oracle.ref_lib()
    d = (ctypes.c_uint32 * 3)()
    getattr(L, "ref_dims_" + tag)(d)
    Mt, Kt, Nt = list(d)
    a = oracle.rand_bf16((Mt * 32, Kt * 32), 11)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), 12)
    c = np.empty(Mt * 32 * Nt * 32, dtype=np.uint16)
    fn = getattr(L, "ref_matmul_" + tag)
    U16 = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
    fn.argtypes = [U16, U16, U16]
    fn(np.ascontiguousarray(a.reshape(-1)), np.ascontiguousarray(b.reshape(-1)), c)
    assert np.array_equal(oracle.matmul(a, b).reshape(-1), c)


@pytest.mark.skipif(oracle.ref_lib() is None, reason="oracle/_ref not built in this checkout")
def test_reference_golden_8192_tile_matches_port():
    """The reference's golden compiled for one 32 x 32 output tile of the
    8192^3 workload (K = 8192; the CPU baseline's unit of work) agrees bit
    for bit with the oracle port."""
    f = oracle.ref_matmul_8192(32)
    assert f is not None
    a = oracle.rand_bf16((32, 8192), 13)
    b = oracle.rand_bf16((8192, 32), 14)
    assert np.array_equal(f(a, b), oracle.matmul(a, b))


def test_reference_golden_library_maps_no_product_library():
    """The reference-built golden library (the checker and the CPU baseline)
    resolves the device API of the test files it includes against a throwing
    stub, so loading it maps none of this repository's runtime libraries."""
    import os
    import subprocess
    if not os.path.exists(oracle.REF_LIB_PATH):
        pytest.skip("oracle/_ref not built")
    out = subprocess.run(["readelf", "-d", oracle.REF_LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    needed = [l for l in out.splitlines() if "(NEEDED)" in l]
    assert needed and not any("foil" in l for l in needed), needed
    assert "RPATH" not in out and "RUNPATH" not in out
