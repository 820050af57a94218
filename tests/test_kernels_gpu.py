"""Parity of the sm_100a kernels (device-resident C-ABI entry points) with the
oracle: bit-exact for tilize / untilize / tile_copy / relu / add / bias_add,
and for the GEMM within the normalised-error bound 1e-2 (error divided by
sqrt(K) * max|a| * max|b|) plus the reference tests' max(0.05, 1%) rule.
"""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

GEMM_NORM_TOL = 1e-2


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch


@pytest.fixture(scope="module")
def tf():
    import ttfoil
    ttfoil.lib()
    return ttfoil


def dev(torch, arr):
    """numpy uint16 -> CUDA int16 tensor with the same bits."""
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).cuda()


def host(t):
    return t.cpu().numpy().view(np.uint16)


def empty(torch, n):
    return torch.empty(n, dtype=torch.int16, device="cuda")


@pytest.mark.parametrize("rows,cols", [(32, 32), (64, 96), (96, 256), (128, 288), (320, 544)])
def test_tilize_untilize_bit_exact(torch_cuda, tf, rows, cols):
    torch = torch_cuda
    rm = oracle.rand_bf16((rows, cols), rows * 1000 + cols)
    t = empty(torch, rows * cols)
    tf.tilize(dev(torch, rm), t, rows, cols)
    assert np.array_equal(host(t), oracle.tilize(rm))
    back = empty(torch, rows * cols)
    tf.untilize(t, back, rows, cols)
    torch.cuda.synchronize()
    assert np.array_equal(host(back).reshape(rows, cols), rm)


def test_tilize_large_round_trip(torch_cuda, tf):
    """4096 x 8192: tilize -> untilize is the identity; tilized sample tiles
    match the oracle."""
    torch = torch_cuda
    rows, cols = 4096, 8192
    g = torch.Generator(device="cuda").manual_seed(7)
    rm = torch.randint(-32768, 32767, (rows * cols,), dtype=torch.int16, device="cuda", generator=g)
    t = empty(torch, rows * cols)
    back = empty(torch, rows * cols)
    tf.tilize(rm, t, rows, cols)
    tf.untilize(t, back, rows, cols)
    torch.cuda.synchronize()
    assert torch.equal(rm, back)
    rm_h = host(rm).reshape(rows, cols)
    t_h = host(t)
    Ct = cols // 32
    for (rt, ct) in [(0, 0), (5, 17), (127, 255), (64, 3)]:
        tile = t_h[(rt * Ct + ct) * 1024:(rt * Ct + ct + 1) * 1024]
        assert np.array_equal(tile, oracle.tilize(rm_h[rt * 32:(rt + 1) * 32, ct * 32:(ct + 1) * 32]))


@pytest.mark.parametrize("nbytes", [2048, 32 * 1024, 3 * 2048 + 16, 64 << 20])
def test_tile_copy_bitwise(torch_cuda, tf, nbytes):
    torch = torch_cuda
    src = torch.arange(nbytes // 2, dtype=torch.int32, device="cuda").to(torch.int16) ^ 0x5A5A
    dst = torch.zeros_like(src)
    tf.tile_copy(src, dst, nbytes)
    torch.cuda.synchronize()
    assert torch.equal(src, dst)


def special_bf16():
    vals = [0x0000, 0x8000, 0x3f80, 0xbf80, 0x7fc0, 0xffc0, 0xff80, 0x7f80, 0x0001, 0x8001, 0x7f7f,
            0xff7f, 0x0080, 0x8080]
    return np.array(vals, dtype=np.uint16)


def test_relu_bit_exact(torch_cuda, tf):
    torch = torch_cuda
    x = np.concatenate([oracle.rand_bf16(1 << 16, 3, -100, 100), np.tile(special_bf16(), 8)])
    x = x[: (x.size // 8) * 8]
    out = empty(torch, x.size)
    tf.relu_tiles(dev(torch, x), out, x.size)
    torch.cuda.synchronize()
    assert np.array_equal(host(out), oracle.relu(x))


def test_add_bit_exact(torch_cuda, tf):
    torch = torch_cuda
    n = (1 << 18) + 8 * 37
    a = oracle.rand_bf16(n, 4)
    b = oracle.rand_bf16(n, 5)
    b[:14] = special_bf16()
    out = empty(torch, n)
    tf.add_tiles(dev(torch, a), dev(torch, b), out, n)
    torch.cuda.synchronize()
    assert np.array_equal(host(out), oracle.add(a, b))


def test_add_every_bf16_and_rounding_edges(torch_cuda, tf):
    """Every bf16 bit pattern as the first operand (NaNs, infinities,
    subnormals, signed zeros) against random second operands, plus pairs
    whose exponents differ by 0..26 (where the golden's fp32 sum stops being
    exact), both signs: bit-exact to the golden."""
    torch = torch_cuda
    rng = np.random.default_rng(11)
    every = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    a1 = np.tile(every, 16)
    b1 = rng.integers(0, 1 << 16, a1.size, dtype=np.uint32).astype(np.uint16)
    base = rng.integers(0, 1 << 16, 8192, dtype=np.uint32)
    base = base[((base >> 7) & 0xff) > 30]                     # exponent room below
    d = np.arange(27, dtype=np.uint32)
    ea = (base[:, None] >> 7) & 0xff
    eb = np.maximum(ea.astype(np.int64) - d[None, :], 0).astype(np.uint32)
    mant = rng.integers(0, 128, eb.shape, dtype=np.uint32)
    sign = rng.integers(0, 2, eb.shape, dtype=np.uint32) << 15
    a2 = np.broadcast_to(base[:, None], eb.shape).ravel().astype(np.uint16)
    b2 = (sign | (eb << 7) | mant).ravel().astype(np.uint16)
    a = np.concatenate([a1, a2, b2])
    b = np.concatenate([b1, b2, a2])
    n = (a.size // 8) * 8
    a, b = a[:n], b[:n]
    out = empty(torch, n)
    tf.add_tiles(dev(torch, a), dev(torch, b), out, n)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    got, exp = host(out), oracle.add(a, b)
    bad = np.nonzero(got != exp)[0]
    assert bad.size == 0, f"{bad.size} mismatches; (a, b, got, golden): " + ", ".join(
        f"({a[i]:04x}, {b[i]:04x}, {got[i]:04x}, {exp[i]:04x})" for i in bad[:24])


@pytest.mark.parametrize("n", [8, 24, 1024 + 8, 4096 * 3 + 40, (1 << 20) + 8 * 1001])
def test_eltwise_ragged_sizes(torch_cuda, tf, n):
    """Sizes that leave a partial last chunk in the streaming pipeline (and
    fewer chunks than CTAs): relu, add and copy stay bit-exact and write
    nothing past n."""
    torch = torch_cuda
    a = oracle.rand_bf16(n, 21, -4, 4)
    b = oracle.rand_bf16(n, 22, -4, 4)
    guard = 64
    out = torch.full((n + guard,), 0x1234, dtype=torch.int16, device="cuda")
    tf.relu_tiles(dev(torch, a), out, n)
    torch.cuda.synchronize()
    h = host(out)
    assert np.array_equal(h[:n], oracle.relu(a)) and np.all(h[n:] == 0x1234)
    tf.add_tiles(dev(torch, a), dev(torch, b), out, n)
    torch.cuda.synchronize()
    h = host(out)
    assert np.array_equal(h[:n], oracle.add(a, b)) and np.all(h[n:] == 0x1234)
    tf.tile_copy(dev(torch, b), out, 2 * n)
    torch.cuda.synchronize()
    h = host(out)
    assert np.array_equal(h[:n], b) and np.all(h[n:] == 0x1234)
    assert tf.device_error() == 0


def test_eltwise_in_place(torch_cuda, tf):
    """out == input: relu and add in place, bias_add in place."""
    torch = torch_cuda
    n = (3 << 20) + 8 * 5
    a = oracle.rand_bf16(n, 31)
    b = oracle.rand_bf16(n, 32)
    x = dev(torch, a)
    tf.relu_tiles(x, x, n)
    torch.cuda.synchronize()
    assert np.array_equal(host(x), oracle.relu(a))
    x = dev(torch, a)
    tf.add_tiles(x, dev(torch, b), x, n)
    torch.cuda.synchronize()
    assert np.array_equal(host(x), oracle.add(a, b))
    rows, cols = 96, 4096
    m = oracle.rand_bf16((rows, cols), 33)
    band = np.zeros((32, cols), dtype=np.uint16)
    band[0] = oracle.rand_bf16(cols, 34, -0.5, 0.5)
    x = dev(torch, oracle.tilize(m))
    tf.bias_add_tiles(x, dev(torch, oracle.tilize(band)), x, rows, cols)
    torch.cuda.synchronize()
    assert np.array_equal(oracle.untilize(host(x), rows, cols), oracle.bias_add(m, band[0]))
    assert tf.device_error() == 0


@pytest.mark.parametrize("rows,cols", [(32, 32), (64, 160), (256, 512), (1056, 3 * 32 * 7)])
def test_bias_add_bit_exact(torch_cuda, tf, rows, cols):
    torch = torch_cuda
    x = oracle.rand_bf16((rows, cols), 6)
    bias = oracle.rand_bf16(cols, 7, -0.5, 0.5)
    # Bias band in the reference's convention: row 0 of a 32-row tile band.
    band = np.zeros((32, cols), dtype=np.uint16)
    band[0] = bias
    out = empty(torch, rows * cols)
    tf.bias_add_tiles(dev(torch, oracle.tilize(x)), dev(torch, oracle.tilize(band)), out, rows, cols)
    torch.cuda.synchronize()
    got = oracle.untilize(host(out), rows, cols)
    assert np.array_equal(got, oracle.bias_add(x, bias))


def run_gemm(torch, tf, a, b, bias=None, relu=False):
    M, K = a.shape
    N = b.shape[1]
    c = empty(torch, M * N)
    bias_t = dev(torch, bias) if bias is not None else None
    tf.matmul_tiles(dev(torch, oracle.tilize(a)), dev(torch, oracle.tilize(b)), c, M // 32, K // 32,
                    N // 32, bias=bias_t, relu=relu)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    return oracle.untilize(host(c), M, N)


def check_gemm(got, exp, a, b, K):
    amax = float(np.max(np.abs(oracle.bf16_to_f32(a))))
    bmax = float(np.max(np.abs(oracle.bf16_to_f32(b))))
    err = oracle.normalized_error(got, exp, K, amax, bmax)
    assert err <= GEMM_NORM_TOL, f"normalized error {err}"
    bad, wa, wr = oracle.compare(got, exp)
    assert bad == 0, f"{bad} elements outside max(0.05, 1%): worst abs {wa}, rel {wr}"


@pytest.mark.parametrize("tag", ["mnk_2_4_2", "mnk_8_8_8", "mnk_3_5_2"])
def test_gemm_against_reference_fixtures(torch_cuda, tf, golden, tag):
    g = golden("matmul_" + tag)
    got = run_gemm(torch_cuda, tf, g["a"], g["b"])
    check_gemm(got, g["c"], g["a"], g["b"], g["a"].shape[1])


@pytest.mark.parametrize("Mt,Kt,Nt", [(1, 1, 1), (1, 4, 1), (4, 2, 8), (5, 7, 9), (9, 3, 17),
                                      (12, 33, 20), (33, 16, 31)])
def test_gemm_shapes_and_tails(torch_cuda, tf, Mt, Kt, Nt):
    a = oracle.rand_bf16((Mt * 32, Kt * 32), Mt * 7 + Kt)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), Nt * 5 + Kt)
    got = run_gemm(torch_cuda, tf, a, b)
    check_gemm(got, oracle.matmul(a, b, threads=8), a, b, Kt * 32)


@pytest.mark.parametrize("Mt,Kt,Nt", [(3, 4, 5), (20, 6, 9), (17, 5, 24)])
def test_gemm_output_only_16_byte_aligned(torch_cuda, tf, Mt, Kt, Nt):
    """C at a 16-byte (not 32-byte) aligned address, as the 16-byte L1 bump
    allocator can hand out: the epilogue's 128-bit store path gives the same
    bits as the 256-bit path (each of the three kernels)."""
    torch = torch_cuda
    a = oracle.rand_bf16((Mt * 32, Kt * 32), 70 + Mt)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), 71 + Nt)
    ad, bd = dev(torch, oracle.tilize(a)), dev(torch, oracle.tilize(b))
    n = Mt * Nt * 1024
    c32 = empty(torch, n)
    buf = torch.full((n + 16,), 0x1234, dtype=torch.int16, device="cuda")
    c16 = buf[8:8 + n]                       # +16 bytes
    assert c16.data_ptr() % 32 == 16
    tf.matmul_tiles(ad, bd, c32, Mt, Kt, Nt)
    tf.matmul_tiles(ad, bd, c16, Mt, Kt, Nt)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    assert torch.equal(c32, c16)
    assert torch.all(buf[:8] == 0x1234) and torch.all(buf[8 + n:] == 0x1234)
    check_gemm(oracle.untilize(host(c16), Mt * 32, Nt * 32), oracle.matmul(a, b, threads=8), a, b, Kt * 32)


def test_gemm_fused_bias_relu(torch_cuda, tf):
    Mt, Kt, Nt = 6, 9, 10
    a = oracle.rand_bf16((Mt * 32, Kt * 32), 21)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), 22)
    bias = oracle.rand_bf16(Nt * 32, 23, -2.0, 2.0)
    got = run_gemm(torch_cuda, tf, a, b, bias=bias, relu=True)
    exp = oracle.relu(oracle.bias_add(oracle.matmul(a, b, threads=8), bias))
    check_gemm(got, exp, a, b, Kt * 32)
    assert np.all(oracle.bf16_to_f32(got) >= 0)


def test_gemm_formula_inputs_exact_rule(torch_cuda, tf):
    """The matmul_mnk test's own inputs and comparator at 256^3."""
    a, b = oracle.gen_matmul_inputs(256, 256, 256)
    got = run_gemm(torch_cuda, tf, a, b)
    bad, wa, wr = oracle.compare(got, oracle.matmul(a, b))
    assert bad == 0, (wa, wr)


def test_gemm_large_sampled(torch_cuda, tf):
    """2048 x 4096 x 1024 (beyond one persistent wave): sampled rows vs oracle."""
    torch = torch_cuda
    M, K, N = 2048, 4096, 1024
    a = oracle.rand_bf16((M, K), 31)
    b = oracle.rand_bf16((K, N), 32)
    got = run_gemm(torch, tf, a, b)
    rows = [0, 1, 127, 128, 1000, 2047]
    for r in rows:
        exp = oracle.matmul(a[r:r + 1], b)
        check_gemm(got[r:r + 1], exp, a[r:r + 1], b, K)
