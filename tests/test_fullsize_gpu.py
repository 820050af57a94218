"""The benchmark workloads at full size, checked through sampled outputs and
size-independent properties (the whole outputs are too large for the CPU
oracle):

* tiled GEMM 65536 x 8192 x 8192 and 16384^3 (tile layout, fp32 accumulate):
  output rows spread over every 2-SM row block, the last tile row and
  interior tiles against the oracle's row products (normalised error <= 1e-2
  and the reference's max(0.05, 1%) rule);
* GEMM linearity: A (B1 + B2) with bf16-exact operands equals A B1 + A B2
  sampled (products of small integers are exact in fp32);
* tilize / untilize of 16384^2: round trip is the identity, sampled tiles
  bit-exact;
* add_tiles / relu on 2^28 elements and bias_add on 16384^2: bit-exact
  against the oracle on 2^20 sampled positions (the golden arithmetic is
  element-wise).
"""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    import ttfoil
    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    ttfoil.lib()
    return torch, ttfoil


def rnd_dev(torch, n, seed, lo=-1.0, hi=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.rand(n, device="cuda", generator=g) * (hi - lo) + lo).to(torch.bfloat16).view(torch.int16)


def bits(t):
    return t.cpu().numpy().view(np.uint16)


def row_of_tiles(t, r, rows_t, cols):
    """Row r of a tile-layout matrix with `cols` columns, from a CUDA tensor."""
    ct = cols // 32
    mt, r0 = divmod(r, 32)
    band = bits(t[mt * ct * 1024:(mt + 1) * ct * 1024])
    return oracle.untilize(band, 32, cols)[r0:r0 + 1]


@pytest.mark.parametrize("M,N,K", [(65536, 8192, 8192), (16384, 16384, 16384)])
def test_gemm_full_size_sampled_rows(env, M, N, K):
    torch, tf = env
    a = rnd_dev(torch, M * K, 1)   # tile layout of a U(-1,1) matrix
    b = rnd_dev(torch, K * N, 2)
    c = torch.empty(M * N, dtype=torch.int16, device="cuda")
    tf.matmul_tiles(a, b, c, M // 32, K // 32, N // 32)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    b_rm = oracle.untilize(bits(b), K, N)
    rows = [0, 1, 31, 255, 256, M // 2 + 7, M - 129, M - 1]
    for r in rows:
        a_row = row_of_tiles(a, r, M // 32, K)
        exp = oracle.matmul(a_row, b_rm, threads=16)
        got = row_of_tiles(c, r, M // 32, N)
        assert oracle.normalized_error(got, exp, K, 1.0, 1.0) <= 1e-2, r
        assert oracle.compare(got, exp)[0] == 0, r
    del a, b, c


def band_rows(t, r0, nrows, cols):
    """Rows [r0, r0 + nrows) (r0, nrows multiples of 32) of a tile-layout
    matrix with `cols` columns, from a CUDA tensor, row-major."""
    ct = cols // 32
    lo, hi = (r0 // 32) * ct * 1024, ((r0 + nrows) // 32) * ct * 1024
    return oracle.untilize(bits(t[lo:hi]), nrows, cols)


def test_gemm_8192_full_block_rows(env):
    """8192^3: every element of the first and the last 128 x N block row
    (the half pair-tiles of the first and last 2-SM row blocks, all 32
    column tiles of each) against the oracle's sequential fp32 dot
    products."""
    torch, tf = env
    M = N = K = 8192
    a = rnd_dev(torch, M * K, 11)
    b = rnd_dev(torch, K * N, 12)
    c = torch.empty(M * N, dtype=torch.int16, device="cuda")
    tf.matmul_tiles(a, b, c, M // 32, K // 32, N // 32)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    b_rm = oracle.untilize(bits(b), K, N)
    for r0 in (0, M - 128):
        exp = oracle.matmul(band_rows(a, r0, 128, K), b_rm, threads=16)
        got = band_rows(c, r0, 128, N)
        assert oracle.normalized_error(got, exp, K, 1.0, 1.0) <= 1e-2, r0
        bad, wa, wr = oracle.compare(got, exp)
        assert bad == 0, (r0, bad, wa, wr)
    del a, b, c


def test_gemm_linearity_full_width(env):
    """C(B1 + B2) == C(B1) + C(B2) exactly for small-integer operands at
    16384 x 8192 x 8192: every product and partial sum is an exact fp32
    integer below 2^24, so any dropped, repeated or misplaced k-block breaks
    the equality."""
    torch, tf = env
    M, N, K = 16384, 8192, 8192
    g = torch.Generator(device="cuda").manual_seed(7)
    ints = lambda n, lo, hi: torch.randint(lo, hi, (n,), device="cuda", generator=g).to(torch.bfloat16)
    a = ints(M * K, -2, 3)
    b1 = ints(K * N, -3, 4)
    b2 = ints(K * N, -3, 4)
    out = [torch.empty(M * N, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    tf.matmul_tiles(a, b1, out[0], M // 32, K // 32, N // 32)
    tf.matmul_tiles(a, b2, out[1], M // 32, K // 32, N // 32)
    tf.matmul_tiles(a, b1 + b2, out[2], M // 32, K // 32, N // 32)
    torch.cuda.synchronize()
    # The accumulators are exact integers; a bf16 output below 256 in
    # magnitude is the exact integer (257 already rounds to 256), so compare
    # where all three outputs are below 256.
    s = (out[0].float() + out[1].float())
    t = out[2].float()
    small = (out[0].float().abs() < 256) & (out[1].float().abs() < 256) & (t.abs() < 256)
    assert small.sum().item() > 1000
    assert torch.equal(s[small], t[small])


def test_tilize_full_size_round_trip(env):
    torch, tf = env
    R = C = 16384
    x = rnd_dev(torch, R * C, 3)
    t = torch.empty_like(x)
    back = torch.empty_like(x)
    tf.tilize(x, t, R, C)
    tf.untilize(t, back, R, C)
    torch.cuda.synchronize()
    assert torch.equal(x, back)
    # tiles (0, 0), (257, 3) and the last one against the oracle
    for (ti, tj) in [(0, 0), (257, 3), (R // 32 - 1, C // 32 - 1)]:
        block = bits(x.view(R, C)[ti * 32:(ti + 1) * 32, tj * 32:(tj + 1) * 32].contiguous())
        tile = bits(t[(ti * (C // 32) + tj) * 1024:(ti * (C // 32) + tj + 1) * 1024])
        assert np.array_equal(tile, oracle.tilize(block.reshape(32, 32)))


def test_eltwise_full_size_sampled(env):
    torch, tf = env
    n = 1 << 28
    x = rnd_dev(torch, n, 4)
    y = rnd_dev(torch, n, 5)
    out = torch.empty_like(x)
    idx = torch.randint(0, n, (1 << 20,), device="cuda", generator=torch.Generator(device="cuda").manual_seed(6))
    xs, ys = bits(x[idx]), bits(y[idx])
    tf.add_tiles(x, y, out, n)
    torch.cuda.synchronize()
    assert np.array_equal(bits(out[idx]), oracle.add(xs, ys))
    tf.relu_tiles(x, out, n)
    torch.cuda.synchronize()
    assert np.array_equal(bits(out[idx]), oracle.relu(xs))
    # bias_add on 16384 x 16384 tiles: sampled tile rows against the oracle
    R = C = 16384
    band = rnd_dev(torch, 32 * C, 8)
    tf.bias_add_tiles(x, band, out, R, C)
    torch.cuda.synchronize()
    bias_row = oracle.untilize(bits(band), 32, C)[0:1]
    for r in [0, 33, R - 1]:
        row_in = row_of_tiles(x, r, R // 32, C)
        row_out = row_of_tiles(out, r, R // 32, C)
        assert np.array_equal(row_out, oracle.bias_add(row_in, bias_row)), r
