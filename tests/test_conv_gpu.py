"""Parity of the implicit-GEMM NHWC convolution (foil_conv2d_nhwc_dev) with the
oracle and with the reference's own conv goldens.

Tolerance (as for the GEMM): normalised error max|d| / (sqrt(K) max|x| max|w|)
<= 1e-2 with K = KH*KW*Cin, and the reference comparator max(0.05, 1%) with
zero failures.  The fused epilogue is checked against the composition of the
goldens relu(bf16(bf16(acc) + bias)).
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tt-foil_b200")


@pytest.fixture(scope="module")
def env():
    import torch
    import ttfoil
    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    ttfoil.lib()
    return torch, ttfoil


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def run_conv(env, x, w, bias, stride, pad, relu):
    torch, tf = env
    N, H, W, Cin = x.shape
    Cout, KH, KW, _ = w.shape
    Ho, Wo = (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KW) // stride + 1
    y = torch.full((N * Ho * Wo * Cout,), 0x7fc0, dtype=torch.int16, device="cuda")
    tf.conv2d_nhwc(dev(torch, x), dev(torch, w), dev(torch, bias) if bias is not None else None, y,
                   N, H, W, Cin, Cout, KH, KW, stride, pad, relu=relu)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    return y.cpu().numpy().view(np.uint16).reshape(N, Ho, Wo, Cout)


def check(got, exp, x, w):
    K = w.shape[1] * w.shape[2] * w.shape[3]
    xm = float(np.max(np.abs(oracle.bf16_to_f32(x)))) or 1.0
    wm = float(np.max(np.abs(oracle.bf16_to_f32(w)))) or 1.0
    err = oracle.normalized_error(got, exp, K, xm, wm)
    assert err <= 1e-2, f"normalized error {err}"
    bad, wa, wr = oracle.compare(got, exp)
    assert bad == 0, (bad, wa, wr)


@pytest.mark.parametrize("tag", ["conv3_1_9_2", "conv3_2_18_14", "conv3s2_1_9_2", "conv3s2_4_18_8",
                                 "conv1_2_2_2", "conv1_8_4_16"])
def test_conv_against_reference_goldens(env, golden, tag):
    """The reference tests' conv goldens (CHW), re-indexed to NHWC."""
    g = golden("conv_" + tag)
    Cin, H, W, Cout, k, stride, pad = (int(v) for v in g["dims"])
    if Cin % 16:
        pytest.skip("Cin not a multiple of 16")
    x = np.ascontiguousarray(g["x"].transpose(1, 2, 0))[None]
    w = np.ascontiguousarray(g["w"].transpose(0, 2, 3, 1))
    got = run_conv(env, x, w, None, stride, pad, relu=False)
    exp = np.ascontiguousarray(g["y"].transpose(1, 2, 0))[None]
    check(got, exp, x, w)


@pytest.mark.parametrize("tag", ["conv3_1_9_2", "conv3_2_18_14", "conv3s2_1_9_2", "conv3s2_4_18_8",
                                 "conv1_2_2_2", "conv1_8_4_16"])
def test_conv_chw_entry_on_reference_goldens(env, golden, tag):
    """foil_conv2d_chw_dev takes the reference tests' own tensors as they are:
    x (Cin, H, W), the reshaped weights (Cout, Cin*KH*KW), y (Cout, Ho, Wo);
    no host transposition or im2col, any channel count."""
    torch, tf = env
    g = golden("conv_" + tag)
    Cin, H, W, Cout, k, stride, pad = (int(v) for v in g["dims"])
    x = np.ascontiguousarray(g["x"])
    w = np.ascontiguousarray(g["w"]).reshape(Cout, Cin * k * k)
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    y = torch.full((Cout * Ho * Wo,), 0x7fc0, dtype=torch.int16, device="cuda")
    tf.conv2d_chw(dev(torch, x), dev(torch, w), None, y, 1, Cin, H, W, Cout, k, k, stride, pad)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    got = y.cpu().numpy().view(np.uint16).reshape(Cout, Ho, Wo)
    check(got, g["y"].reshape(Cout, Ho, Wo), x, w.reshape(Cout, Cin, k, k))


def test_conv_chw_entry_batch_bias_relu(env):
    """Batch 3, channel counts that are not multiples of 16, bias + relu:
    against the oracle's NHWC convolution of the same tensors."""
    torch, tf = env
    N, Cin, H, W, Cout, k, stride, pad = 3, 24, 15, 13, 40, 3, 2, 1
    x = oracle.rand_bf16((N, Cin, H, W), 81)
    w = oracle.randn_bf16((Cout, Cin, k, k), 82, np.sqrt(2.0 / (Cin * k * k)))
    b = oracle.rand_bf16((Cout,), 83, -0.1, 0.1)
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    y = torch.zeros(N * Cout * Ho * Wo, dtype=torch.int16, device="cuda")
    tf.conv2d_chw(dev(torch, x), dev(torch, w), dev(torch, b), y, N, Cin, H, W, Cout, k, k, stride, pad, relu=True)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    got = y.cpu().numpy().view(np.uint16).reshape(N, Cout, Ho, Wo).transpose(0, 2, 3, 1)
    xn = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    wn = np.ascontiguousarray(w.transpose(0, 2, 3, 1))
    exp = oracle.conv_nhwc(xn, wn, b, stride, pad, relu=True, threads=8)
    check(np.ascontiguousarray(got), exp, xn, wn)


def test_config2_conv3x3_s1_bias_relu(env):
    """N=1, 56x56, 64 -> 64, 3x3 stride 1 pad 1, bias + relu (M=3136, N=64, K=576)."""
    x = oracle.rand_bf16((1, 56, 56, 64), 2)
    w = oracle.randn_bf16((64, 3, 3, 64), 21, np.sqrt(1.0 / 576))
    bias = oracle.rand_bf16((64,), 22, -0.1, 0.1)
    got = run_conv(env, x, w, bias, 1, 1, relu=True)
    exp = oracle.conv_nhwc(x, w, bias, 1, 1, relu=True, threads=8)
    check(got, exp, x, w)


def test_config3_pair_sampled(env):
    """Batch 32: 3x3 s2 112^2 x 64 -> 128, then 1x1 56^2 x 128 -> 256, bias + relu
    each; images 0 and 31 against the oracle, every image finite and >= 0."""
    torch, tf = env
    x = oracle.rand_bf16((32, 112, 112, 64), 3)
    w1 = oracle.randn_bf16((128, 3, 3, 64), 31, np.sqrt(2.0 / 576))
    b1 = oracle.rand_bf16((128,), 32, -0.1, 0.1)
    w2 = oracle.randn_bf16((256, 1, 1, 128), 33, np.sqrt(2.0 / 128))
    b2 = oracle.rand_bf16((256,), 34, -0.1, 0.1)
    y1 = run_conv(env, x, w1, b1, 2, 1, relu=True)
    y2 = run_conv(env, y1, w2, b2, 1, 0, relu=True)
    assert y1.shape == (32, 56, 56, 128) and y2.shape == (32, 56, 56, 256)
    for img in (0, 31):
        e1 = oracle.conv_nhwc(x, w1, b1, 2, 1, relu=True, images=(img, img + 1), threads=8)[img]
        check(y1[img:img + 1], e1[None], x, w1)
        e2 = oracle.conv_nhwc(y1, w2, b2, 1, 0, relu=True, images=(img, img + 1), threads=8)[img]
        check(y2[img:img + 1], e2[None], y1, w2)
    f = oracle.bf16_to_f32(y2)
    assert np.all(np.isfinite(f)) and np.all(f >= 0)


@pytest.mark.parametrize("N,H,W,Cin,Cout,k,stride,pad,bias,relu", [
    (1, 7, 9, 16, 16, 3, 1, 1, True, False),     # kc = 16, Cout = one 16-wide block
    (2, 10, 6, 32, 48, 3, 2, 1, True, True),     # kc = 32, Cout tail inside BN = 64
    (1, 13, 11, 96, 320, 3, 1, 1, False, True),  # kc = 32 over 3 blocks, 2 column tiles of 256
    (3, 9, 9, 128, 192, 1, 2, 0, True, True),    # 1x1 stride 2, BN = 256 with tail
    (1, 5, 5, 64, 128, 3, 1, 0, True, True),     # no padding, tiny M
    (4, 16, 16, 64, 64, 5, 1, 2, False, False),  # 5x5 kernel
])
def test_conv_shapes(env, N, H, W, Cin, Cout, k, stride, pad, bias, relu):
    x = oracle.rand_bf16((N, H, W, Cin), N * 100 + H)
    w = oracle.randn_bf16((Cout, k, k, Cin), Cout + k, np.sqrt(2.0 / (k * k * Cin)))
    b = oracle.rand_bf16((Cout,), 7, -0.2, 0.2) if bias else None
    got = run_conv(env, x, w, b, stride, pad, relu)
    exp = oracle.conv_nhwc(x, w, b, stride, pad, relu=relu, threads=8)
    check(got, exp, x, w)


@pytest.mark.parametrize("N,H,W,Cin,Cout,kh,kw,stride,pad", [
    (2, 12, 10, 64, 64, 3, 5, 1, 1),    # non-square kernel: W and H bounding boxes differ
    (1, 20, 17, 64, 128, 3, 3, 3, 1),   # stride 3
    (1, 9, 31, 192, 64, 1, 3, 2, 0),    # 1 x 3, three channel blocks
])
def test_conv_rectangular_and_strided(env, N, H, W, Cin, Cout, kh, kw, stride, pad):
    x = oracle.rand_bf16((N, H, W, Cin), 11 + W)
    w = oracle.randn_bf16((Cout, kh, kw, Cin), 12 + kw, np.sqrt(2.0 / (kh * kw * Cin)))
    b = oracle.rand_bf16((Cout,), 13, -0.2, 0.2)
    got = run_conv(env, x, w, b, stride, pad, relu=True)
    exp = oracle.conv_nhwc(x, w, b, stride, pad, relu=True, threads=8)
    check(got, exp, x, w)


VARIANTS = {
    "gather": {"FOIL_CONV_PRODUCER": "gather"},
    "single": {"FOIL_CONV_PRODUCER": "single"},
    "pair": {"FOIL_CONV_PRODUCER": "pair"},
    "plane": {"FOIL_CONV_PRODUCER": "plane"},
    "resident": {"FOIL_CONV_PRODUCER": "resident"},
    # epilogue store paths: rows straight from registers, or staged for
    # tensor stores (each kernel's default is the other one for some shapes)
    "single_direct": {"FOIL_CONV_PRODUCER": "single", "FOIL_CONV_EPILOGUE": "direct"},
    "pair_staged": {"FOIL_CONV_PRODUCER": "pair", "FOIL_CONV_EPILOGUE": "staged"},
    "gather_direct": {"FOIL_CONV_PRODUCER": "gather", "FOIL_CONV_EPILOGUE": "direct"},
}

VARIANT_CASES = [  # x shape, w shape, stride, pad
    ((1, 56, 56, 64), (64, 3, 3, 64), 1, 1),       # config-2 shape
    ((2, 30, 30, 128), (256, 3, 3, 128), 2, 1),    # BN 256, two channel blocks
    ((3, 10, 10, 64), (192, 3, 3, 64), 1, 1),      # M = 300: the second pair's odd CTA has no valid row
    ((2, 14, 14, 256), (64, 3, 3, 256), 1, 1),     # K = 2304: 144 KiB of resident weights
    ((1, 23, 29, 128), (128, 3, 3, 128), 2, 1),    # M = 180, odd sizes
    ((4, 16, 16, 64), (64, 5, 5, 64), 1, 2),       # 5x5
    ((2, 28, 28, 128), (256, 1, 1, 128), 1, 0),    # 1x1, BN 256 (resident weights: 64 KiB)
    ((1, 20, 20, 64), (96, 1, 1, 64), 1, 0),       # 1x1, Cout tail in BN 128
]

# Shapes the plane kernel serves (Cin a multiple of 64, Ho Wo a multiple of
# 32, Wo a multiple of 8, Cout <= 256, <= 25 taps): short and odd window
# counts, a window pair split over two images, Cout tails, strides 2 and 3,
# 1x1, 5x5, three channel blocks, and the two batch-32 configurations at
# batch 2.
PLANE_CASES = [  # x shape, w shape, stride, pad
    ((1, 8, 8, 64), (64, 3, 3, 64), 1, 1),         # one short window; the pair's odd CTA idle
    ((3, 16, 16, 64), (96, 3, 3, 64), 1, 1),       # 6 windows, Cout tail in BN = 128
    ((2, 32, 32, 64), (128, 3, 3, 64), 2, 1),      # stride 2: 6 planes
    ((1, 48, 48, 64), (64, 3, 3, 64), 3, 1),       # stride 3: 9 planes
    ((2, 64, 32, 64), (128, 3, 3, 64), 2, 1),      # Ho != Wo
    ((1, 24, 40, 128), (64, 3, 3, 128), 1, 1),     # two channel blocks, 2 slots
    ((1, 12, 16, 192), (48, 1, 1, 192), 1, 0),     # 1x1, three channel blocks, Cout 48
    ((2, 56, 56, 128), (256, 1, 1, 128), 1, 0),    # config-3 1x1 shape
    ((2, 112, 112, 64), (128, 3, 3, 64), 2, 1),    # config-3 3x3 stride-2 shape
    ((4, 16, 16, 64), (64, 5, 5, 64), 1, 2),       # 25 taps
]

RUN_CASES = (
    "import sys, numpy as np, torch\n"
    f"sys.path.insert(0, {PKG!r})\n"
    "import ttfoil\n"
    "for inp, outp in zip(sys.argv[1::2], sys.argv[2::2]):\n"
    "    d = np.load(inp)\n"
    "    x, w, b = (torch.from_numpy(d[k].view(np.int16)).cuda() for k in ('x', 'w', 'b'))\n"
    "    N, H, W, Cin = d['x'].shape; Cout, KH, KW, _ = d['w'].shape; s, p = int(d['s']), int(d['p'])\n"
    "    Ho, Wo = (H + 2 * p - KH) // s + 1, (W + 2 * p - KW) // s + 1\n"
    "    y = torch.zeros(N * Ho * Wo * Cout, dtype=torch.int16, device='cuda')\n"
    "    try:\n"
    "        ttfoil.conv2d_nhwc(x, w, b, y, N, H, W, Cin, Cout, KH, KW, s, p, relu=True)\n"
    "    except ttfoil.FoilError as e:\n"
    "        assert e.status == 6, e  # FOIL_ERR_UNSUPPORTED: this variant does not serve the shape\n"
    "        continue\n"
    "    torch.cuda.synchronize(); assert ttfoil.device_error() == 0\n"
    "    np.save(outp, y.cpu().numpy())\n")


def make_case(d, i, xs, ws, stride, pad, seed):
    x = oracle.rand_bf16(xs, seed)
    w = oracle.randn_bf16(ws, seed + 10, np.sqrt(2.0 / (ws[1] * ws[2] * ws[3])))
    b = oracle.rand_bf16((ws[0],), seed + 20, -0.1, 0.1)
    inp = d / f"in{i}.npz"
    np.savez(inp, x=x, w=w, b=b, s=stride, p=pad)
    return inp, x, w, b


def run_variant(script, variant, inputs, out_dir):
    """Run every case of `inputs` in one subprocess with the variant forced;
    returns the output path of each case (missing when not served)."""
    outs = [out_dir / f"{variant}_{i}.npy" for i in range(len(inputs))]
    args = [a for pair in zip(map(str, inputs), map(str, outs)) for a in pair]
    r = subprocess.run([sys.executable, str(script)] + args, env=dict(os.environ, **VARIANTS[variant]),
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return outs


@pytest.fixture(scope="module")
def variant_inputs(env, tmp_path_factory):
    """Seeded inputs of VARIANT_CASES, their default-path outputs (checked
    against the oracle) and the script that reruns cases in a subprocess."""
    d = tmp_path_factory.mktemp("variants")
    script = d / "run_cases.py"
    script.write_text(RUN_CASES)
    cases = []
    for i, (xs, ws, stride, pad) in enumerate(VARIANT_CASES):
        inp, x, w, b = make_case(d, i, xs, ws, stride, pad, 40 + i)
        got = run_conv(env, x, w, b, stride, pad, relu=True)
        check(got, oracle.conv_nhwc(x, w, b, stride, pad, relu=True, threads=8), x, w)
        cases.append((inp, got, x, w, b, stride, pad))
    return script, cases


@pytest.mark.parametrize("variant", ["gather", "single", "pair", "plane", "resident", "single_direct",
                                     "pair_staged", "gather_direct"])
def test_kernel_variants(variant_inputs, tmp_path, variant):
    """The im2col kernels (gather producer, single-CTA tensor copies, 2-SM
    weight-stationary pair, single-CTA with resident weights, where it fits)
    feed identical operand tiles in the same K order, and both epilogue
    store paths write the same values, so each reproduces the default path's
    output bit for bit on every case.
    The plane kernel sums the same products in plane order: where it serves
    a case, its output is checked against the oracle."""
    script, cases = variant_inputs
    outs = run_variant(script, variant, [c[0] for c in cases], tmp_path)
    served = 0
    for i, ((inp, got, x, w, b, stride, pad), out) in enumerate(zip(cases, outs)):
        if not out.exists():
            assert variant in ("plane", "resident"), f"{variant} must serve case {i}"
            continue
        served += 1
        y = np.load(out).view(np.uint16).reshape(got.shape)
        if variant == "plane":
            check(y, oracle.conv_nhwc(x, w, b, stride, pad, relu=True, threads=8), x, w)
        else:
            assert np.array_equal(y, got), (i, int(np.sum(y != got)))
    assert served >= 2


def test_plane_kernel_shapes(env, tmp_path):
    """Every PLANE_CASES shape through the plane kernel (forced: the run fails
    if it does not serve the shape), against the oracle; the larger cases
    on sampled images."""
    script = tmp_path / "run_cases.py"
    script.write_text(RUN_CASES)
    made = [make_case(tmp_path, i, *c, 700 + 30 * i) for i, c in enumerate(PLANE_CASES)]
    outs = run_variant(script, "plane", [m[0] for m in made], tmp_path)
    for i, ((inp, x, w, b), out, (xs, ws, stride, pad)) in enumerate(zip(made, outs, PLANE_CASES)):
        assert out.exists(), f"plane kernel did not serve case {i}"
        N, H, W, _ = xs
        Ho, Wo = (H + 2 * pad - ws[1]) // stride + 1, (W + 2 * pad - ws[2]) // stride + 1
        y = np.load(out).view(np.uint16).reshape(N, Ho, Wo, ws[0])
        imgs = (0, N - 1) if H * W > 4096 else tuple(range(N))
        for n in sorted(set(imgs)):
            e = oracle.conv_nhwc(x, w, b, stride, pad, relu=True, images=(n, n + 1), threads=8)[n]
            check(y[n:n + 1], e[None], x, w)


def test_conv_rejects_bad_shapes(env):
    torch, tf = env
    z = torch.zeros(1024, dtype=torch.int16, device="cuda")
    with pytest.raises(tf.FoilError, match="multiples of 16"):
        tf.conv2d_nhwc(z, z, None, z, 1, 4, 4, 8, 16, 3, 3, 1, 1)
    with pytest.raises(tf.FoilError, match="unsupported"):
        tf.conv2d_nhwc(z, z, None, z, 1, 4, 4, 16, 16, 3, 3, 0, 1)


@pytest.mark.parametrize("shape", [
    ((8, 56, 56, 64), (64, 3, 3, 64), 1, 1),      # pair kernel (rows from registers)
    ((2, 28, 28, 128), (256, 1, 1, 128), 1, 0),   # resident-weight kernel (tensor stores)
])
def test_output_only_16_byte_aligned(env, shape):
    """An output buffer that is 16- but not 32-byte aligned: the pair
    kernel's register epilogue takes its 128-bit store path, the tensor-store
    epilogues start their boxes there; both bit-equal to an aligned run."""
    torch, tf = env
    xs, ws, stride, pad = shape
    x = oracle.rand_bf16(xs, 911)
    w = oracle.randn_bf16(ws, 912, np.sqrt(2.0 / (ws[1] * ws[2] * ws[3])))
    b = oracle.rand_bf16((ws[0],), 913, -0.1, 0.1)
    N, H, W, Cin = xs
    Cout, KH, KW, _ = ws
    Ho, Wo = (H + 2 * pad - KH) // stride + 1, (W + 2 * pad - KW) // stride + 1
    n = N * Ho * Wo * Cout
    ref = run_conv(env, x, w, b, stride, pad, relu=True)
    big = torch.full((n + 16,), 0x7fc0, dtype=torch.int16, device="cuda")
    y = big[8:8 + n]                                   # base + 16 bytes
    assert y.data_ptr() % 32 == 16
    tf.conv2d_nhwc(dev(torch, x), dev(torch, w), dev(torch, b), y, N, H, W, Cin, Cout, KH, KW, stride, pad,
                   relu=True)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    got = big.cpu().numpy().view(np.uint16)
    assert np.array_equal(got[8:8 + n].reshape(ref.shape), ref)
    assert np.all(got[:8] == 0x7fc0) and np.all(got[8 + n:] == 0x7fc0), "bytes outside y written"
