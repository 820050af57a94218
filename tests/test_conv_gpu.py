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
}

VARIANT_CASES = [  # x shape, w shape, stride, pad
    ((1, 56, 56, 64), (64, 3, 3, 64), 1, 1),       # config-2 shape
    ((2, 30, 30, 128), (256, 3, 3, 128), 2, 1),    # BN 256, two channel blocks
    ((3, 10, 10, 64), (192, 3, 3, 64), 1, 1),      # M = 300: the second pair's odd CTA has no valid row
    ((2, 14, 14, 256), (64, 3, 3, 256), 1, 1),     # K = 2304: 144 KiB of resident weights
    ((1, 23, 29, 128), (128, 3, 3, 128), 2, 1),    # M = 180, odd sizes
    ((4, 16, 16, 64), (64, 5, 5, 64), 1, 2),       # 5x5
]


@pytest.fixture(scope="module")
def variant_inputs(env, tmp_path_factory):
    """Seeded inputs of VARIANT_CASES, their default-path outputs (checked
    against the oracle) and the script that reruns a case in a subprocess."""
    d = tmp_path_factory.mktemp("variants")
    script = d / "run_case.py"
    script.write_text(
        "import sys, numpy as np, torch\n"
        f"sys.path.insert(0, {PKG!r})\n"
        "import ttfoil\n"
        "d = np.load(sys.argv[1])\n"
        "x, w, b = (torch.from_numpy(d[k].view(np.int16)).cuda() for k in ('x', 'w', 'b'))\n"
        "N, H, W, Cin = d['x'].shape; Cout, KH, KW, _ = d['w'].shape; s, p = int(d['s']), int(d['p'])\n"
        "Ho, Wo = (H + 2 * p - KH) // s + 1, (W + 2 * p - KW) // s + 1\n"
        "y = torch.zeros(N * Ho * Wo * Cout, dtype=torch.int16, device='cuda')\n"
        "ttfoil.conv2d_nhwc(x, w, b, y, N, H, W, Cin, Cout, KH, KW, s, p, relu=True)\n"
        "torch.cuda.synchronize(); assert ttfoil.device_error() == 0\n"
        "np.save(sys.argv[2], y.cpu().numpy())\n")
    cases = []
    for i, (xs, ws, stride, pad) in enumerate(VARIANT_CASES):
        x = oracle.rand_bf16(xs, 40 + i)
        w = oracle.randn_bf16(ws, 50 + i, np.sqrt(2.0 / (ws[1] * ws[2] * ws[3])))
        b = oracle.rand_bf16((ws[0],), 60 + i, -0.1, 0.1)
        got = run_conv(env, x, w, b, stride, pad, relu=True)
        check(got, oracle.conv_nhwc(x, w, b, stride, pad, relu=True, threads=8), x, w)
        inp = d / f"in{i}.npz"
        np.savez(inp, x=x, w=w, b=b, s=stride, p=pad)
        cases.append((inp, got))
    return script, cases


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_kernel_variants_agree_bitwise(variant_inputs, tmp_path, variant):
    """Every kernel variant (gather producer, single-CTA tensor copies, 2-SM
    weight-stationary pair) feeds identical operand tiles in the same K order,
    so each reproduces the default path's output bit for bit on every case;
    the default outputs are themselves checked against the oracle."""
    script, cases = variant_inputs
    env_vars = dict(os.environ, **VARIANTS[variant])
    for i, (inp, got) in enumerate(cases):
        out = tmp_path / f"out{i}.npy"
        r = subprocess.run([sys.executable, str(script), str(inp), str(out)], env=env_vars,
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        ref = np.load(out).view(np.uint16).reshape(got.shape)
        assert np.array_equal(got, ref), (i, int(np.sum(got != ref)))


def test_conv_rejects_bad_shapes(env):
    torch, tf = env
    z = torch.zeros(1024, dtype=torch.int16, device="cuda")
    with pytest.raises(tf.FoilError, match="multiples of 16"):
        tf.conv2d_nhwc(z, z, None, z, 1, 4, 4, 8, 16, 3, 3, 1, 1)
    with pytest.raises(tf.FoilError, match="unsupported"):
        tf.conv2d_nhwc(z, z, None, z, 1, 4, 4, 16, 16, 3, 3, 0, 1)
