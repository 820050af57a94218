"""The device-side failure path: a bounded wait that runs out.

Every mbarrier / counter wait inside the tensor-core kernels gives up after a
wall-time limit (a launch parameter, 2 s by default, set here through
foil_set_wait_limit_ns).  On expiry the kernel records FOIL_DEVERR_WAIT_TIMEOUT
in the device error word, its roles leave their loops, it waits (bounded) for
its copies and tensor-core operations in flight, frees its tensor memory and
returns.  This is the B200 counterpart of the reference's dispatch timeout
(src/dispatch.cpp:203-208), moved into the kernels.

The test makes a wait run out on purpose without faulting anything: the
limit is set to 5 us on GEMMs whose first output tile takes far longer
(K = 16384), so the epilogue's first wait for a finished accumulator must
expire.  Each GEMM kernel variant is driven that way.  Afterwards, with the
default limit back, a GEMM and a convolution on the same device must pass
parity, so nothing was left waiting and tensor memory was released.
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
    assert ttfoil.device_error() == 0
    return torch, ttfoil


def dev(torch, x):
    return torch.from_numpy(np.ascontiguousarray(x).reshape(-1).view(np.int16)).cuda()


# (Mt, Kt, Nt): single-SM kernel (Mt <= 4), 2-SM 256-column kernel (Nt <= 8),
# 2-SM 512-column kernel.  K = 32 Kt = 16384 in each.
SHAPES = [(4, 512, 8), (16, 512, 8), (16, 512, 32)]


@pytest.mark.parametrize("Mt,Kt,Nt", SHAPES)
def test_wait_limit_expires_then_device_recovers(env, Mt, Kt, Nt):
    torch, tf = env
    g = torch.Generator(device="cuda").manual_seed(Mt * 1000 + Nt)
    a = ((torch.rand(Mt * Kt * 1024, device="cuda", generator=g) * 2 - 1)).to(torch.bfloat16)
    b = ((torch.rand(Kt * Nt * 1024, device="cuda", generator=g) * 2 - 1)).to(torch.bfloat16)
    c = torch.zeros(Mt * Nt * 1024, dtype=torch.bfloat16, device="cuda")

    prev = tf.set_wait_limit_ns(5000)
    try:
        tf.matmul_tiles(a, b, c, Mt, Kt, Nt)
        torch.cuda.synchronize()
    finally:
        tf.set_wait_limit_ns(prev)
    err = tf.device_error()
    assert err & tf.DEVERR_WAIT_TIMEOUT, f"error word {err:#x}: no wait expired"
    assert tf.device_error() == 0, "reading the word clears it"

    # Default limit: the same GEMM completes and matches the oracle.
    tf.matmul_tiles(a, b, c, Mt, Kt, Nt)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    bits = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)
    a_rm = oracle.untilize(bits(a), Mt * 32, Kt * 32)
    b_rm = oracle.untilize(bits(b), Kt * 32, Nt * 32)
    c_rm = oracle.untilize(bits(c), Mt * 32, Nt * 32)
    rows = [0, Mt * 32 // 2 + 3, Mt * 32 - 1]
    exp = oracle.matmul(a_rm[rows], b_rm, threads=8)
    assert oracle.normalized_error(c_rm[rows], exp, Kt * 32, 1.0, 1.0) <= 1e-2
    assert oracle.compare(c_rm[rows], exp)[0] == 0


def test_conv_after_expired_waits(env):
    """A convolution right after the expired GEMM waits: tensor memory and
    the SMs are free again (full-size oracle comparison)."""
    torch, tf = env
    N, H, W, Cin, Cout = 2, 28, 28, 64, 128
    x = oracle.rand_bf16((N, H, W, Cin), 501)
    w = oracle.randn_bf16((Cout, 3, 3, Cin), 502, np.sqrt(2.0 / 576))
    cb = oracle.rand_bf16((Cout,), 503, -0.1, 0.1)
    y = torch.zeros(N * H * W * Cout, dtype=torch.int16, device="cuda")
    tf.conv2d_nhwc(dev(torch, x), dev(torch, w), dev(torch, cb), y, N, H, W, Cin, Cout, 3, 3, 1, 1, relu=True)
    torch.cuda.synchronize()
    assert tf.device_error() == 0
    exp = oracle.conv_nhwc(x, w, cb, 1, 1, relu=True, threads=8)
    got = y.cpu().numpy().view(np.uint16).reshape(exp.shape)
    assert oracle.compare(got, exp)[0] == 0


def test_wait_limit_setter_round_trip(env):
    torch, tf = env
    prev = tf.set_wait_limit_ns(123456)
    assert tf.set_wait_limit_ns(0) == 123456
    assert tf.set_wait_limit_ns(prev) == 2_000_000_000
