"""Host-buffer pipelines (foil_matmul_tiles_host, foil_conv2d_nhwc_host):
chunked copies overlapping the kernels must give the device entry points'
results.  Chunks of whole 2-SM row blocks run the same kernel on the same
tiles as one device call, so those results are compared bit for bit; other
chunkings are checked against the oracle with the GEMM tolerance."""
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


def pinned(torch, a):
    t = torch.empty(a.size, dtype=torch.int16, pin_memory=True)
    t.numpy()[:] = np.ascontiguousarray(a).reshape(-1).view(np.int16)
    return t


def gemm_device(torch, tf, a, b, Mt, Kt, Nt, bias, relu):
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x).reshape(-1).view(np.int16)).cuda()
    c = torch.zeros(Mt * Nt * 1024, dtype=torch.int16, device="cuda")
    tf.matmul_tiles(dev(a), dev(b), c, Mt, Kt, Nt, bias=None if bias is None else dev(bias), relu=relu)
    torch.cuda.synchronize()
    return c.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("Mt,Kt,Nt,chunk", [(32, 8, 12, 8), (24, 5, 9, 16), (64, 16, 8, 0)])
def test_matmul_host_matches_device_bitwise(env, Mt, Kt, Nt, chunk):
    torch, tf = env
    a = oracle.tilize(oracle.rand_bf16((Mt * 32, Kt * 32), 70 + Mt))
    b = oracle.tilize(oracle.rand_bf16((Kt * 32, Nt * 32), 71 + Nt))
    bias = oracle.rand_bf16((Nt * 32,), 72, -0.5, 0.5)
    exp = gemm_device(torch, tf, a, b, Mt, Kt, Nt, bias, True)
    c = torch.zeros(Mt * Nt * 1024, dtype=torch.int16, pin_memory=True)
    before = torch.cuda.current_device()
    tf.matmul_tiles_host(0, pinned(torch, a), pinned(torch, b), c, Mt, Kt, Nt,
                         bias=pinned(torch, bias), relu=True, chunk_rows=chunk)
    assert torch.cuda.current_device() == before
    assert np.array_equal(c.numpy().view(np.uint16), exp)


def test_matmul_host_ragged_chunks_and_pageable(env):
    """Chunks of 3 tile rows (the last one shorter), pageable numpy buffers."""
    torch, tf = env
    Mt, Kt, Nt = 11, 6, 5
    a_rm = oracle.rand_bf16((Mt * 32, Kt * 32), 81)
    b_rm = oracle.rand_bf16((Kt * 32, Nt * 32), 82)
    c = np.zeros(Mt * Nt * 1024, dtype=np.uint16)
    tf.matmul_tiles_host(0, oracle.tilize(a_rm), oracle.tilize(b_rm), c, Mt, Kt, Nt, chunk_rows=3)
    got = oracle.untilize(c, Mt * 32, Nt * 32)
    exp = oracle.matmul(a_rm, b_rm, threads=8)
    assert oracle.normalized_error(got, exp, Kt * 32, 1.0, 1.0) <= 1e-2
    assert oracle.compare(got, exp)[0] == 0


def test_conv_host_matches_device_bitwise(env):
    torch, tf = env
    N, H, W, Cin, Cout = 5, 14, 14, 64, 64
    x = oracle.rand_bf16((N, H, W, Cin), 91)
    w = oracle.randn_bf16((Cout, 3, 3, Cin), 92, np.sqrt(2.0 / 576))
    bias = oracle.rand_bf16((Cout,), 93, -0.1, 0.1)
    dev = lambda t: torch.from_numpy(np.ascontiguousarray(t).reshape(-1).view(np.int16)).cuda()
    y_dev = torch.zeros(N * H * W * Cout, dtype=torch.int16, device="cuda")
    tf.conv2d_nhwc(dev(x), dev(w), dev(bias), y_dev, N, H, W, Cin, Cout, 3, 3, 1, 1, relu=True)
    torch.cuda.synchronize()
    y = torch.zeros(N * H * W * Cout, dtype=torch.int16, pin_memory=True)
    tf.conv2d_nhwc_host(0, pinned(torch, x), pinned(torch, w), pinned(torch, bias), y, N, H, W, Cin, Cout,
                        3, 3, 1, 1, relu=True, chunk_images=2)
    assert np.array_equal(y.numpy(), y_dev.cpu().numpy())
    exp = oracle.conv_nhwc(x, w, bias, 1, 1, relu=True, threads=8)
    assert oracle.compare(y.numpy().view(np.uint16).reshape(exp.shape), exp)[0] == 0


def test_host_pipeline_release_and_errors(env):
    torch, tf = env
    tf.host_pipeline_release(0)
    with pytest.raises(tf.FoilError, match="null pointer"):
        tf.matmul_tiles_host(0, None, None, None, 1, 1, 1)
    with pytest.raises(tf.FoilError, match="device"):
        tf.matmul_tiles_host(63, 1, 1, 1, 1, 1, 1)


def _host_gemm_and_conv_on(torch, tf, device):
    """foil_matmul_tiles_host and foil_conv2d_nhwc_host on `device`, each
    compared bit for bit with the device entry point run on that device."""
    Mt, Kt, Nt = 16, 8, 12  # 2-SM 512-column kernel (> 48 KiB of shared memory)
    a = oracle.tilize(oracle.rand_bf16((Mt * 32, Kt * 32), 170))
    b = oracle.tilize(oracle.rand_bf16((Kt * 32, Nt * 32), 171))
    N, H, W, Cin, Cout = 2, 20, 20, 64, 128
    x = oracle.rand_bf16((N, H, W, Cin), 172)
    w = oracle.randn_bf16((Cout, 3, 3, Cin), 173, np.sqrt(2.0 / 576))
    cb = oracle.rand_bf16((Cout,), 174, -0.1, 0.1)
    Ho = (H + 2 - 3) // 2 + 1
    with torch.cuda.device(device):
        dev = lambda t: torch.from_numpy(np.ascontiguousarray(t).reshape(-1).view(np.int16)).cuda()
        c_dev = torch.zeros(Mt * Nt * 1024, dtype=torch.int16, device="cuda")
        tf.matmul_tiles(dev(a), dev(b), c_dev, Mt, Kt, Nt)
        y_dev = torch.zeros(N * Ho * Ho * Cout, dtype=torch.int16, device="cuda")
        tf.conv2d_nhwc(dev(x), dev(w), dev(cb), y_dev, N, H, W, Cin, Cout, 3, 3, 2, 1, relu=True)
        torch.cuda.synchronize()
        assert tf.device_error() == 0
        c_exp, y_exp = c_dev.cpu().numpy(), y_dev.cpu().numpy()
    c = torch.zeros(Mt * Nt * 1024, dtype=torch.int16, pin_memory=True)
    before = torch.cuda.current_device()
    tf.matmul_tiles_host(device, pinned(torch, a), pinned(torch, b), c, Mt, Kt, Nt)
    assert torch.cuda.current_device() == before
    assert np.array_equal(c.numpy(), c_exp)
    y = torch.zeros(N * Ho * Ho * Cout, dtype=torch.int16, pin_memory=True)
    tf.conv2d_nhwc_host(device, pinned(torch, x), pinned(torch, w), pinned(torch, cb), y, N, H, W, Cin,
                        Cout, 3, 3, 2, 1, relu=True)
    assert torch.cuda.current_device() == before
    assert np.array_equal(y.numpy(), y_exp)
    return c.numpy().copy(), y.numpy().copy()


def test_host_entry_points_on_two_devices_in_one_process(env):
    """Kernel attributes (the dynamic shared-memory opt-in) and SM counts are
    kept per device: device 0, then device 1, then device 0 again in one
    process, each bitwise equal to the device-resident result, with the
    caller's current device unchanged after every call."""
    torch, tf = env
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    r0 = _host_gemm_and_conv_on(torch, tf, 0)
    r1 = _host_gemm_and_conv_on(torch, tf, 1)
    r0b = _host_gemm_and_conv_on(torch, tf, 0)
    for u, v in zip(r0, r1):
        assert np.array_equal(u, v)
    for u, v in zip(r0, r0b):
        assert np.array_equal(u, v)
    tf.host_pipeline_release(1)
    assert torch.cuda.current_device() == 0
