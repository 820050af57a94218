"""The allocation-free GEMM entry point (foil_matmul_tiles_noalloc_dev).

It exists for callers that cannot allocate device memory when they launch
(allocator callbacks, processes whose GPU memory another allocator owns,
loops that forbid allocation after start-up): its scratch — the kernel's
4-byte error word — lives in a 256-byte array compiled into libfoil instead of
a cudaMalloc'd word.  Checked here through the C-ABI: two calls in a row, each
against the allocating entry point foil_matmul_tiles_dev on the same inputs.
Both launch the same kernel on the same operands, so the outputs must agree
bit for bit; each is also within the GEMM tolerance of the oracle
(normalised error <= 1e-2).  Plus: status 0, one kernel launch per call, and
no change in free device memory across a call after the first.

The file name sorts last so that a stopping run has executed every other test
first; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


def test_noalloc_gemm_matches_allocating_entry_point():
    import torch
    import ttfoil

    assert torch.cuda.is_available()
    torch.cuda.set_device(0)
    L = ttfoil.lib()
    stream = torch.cuda.current_stream()

    def dev(x):
        return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda()

    cases = [  # (Mt, Kt, Nt, bias+relu): a one-block and a two-SM shape
        (3, 5, 9, True),
        (12, 8, 10, False),
    ]
    status = ctypes.c_uint32(123)
    for call, (Mt, Kt, Nt, fused) in enumerate(cases):
        a = oracle.rand_bf16((Mt * 32, Kt * 32), 100 + call)
        b = oracle.rand_bf16((Kt * 32, Nt * 32), 200 + call)
        bias = oracle.rand_bf16(Nt * 32, 300 + call, -0.5, 0.5) if fused else None
        a_d, b_d = dev(oracle.tilize(a)), dev(oracle.tilize(b))
        bias_d = dev(bias) if fused else None
        c_ref = torch.full((Mt * Nt * 1024,), 7, dtype=torch.int16, device="cuda")
        c_new = torch.full((Mt * Nt * 1024,), 9, dtype=torch.int16, device="cuda")

        ttfoil.matmul_tiles(a_d, b_d, c_ref, Mt, Kt, Nt, bias=bias_d, relu=fused, stream=stream)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        launches = ttfoil.launch_count()
        rc = L.foil_matmul_tiles_noalloc_dev(
            a_d.data_ptr(), b_d.data_ptr(), c_new.data_ptr(), Mt, Kt, Nt,
            bias_d.data_ptr() if fused else None, 1 if fused else 0, stream.cuda_stream,
            ctypes.byref(status))
        assert rc == 0, L.foil_last_error()
        assert status.value == 0
        assert ttfoil.launch_count() == launches + 1
        torch.cuda.synchronize()
        if call > 0:  # after the per-device set-up of the first call
            assert torch.cuda.mem_get_info()[0] == free_before

        got = oracle.untilize(c_new.cpu().numpy().view(np.uint16), Mt * 32, Nt * 32)
        ref = oracle.untilize(c_ref.cpu().numpy().view(np.uint16), Mt * 32, Nt * 32)
        assert np.array_equal(got, ref), "same kernel, same inputs: bitwise equal"
        exp = oracle.matmul(a, b)
        if fused:
            exp = oracle.relu(oracle.bias_add(exp, bias))
        assert oracle.normalized_error(got, exp, Kt * 32, 1.0, 1.0) <= 1e-2
