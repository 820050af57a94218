"""The tt-foil runtime boundary (C-ABI, include/foil_c.h) on the GPU: every
program of the accelerated path driven exactly as the reference tests drive
it (open_device, allocate_buffer, write_buffer, load_kernel, register_cbs,
set_runtime_args, execute, read_buffer), compared with the oracle, plus the
reference's error behaviour.
"""
import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu

TILE = 2048


@pytest.fixture(scope="module")
def tf():
    import ttfoil
    ttfoil.lib()
    return ttfoil


def u16(a):
    return np.ascontiguousarray(a, dtype=np.uint16)


def test_dram_roundtrip_and_alignment(tf):
    with tf.Device(0) as d:
        b1 = d.allocate(tf.LOC_DRAM, 100)
        b2 = d.allocate(tf.LOC_DRAM, 32 * 1024)
        assert b2.device_addr % 32 == 0 and b2.device_addr >= b1.device_addr + 100
        src = (np.arange(8192, dtype=np.uint32) * 0x10001).astype(np.uint32)
        d.write_array(b2, src)
        assert np.array_equal(d.read_array(b2, np.uint32, 8192), src)
        l1 = d.allocate(tf.LOC_L1, 10)
        l2 = d.allocate(tf.LOC_L1, 10)
        assert l2.device_addr % 16 == 0 and l2.device_addr >= l1.device_addr + 10


def test_dram_grows_past_first_chunk(tf):
    with tf.Device(0) as d:
        big = d.allocate(tf.LOC_DRAM, 300 << 20)
        data = np.random.default_rng(0).integers(0, 2**32, (300 << 20) // 4, dtype=np.uint32)
        d.write_array(big, data)
        assert np.array_equal(d.read_array(big, np.uint32, data.size), data)


def test_tile_copy_program(tf):
    with tf.Device(0) as d:
        src = d.allocate(tf.LOC_L1, TILE)
        dst = d.allocate(tf.LOC_L1, TILE)
        cb_in = d.allocate(tf.LOC_L1, TILE)
        cb_out = d.allocate(tf.LOC_L1, TILE)
        data = (np.arange(1024, dtype=np.uint32) ^ 0xA5A5).astype(np.uint16)
        d.write_array(src, data)
        k = d.load_program("tile_copy")
        d.register_cbs(k, [(0, cb_in.device_addr, TILE, 1, TILE), (16, cb_out.device_addr, TILE, 1, TILE)])
        d.set_runtime_args(k, tf.BRISC, [src.device_addr])
        d.set_runtime_args(k, tf.NCRISC, [dst.device_addr])
        d.execute(k)
        assert np.array_equal(d.read_array(dst, np.uint16, 1024), data)


@pytest.mark.parametrize("prog", ["relu", "add_tiles", "bias_add"])
def test_eltwise_programs(tf, prog):
    x = oracle.rand_bf16((32, 32), 1, -4, 4)
    y = oracle.rand_bf16((32, 32), 2, -1, 1)
    if prog == "relu":
        exp = oracle.relu(x)
    elif prog == "add_tiles":
        exp = oracle.add(x, y)
    else:
        y[1:] = 0  # bias tile: row 0 populated
        exp = oracle.bias_add(x, y[0])
    with tf.Device(0) as d:
        bx = d.allocate(tf.LOC_L1, TILE)
        by = d.allocate(tf.LOC_L1, TILE)
        bo = d.allocate(tf.LOC_L1, TILE)
        d.write_array(bx, oracle.tilize(x))
        d.write_array(by, oracle.tilize(y))
        k = d.load_program(prog)
        args = [bx.device_addr] if prog == "relu" else [bx.device_addr, by.device_addr]
        d.set_runtime_args(k, tf.BRISC, args)
        d.set_runtime_args(k, tf.NCRISC, [bo.device_addr])
        d.execute(k)
        got = oracle.untilize(d.read_array(bo, np.uint16, 1024), 32, 32)
    assert np.array_equal(got, exp)


def gemm_ok(got, exp, K):
    assert oracle.normalized_error(got, exp, K, 1.0, 1.0) <= 1e-2
    assert oracle.compare(got, exp)[0] == 0


@pytest.mark.parametrize("Mt,Kt,Nt", [(2, 4, 2), (8, 8, 8), (3, 11, 5)])
def test_matmul_mnk_program(tf, Mt, Kt, Nt):
    a = oracle.rand_bf16((Mt * 32, Kt * 32), 3)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), 4)
    with tf.Device(0) as d:
        ba = d.allocate(tf.LOC_L1, Mt * Kt * TILE)
        bb = d.allocate(tf.LOC_L1, Kt * Nt * TILE)
        bc = d.allocate(tf.LOC_L1, Mt * Nt * TILE)
        d.write_array(ba, oracle.tilize(a))
        d.write_array(bb, oracle.tilize(b))
        k = d.load_program("matmul_mnk")
        d.set_runtime_args(k, tf.BRISC, [ba.device_addr, bb.device_addr, Mt, Kt, Nt])
        d.set_runtime_args(k, tf.NCRISC, [bc.device_addr, Mt * Nt])
        d.execute(k)
        got = oracle.untilize(d.read_array(bc, np.uint16, Mt * Nt * 1024), Mt * 32, Nt * 32)
    gemm_ok(got, oracle.matmul(a, b), Kt * 32)


def test_matmul_kt_and_1tile_programs(tf):
    Kt = 6
    a = oracle.rand_bf16((32, Kt * 32), 5)
    b = oracle.rand_bf16((Kt * 32, 32), 6)
    with tf.Device(0) as d:
        ba = d.allocate(tf.LOC_L1, Kt * TILE)
        bb = d.allocate(tf.LOC_L1, Kt * TILE)
        bc = d.allocate(tf.LOC_L1, TILE)
        d.write_array(ba, oracle.tilize(a))
        d.write_array(bb, oracle.tilize(b))
        k = d.load_program("matmul_kt")
        d.set_runtime_args(k, tf.BRISC, [ba.device_addr, bb.device_addr, Kt])
        d.set_runtime_args(k, tf.NCRISC, [bc.device_addr])
        d.execute(k)
        got = oracle.untilize(d.read_array(bc, np.uint16, 1024), 32, 32)
        gemm_ok(got, oracle.matmul(a, b), Kt * 32)
        k1 = d.load_program("matmul_1tile")
        d.set_runtime_args(k1, tf.BRISC, [ba.device_addr, bb.device_addr])
        d.set_runtime_args(k1, tf.NCRISC, [bc.device_addr])
        d.execute(k1)
        got1 = oracle.untilize(d.read_array(bc, np.uint16, 1024), 32, 32)
        gemm_ok(got1, oracle.matmul(a[:, :32], b[:32]), 32)


def test_matmul_dram_two_cores_one_execute(tf):
    """matmul_2core schedule: M split across two cores, one execute call."""
    Mt_pc, Kt, Nt = 3, 5, 4
    a = oracle.rand_bf16((2 * Mt_pc * 32, Kt * 32), 7)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), 8)
    with tf.Device(0, cores=[(0, 0), (0, 1)]) as d:
        ba = d.allocate(tf.LOC_DRAM, 2 * Mt_pc * Kt * TILE)
        bb = d.allocate(tf.LOC_DRAM, Kt * Nt * TILE)
        bc = d.allocate(tf.LOC_DRAM, 2 * Mt_pc * Nt * TILE)
        d.write_array(ba, oracle.tilize(a))
        d.write_array(bb, oracle.tilize(b))
        ks = []
        for cid, core in enumerate([(0, 0), (0, 1)]):
            k = d.load_program("matmul_2core", core)
            an = d.noc_dram_addr(ba.device_addr + cid * Mt_pc * Kt * TILE)
            bn = d.noc_dram_addr(bb.device_addr)
            cn = d.noc_dram_addr(bc.device_addr + cid * Mt_pc * Nt * TILE)
            d.set_runtime_args(k, tf.BRISC, [tf.lo(an), tf.hi(an), tf.lo(bn), tf.hi(bn), Mt_pc, Kt, Nt])
            d.set_runtime_args(k, tf.NCRISC, [tf.lo(cn), tf.hi(cn), Mt_pc * Nt])
            ks.append(k)
        d.execute(ks)
        got = oracle.untilize(d.read_array(bc, np.uint16, 2 * Mt_pc * Nt * 1024), 2 * Mt_pc * 32, Nt * 32)
    gemm_ok(got, oracle.matmul(a, b), Kt * 32)


def mcast_setup(tf, d, Mt, Kt, Nt, a, b, with_producer=True):
    cp, cc = (0, 0), (0, 1)
    ba = d.allocate(tf.LOC_DRAM, 2 * Mt * Kt * TILE)
    bb = d.allocate(tf.LOC_DRAM, Kt * Nt * TILE)
    bo = d.allocate(tf.LOC_DRAM, 2 * Mt * Nt * TILE)
    d.write_array(ba, oracle.tilize(a))
    d.write_array(bb, oracle.tilize(b))
    stage_p = d.allocate(tf.LOC_L1, Kt * Nt * TILE, cp)
    flag_src = d.allocate(tf.LOC_L1, 4, cp)
    ckpt = d.allocate(tf.LOC_L1, 64, cp)
    d.write_array(flag_src, np.array([1], dtype=np.uint32))
    stage_c = d.allocate(tf.LOC_L1, Kt * Nt * TILE, cc)
    flag_c = d.allocate(tf.LOC_L1, 4, cc)
    d.write_array(flag_c, np.array([0], dtype=np.uint32))
    kp = d.load_program("matmul_2core_mcast", cp, reader="reader_producer.brisc.elf")
    kc = d.load_program("matmul_2core_mcast", cc, reader="reader_consumer.brisc.elf")
    a_p, a_c = (d.noc_dram_addr(ba.device_addr + i * Mt * Kt * TILE) for i in (0, 1))
    o_p, o_c = (d.noc_dram_addr(bo.device_addr + i * Mt * Nt * TILE) for i in (0, 1))
    b_n = d.noc_dram_addr(bb.device_addr)
    st_n = d.noc_unicast_addr(cc, stage_c.device_addr)
    fl_n = d.noc_unicast_addr(cc, flag_c.device_addr)
    lo, hi = tf.lo, tf.hi
    d.set_runtime_args(kp, tf.BRISC, [lo(a_p), hi(a_p), lo(b_n), hi(b_n), lo(st_n), hi(st_n), lo(fl_n),
                                      hi(fl_n), stage_p.device_addr, flag_src.device_addr, Mt, Kt, Nt,
                                      ckpt.device_addr])
    d.set_runtime_args(kp, tf.NCRISC, [lo(o_p), hi(o_p), Mt * Nt])
    d.set_runtime_args(kc, tf.BRISC, [lo(a_c), hi(a_c), stage_c.device_addr, flag_c.device_addr, Mt, Kt, Nt])
    d.set_runtime_args(kc, tf.NCRISC, [lo(o_c), hi(o_c), Mt * Nt])
    return kp, kc, bo, stage_c, flag_c


@pytest.mark.parametrize("consumer_first", [False, True])
def test_matmul_2core_mcast_program(tf, consumer_first):
    """Producer and consumer run as one launch (one CTA per core, resident
    together): the consumer's device-side wait sees the flag the producer
    sets after forwarding B, in either order of the execute list."""
    Mt, Kt, Nt = 2, 6, 3
    a = oracle.rand_bf16((2 * Mt * 32, Kt * 32), 9)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), 10)
    with tf.Device(0, cores=[(0, 0), (0, 1)]) as d:
        kp, kc, bo, stage_c, flag_c = mcast_setup(tf, d, Mt, Kt, Nt, a, b)
        launches = tf.launch_count()
        d.execute([kc, kp] if consumer_first else [kp, kc])
        assert tf.launch_count() == launches + 1, "both core programs in one launch"
        got = oracle.untilize(d.read_array(bo, np.uint16, 2 * Mt * Nt * 1024), 2 * Mt * 32, Nt * 32)
        # B was forwarded into the consumer's L1 and its flag set.
        assert np.array_equal(d.read_array(stage_c, np.uint16, Kt * Nt * 1024), oracle.tilize(b))
        assert d.read_array(flag_c, np.uint32, 1)[0] == 1
    gemm_ok(got, oracle.matmul(a, b), Kt * 32)


def test_mcast_consumer_alone_times_out(tf):
    """A consumer whose ready flag nobody sets ends in the reference's timeout
    error (reader_consumer.cpp:40-44 spins until the host's deadline): its
    device-side wait runs out at the execute's deadline and the kernel
    returns; the device then runs the pair normally."""
    Mt, Kt, Nt = 1, 2, 2
    a = oracle.rand_bf16((2 * Mt * 32, Kt * 32), 11)
    b = oracle.rand_bf16((Kt * 32, Nt * 32), 12)
    with tf.Device(0, cores=[(0, 0), (0, 1)]) as d:
        kp, kc, *_ = mcast_setup(tf, d, Mt, Kt, Nt, a, b)
        launches = tf.launch_count()
        with pytest.raises(tf.FoilError) as e:
            d.execute([kc], timeout_ms=300)
        assert e.value.status == 5 and "timeout" in str(e.value) and "(0,1)" in str(e.value)
        assert tf.launch_count() == launches + 1, "the consumer was launched and its wait ran out"
        d.execute([kp, kc])  # the context is still usable


def test_error_behaviour(tf):
    with tf.Device(0) as d:
        with pytest.raises(tf.FoilError, match="size must be > 0"):
            d.allocate(tf.LOC_DRAM, 0)
        with pytest.raises(tf.FoilError, match="L1 out of memory"):
            d.allocate(tf.LOC_L1, 2 << 20)
        with pytest.raises(tf.FoilError, match="not opened"):
            d.allocate(tf.LOC_L1, 16, (3, 3))
        buf = d.allocate(tf.LOC_L1, 64)
        with pytest.raises(tf.FoilError, match="exceeds allocation"):
            d.write(buf, np.zeros(128, np.uint8).ctypes.data, 128)
        with pytest.raises(tf.FoilError, match="ELF not found"):
            d.load_kernel([(tf.BRISC, "/nonexistent/reader.brisc.elf")])
        k = d.load_program("relu")
        with pytest.raises(tf.FoilError, match="too many runtime args"):
            d.set_runtime_args(k, tf.BRISC, list(range(65)))
        with pytest.raises(tf.FoilError, match="cb_index must be < 32"):
            d.register_cbs(k, [(32, buf.device_addr, 64, 1, 64)])
        with pytest.raises(tf.FoilError, match="listed twice"):
            d.register_cbs(k, [(0, buf.device_addr, 64, 1, 64), (0, buf.device_addr, 64, 1, 64)])
        with pytest.raises(tf.FoilError, match="needs 1 runtime args"):
            d.execute(k)
        # An address outside allocated L1 is refused before any launch.
        d.set_runtime_args(k, tf.BRISC, [0x100000])
        d.set_runtime_args(k, tf.NCRISC, [buf.device_addr])
        with pytest.raises(tf.FoilError, match="outside allocated L1"):
            d.execute(k)
        with pytest.raises(tf.FoilError, match="no kernels"):
            d.execute([])


def scalar_bins(tf, program, *names):
    d = os.path.join(tf.PROGRAMS_DIR, program)
    risc = {"add_brisc.elf": tf.BRISC, "add_ncrisc.elf": tf.NCRISC, "producer.elf": tf.BRISC,
            "consumer.elf": tf.BRISC}
    return [(risc[n], os.path.join(d, n)) for n in names]


def test_add_two_numbers_on_eight_cores(tf):
    """examples/add_two_numbers on 8 cores in one execute: BRISC writes
    a + b, NCRISC a * b (wrapping u32, like the RISC-V cores), each core
    with its own operands; all cores are one launch."""
    cores = [(x, y) for x in range(2) for y in range(4)]
    rng = np.random.default_rng(21)
    vals = rng.integers(0, 2**32, size=(len(cores), 2), dtype=np.uint64).astype(np.uint32)
    vals[0] = [0xFFFFFFFF, 2]  # both results wrap
    with tf.Device(0, cores=cores) as d:
        ks, outs = [], []
        for (x, y), (a, b) in zip(cores, vals):
            ba, bb, bs, bp = (d.allocate(tf.LOC_L1, 4, (x, y)) for _ in range(4))
            d.write_array(ba, np.array([a], np.uint32))
            d.write_array(bb, np.array([b], np.uint32))
            d.write_array(bs, np.zeros(1, np.uint32))
            d.write_array(bp, np.zeros(1, np.uint32))
            k = d.load_kernel(scalar_bins(tf, "add_two_numbers", "add_brisc.elf", "add_ncrisc.elf"), (x, y))
            d.set_runtime_args(k, tf.BRISC, [ba.device_addr, bb.device_addr, bs.device_addr])
            d.set_runtime_args(k, tf.NCRISC, [ba.device_addr, bb.device_addr, bp.device_addr])
            ks.append(k)
            outs.append((bs, bp))
        launches = tf.launch_count()
        d.execute(ks)
        assert tf.launch_count() == launches + 1
        for (bs, bp), (a, b) in zip(outs, vals):
            assert d.read_array(bs, np.uint32, 1)[0] == np.uint32((int(a) + int(b)) & 0xFFFFFFFF)
            assert d.read_array(bp, np.uint32, 1)[0] == np.uint32((int(a) * int(b)) & 0xFFFFFFFF)


def noc_setup(tf, d, a, b):
    cp, cc = (0, 0), (0, 1)
    ba, bb, sum_s, flag_s = (d.allocate(tf.LOC_L1, 4, cp) for _ in range(4))
    sum_d, flag_d, res = (d.allocate(tf.LOC_L1, 4, cc) for _ in range(3))
    d.write_array(ba, np.array([a], np.uint32))
    d.write_array(bb, np.array([b], np.uint32))
    for buf in (sum_s, flag_s, sum_d, flag_d, res):
        d.write_array(buf, np.zeros(1, np.uint32))
    kp = d.load_kernel(scalar_bins(tf, "noc_passthrough", "producer.elf"), cp)
    kc = d.load_kernel(scalar_bins(tf, "noc_passthrough", "consumer.elf"), cc)
    sn = d.noc_unicast_addr(cc, sum_d.device_addr)
    fn = d.noc_unicast_addr(cc, flag_d.device_addr)
    d.set_runtime_args(kp, tf.BRISC, [ba.device_addr, bb.device_addr, sum_s.device_addr, tf.lo(sn), tf.hi(sn),
                                      flag_s.device_addr, tf.lo(fn), tf.hi(fn)])
    d.set_runtime_args(kc, tf.BRISC, [flag_d.device_addr, sum_d.device_addr, res.device_addr])
    return kp, kc, dict(sum_s=sum_s, flag_s=flag_s, sum_d=sum_d, flag_d=flag_d, res=res)


@pytest.mark.parametrize("consumer_first", [False, True])
def test_noc_passthrough_program(tf, consumer_first):
    """examples/noc_passthrough: the producer sends a + b to the consumer's
    L1 and then the 0xCAFEBABE sentinel; the consumer waits (bounded, on the
    device) for the sentinel and writes 2 (a + b).  One launch, either order."""
    a, b = 0x9E3779B9, 0x7F4A7C15  # the sum wraps
    with tf.Device(0, cores=[(0, 0), (0, 1)]) as d:
        kp, kc, buf = noc_setup(tf, d, a, b)
        launches = tf.launch_count()
        d.execute([kc, kp] if consumer_first else [kp, kc])
        assert tf.launch_count() == launches + 1
        s = (a + b) & 0xFFFFFFFF
        rd = lambda n: int(d.read_array(buf[n], np.uint32, 1)[0])
        assert rd("res") == (2 * s) & 0xFFFFFFFF
        assert rd("sum_s") == s and rd("sum_d") == s
        assert rd("flag_s") == 0xCAFEBABE and rd("flag_d") == 0xCAFEBABE


def test_noc_consumer_alone_times_out(tf):
    """The consumer without its producer: the device-side wait for the
    sentinel runs out at the execute's deadline, the execute fails with the
    timeout status naming the core, the result stays unwritten, and the pair
    then runs normally."""
    with tf.Device(0, cores=[(0, 0), (0, 1)]) as d:
        kp, kc, buf = noc_setup(tf, d, 5, 6)
        with pytest.raises(tf.FoilError) as e:
            d.execute([kc], timeout_ms=300)
        assert e.value.status == 5 and "(0,1)" in str(e.value)
        assert d.read_array(buf["res"], np.uint32, 1)[0] == 0
        d.execute([kp, kc])
        assert d.read_array(buf["res"], np.uint32, 1)[0] == 22


def test_unsupported_program_rejected(tf, tmp_path):
    p = tmp_path / "reader.brisc.elf"
    p.write_text("TTFOIL-B200-PROGRAM 1\nprogram=erisc_ping\nrole=reader\n")
    with tf.Device(0) as d:
        with pytest.raises(tf.FoilError) as e:
            d.load_kernel([(tf.BRISC, str(p))])
        assert e.value.status == 6


def test_open_device_errors(tf):
    with pytest.raises(tf.FoilError, match="at least one"):
        tf.Device(0, cores=[])
    with pytest.raises(tf.FoilError, match="no CUDA device"):
        tf.Device(4096)
