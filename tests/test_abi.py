"""CPU checks of the drop-in boundary: the C-ABI library loads, exports every
function include/foil_c.h declares, and the C++ API library exports the
tt-foil API; program descriptors exist for every accelerated example; argument
validation that needs no GPU behaves like the reference (errors, not crashes).
"""
import ctypes
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "tt-foil_b200")
LIB = os.path.join(PKG, "lib", "libfoil.so")
CPPLIB = os.path.join(PKG, "lib", "libtt_foil.so")
HEADER = os.path.join(REPO, "include", "foil_c.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"FOIL_API\s+[\w\s\*]+?\b(foil_\w+)\s*\(", text)))


def declared_arg_counts():
    """Number of parameters of every FOIL_API function in the header."""
    text = open(HEADER).read()
    counts = {}
    for m in re.finditer(r"FOIL_API\s+[\w\s\*]+?\b(foil_\w+)\s*\(([^)]*)\)", text):
        args = m.group(2).strip()
        counts[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return counts


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_header_declares_the_boundary():
    fns = declared_functions()
    for name in ["foil_open_device", "foil_close_device", "foil_allocate_buffer", "foil_write_buffer",
                 "foil_read_buffer", "foil_load_kernel", "foil_set_runtime_args", "foil_register_cbs",
                 "foil_execute", "foil_make_noc_unicast_addr", "foil_make_noc_dram_addr",
                 "foil_matmul_tiles_dev", "foil_tilize_dev", "foil_untilize_dev"]:
        assert name in fns


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "build with: make -C tt-foil_b200"
    syms = exported(LIB)
    missing = [f for f in declared_functions() if f not in syms]
    assert not missing, missing


def test_library_loads_and_binding_matches_header():
    import ttfoil
    L = ttfoil.lib()
    for name in declared_functions():
        assert hasattr(L, name)
        assert name in ttfoil.SIGNATURES, f"ttfoil binding lacks {name}"
    assert b"sm_100a" in L.foil_version()


def test_binding_argument_counts_match_header():
    import ttfoil
    for name, n in declared_arg_counts().items():
        assert len(ttfoil.SIGNATURES[name][1]) == n, name


def test_cpp_api_exports_tt_foil_functions():
    out = subprocess.run(["nm", "-DC", "--defined-only", CPPLIB], capture_output=True, text=True,
                         check=True).stdout
    for fn in ["tt::foil::open_device(", "tt::foil::close_device(", "tt::foil::allocate_buffer(",
               "tt::foil::free_buffer(", "tt::foil::write_buffer(", "tt::foil::read_buffer(",
               "tt::foil::load_kernel(", "tt::foil::set_runtime_args(", "tt::foil::execute(",
               "tt::foil::make_noc_unicast_addr(", "tt::foil::make_noc_dram_addr(",
               "tt::foil::register_cbs("]:
        assert fn in out, fn


def test_program_descriptors_present():
    import ttfoil
    for prog in ["tile_copy", "matmul_1tile", "matmul_kt", "matmul_mnk", "matmul_dram",
                 "matmul_2core", "matmul_2x2", "matmul_4x2", "conv_1x1", "conv_3x3",
                 "conv_3x3_2core", "conv_3x3_s2", "relu", "add_tiles", "bias_add"]:
        d = os.path.join(ttfoil.PROGRAMS_DIR, prog)
        for f in ["reader.brisc.elf", "writer.ncrisc.elf", "compute.trisc0.elf",
                  "compute.trisc1.elf", "compute.trisc2.elf"]:
            text = open(os.path.join(d, f)).read()
            assert text.startswith("TTFOIL-B200-PROGRAM 1") and f"program={prog}" in text
    mc = os.path.join(ttfoil.PROGRAMS_DIR, "matmul_2core_mcast")
    assert "variant=producer" in open(os.path.join(mc, "reader_producer.brisc.elf")).read()
    assert "variant=consumer" in open(os.path.join(mc, "reader_consumer.brisc.elf")).read()
    # the scalar dispatch examples, under the reference's binary names
    add = os.path.join(ttfoil.PROGRAMS_DIR, "add_two_numbers")
    assert "role=reader" in open(os.path.join(add, "add_brisc.elf")).read()
    assert "role=writer" in open(os.path.join(add, "add_ncrisc.elf")).read()
    noc = os.path.join(ttfoil.PROGRAMS_DIR, "noc_passthrough")
    assert "variant=producer" in open(os.path.join(noc, "producer.elf")).read()
    assert "variant=consumer" in open(os.path.join(noc, "consumer.elf")).read()


def test_make_programs_reproduces_the_committed_descriptors(tmp_path):
    """programs/make_programs.py writes exactly the committed descriptor
    files, and every program directory a drop-in test uses exists."""
    import filecmp
    import subprocess
    import sys
    import ttfoil
    subprocess.run([sys.executable, os.path.join(ttfoil.PROGRAMS_DIR, "make_programs.py"), str(tmp_path)],
                   check=True)
    made = sorted(os.path.relpath(os.path.join(r, f), tmp_path) for r, _, fs in os.walk(tmp_path) for f in fs)
    assert made, "no descriptors written"
    for rel in made:
        assert filecmp.cmp(os.path.join(tmp_path, rel), os.path.join(ttfoil.PROGRAMS_DIR, rel), shallow=False), rel
    with open(os.path.join(REPO, "oracle", "ref", "droptests.txt")) as f:
        progs = {line.split()[2] for line in f if line.strip() and not line.startswith("#")}
    for prog in progs:
        assert os.path.isdir(os.path.join(ttfoil.PROGRAMS_DIR, prog)), prog


def test_validation_errors_without_gpu():
    """Argument checks that precede any CUDA call return errors, never crash."""
    import ttfoil
    L = ttfoil.lib()
    h = ctypes.c_void_p()
    rc = L.foil_open_device(0, b"", None, 0, ctypes.byref(h))
    assert rc == 1 and b"at least one" in L.foil_last_error()
    assert L.foil_tilize_dev(None, None, 33, 32, None) == 1
    assert b"multiples of 32" in L.foil_last_error()
    assert L.foil_tile_copy_dev(None, None, 17, None) == 1
    assert L.foil_add_tiles_dev(None, None, None, 7, None) == 1
    assert L.foil_relu_tiles_dev(None, None, 12, None) == 1
    assert L.foil_bias_add_tiles_dev(None, None, None, 32, 48, None) == 1
    # element-wise stages: misaligned pointers, partial overlap of the output
    # with an input, and an output over the bias band are rejected before
    # anything is launched (the addresses are never dereferenced)
    base = 1 << 40
    assert L.foil_relu_tiles_dev(base + 8, base + 4096, 8, None) == 1
    assert b"misaligned" in L.foil_last_error()
    assert L.foil_relu_tiles_dev(base, base + 16, 64, None) == 1
    assert b"partially overlaps" in L.foil_last_error()
    assert L.foil_add_tiles_dev(base, base + 4096, base + 4096 - 16, 64, None) == 1
    assert b"partially overlaps" in L.foil_last_error()
    assert L.foil_tile_copy_dev(base + 16, base, 64, None) == 1
    assert L.foil_bias_add_tiles_dev(base, base + (1 << 20) + 512, base + (1 << 20), 32, 64, None) == 1
    assert b"bias band" in L.foil_last_error()
    assert L.foil_matmul_tiles_dev(None, None, None, 70000, 1, 1, None, 0, None) == 1
    # GEMM with its own all-gather: peer-list checks precede any CUDA call
    peers = (ctypes.c_void_p * 8)(*([base] * 8))
    assert L.foil_matmul_tiles_gather_dev(None, None, None, peers, 8, 1, 1, 1, None, 0, None) == 1
    assert b"at most 7" in L.foil_last_error()
    assert L.foil_matmul_tiles_gather_dev(None, None, None, None, 2, 1, 1, 1, None, 0, None) == 1
    peers[1] = base + 8
    assert L.foil_matmul_tiles_gather_dev(None, None, None, peers, 2, 1, 1, 1, None, 0, None) == 1
    assert b"peer buffer" in L.foil_last_error()
    assert L.foil_peer_alloc(0, 0, None, None) == 1
    assert L.foil_matmul_tiles_host(0, None, None, None, 1, 1, 1, None, 0, 0) == 1
    assert b"null pointer" in L.foil_last_error()
    assert L.foil_matmul_tiles_host(0, None, None, None, 70000, 1, 1, None, 0, 0) == 1
    assert L.foil_conv2d_nhwc_host(0, None, None, None, None, 1, 4, 4, 16, 16, 3, 3, 1, 1, 0, 0) == 1
    # zero-sized work is a no-op
    assert L.foil_tile_copy_dev(None, None, 0, None) == 0
    assert L.foil_matmul_tiles_dev(None, None, None, 0, 4, 4, None, 0, None) == 0
    assert L.foil_matmul_tiles_host(0, None, None, None, 0, 4, 4, None, 0, 0) == 0


def test_host_logic_unit_binary(tmp_path):
    """tests/cpp/test_host_logic.cpp: allocators, address packing, descriptor
    parsing, CB validation and runtime-arg planning (no GPU)."""
    exe = tmp_path / "test_host_logic"
    subprocess.run(["g++", "-std=c++20", "-O1", "-I", os.path.join(REPO, "include"),
                    os.path.join(REPO, "tests", "cpp", "test_host_logic.cpp"),
                    os.path.join(PKG, "csrc", "host_logic.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout
