"""ORACLE build recipe — test infrastructure only.

Builds
  oracle/liboracle.so          the CPU restatement (oracle/golden.cpp)
and, when the reference tree is present (it is read-only and is never
needed at run time),
  oracle/_ref/libref_golden.so the reference's own golden functions, compiled
                               from its test sources (oracle/ref/wrap_*.cpp)
  oracle/_ref/droptests/*      the reference's hot-path tests compiled
                               unchanged against libtt_foil (oracle/ref/
                               droptests.txt), run by tests/test_dropin.py
                               on a GPU.

The golden library links oracle/ref/runtime_stub.cpp for the device-API
symbols that the included test files refer to, never the product libraries.

Usage: python oracle/build.py [--reference /path/to/reference]
The reference root comes from --reference, else from the TT_FOIL_REFERENCE
environment variable; without either, only liboracle.so is built.
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
REF_OUT = os.path.join(HERE, "_ref")
CXX = shutil.which("g++") or "g++"

# Golden wrappers: (tag, test source, kind, defines).  kind: 1 matmul,
# 2 conv_3x3, 3 conv_3x3_s2, 4 conv_1x1 (see oracle/ref/wrap_golden.cpp).
GOLDEN_WRAPPERS = [
    ("mnk_2_4_2", "test_matmul_mnk.cpp", 1, {"MM_MT": 2, "MM_KT": 4, "MM_NT": 2}),
    ("mnk_8_8_8", "test_matmul_mnk.cpp", 1, {"MM_MT": 8, "MM_KT": 8, "MM_NT": 8}),
    ("mnk_3_5_2", "test_matmul_mnk.cpp", 1, {"MM_MT": 3, "MM_KT": 5, "MM_NT": 2}),
    ("conv3_1_9_2", "test_conv_3x3.cpp", 2, {"MM_MT": 1, "MM_KT": 9, "MM_NT": 2}),
    ("conv3_2_18_14", "test_conv_3x3.cpp", 2, {"MM_MT": 2, "MM_KT": 18, "MM_NT": 14}),
    ("conv3s2_1_9_2", "test_conv_3x3_s2.cpp", 3, {"MM_MT": 1, "MM_KT": 9, "MM_NT": 2}),
    ("conv3s2_4_18_8", "test_conv_3x3_s2.cpp", 3, {"MM_MT": 4, "MM_KT": 18, "MM_NT": 8}),
    ("conv1_2_2_2", "test_conv_1x1.cpp", 4, {"MM_MT": 2, "MM_KT": 2, "MM_NT": 2}),
    ("conv1_8_4_16", "test_conv_1x1.cpp", 4, {"MM_MT": 8, "MM_KT": 4, "MM_NT": 16}),
    # one 32-row block / one 32 x 32 tile (K = 8192) of the 8192^3 GEMM: the
    # CPU baselines of bench.py
    ("mnk_1_256_256", "test_matmul_mnk.cpp", 1, {"MM_MT": 1, "MM_KT": 256, "MM_NT": 256}),
    ("mnk_1_256_1", "test_matmul_mnk.cpp", 1, {"MM_MT": 1, "MM_KT": 256, "MM_NT": 1}),
]


def run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise SystemExit(f"oracle build failed: {cmd[-1]}")


def newer(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs if os.path.exists(s))


def build_oracle():
    src = os.path.join(HERE, "golden.cpp")
    out = os.path.join(HERE, "liboracle.so")
    if newer(out, [src]):
        run([CXX, "-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", src, "-o", out])
    return out


def read_droptests():
    rows = []
    with open(os.path.join(HERE, "ref", "droptests.txt")) as f:
        for line in f:
            line = line.strip()
            if not line or line.startswith("#"):
                continue
            parts = line.split()
            rows.append((parts[0], parts[1], parts[2], parts[3:]))
    return rows


def build_reference(ref_root):
    tests_dir = os.path.join(ref_root, "tests")
    if not os.path.isdir(tests_dir):
        print(f"oracle: reference tree not found at {ref_root}; skipping oracle/_ref")
        return False
    os.makedirs(os.path.join(REF_OUT, "droptests"), exist_ok=True)
    inc = ["-I", os.path.join(REPO, "include"), "-I", os.path.join(REPO, "include", "tt_foil"),
           "-I", tests_dir]
    libdir = os.path.join(REPO, "tt-foil_b200", "lib")
    if not os.path.exists(os.path.join(libdir, "libtt_foil.so")):
        raise SystemExit("oracle: build tt-foil_b200 (make -C tt-foil_b200) before oracle/_ref")
    link = ["-L", libdir, "-ltt_foil", "-lfoil"]

    # 1. Golden wrappers -> one shared library, linked with the throwing
    #    device-API stub (no product library is mapped by it).
    objs = []
    stub = os.path.join(HERE, "ref", "runtime_stub.cpp")
    obj = os.path.join(REF_OUT, "runtime_stub.o")
    if newer(obj, [stub]):
        run([CXX, "-O2", "-std=c++20", "-fPIC", "-c", stub, "-o", obj] + inc)
    objs.append(obj)
    tu = os.path.join(HERE, "ref", "wrap_tile_utils.cpp")
    obj = os.path.join(REF_OUT, "wrap_tile_utils.o")
    if newer(obj, [tu]):
        run([CXX, "-O2", "-std=c++20", "-fPIC", "-c", tu, "-o", obj] + inc)
    objs.append(obj)
    wrap = os.path.join(HERE, "ref", "wrap_golden.cpp")
    for tag, test, kind, defs in GOLDEN_WRAPPERS:
        obj = os.path.join(REF_OUT, f"wrap_{tag}.o")
        src = os.path.join(tests_dir, test)
        if newer(obj, [wrap, src]):
            d = [f"-D{k}={v}" for k, v in defs.items()]
            run([CXX, "-O2", "-std=c++20", "-fPIC", "-c", wrap, "-o", obj,
                 f"-DREF_TEST={src}", f"-DREF_TAG={tag}", f"-DREF_KIND={kind}"] + d + inc)
        objs.append(obj)
    lib = os.path.join(REF_OUT, "libref_golden.so")
    if newer(lib, objs + [os.path.abspath(__file__)]):
        run([CXX, "-shared", "-Wl,--no-undefined", "-o", lib] + objs)

    # 2. Drop-in test binaries.
    rpath = "-Wl,-rpath,$ORIGIN/../../../tt-foil_b200/lib"
    for name, src, _prog, defs in read_droptests():
        out = os.path.join(REF_OUT, "droptests", name)
        s = os.path.join(tests_dir, src)
        if newer(out, [s, os.path.join(libdir, "libtt_foil.so")]):
            run([CXX, "-O2", "-std=c++20", s, "-o", out] + [f"-D{d}" for d in defs] + inc + link +
                [rpath])
    return True


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TT_FOIL_REFERENCE"))
    args = ap.parse_args()
    build_oracle()
    if args.reference:
        build_reference(args.reference)
    else:
        print("oracle: no reference tree given (--reference or TT_FOIL_REFERENCE); "
              "skipping oracle/_ref")


if __name__ == "__main__":
    main()
