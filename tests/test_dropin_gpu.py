"""Drop-in runs: the reference's own tests (tests/test_*.cpp of tt-foil) for
the hot path and for the scalar dispatch examples (add_two_numbers on one,
two and BRISC + NCRISC, noc_passthrough producer / consumer), compiled
unchanged against libtt_foil by oracle/build.py, executed on the GPU.  Each
binary builds its inputs, computes its own CPU golden and compares with the
device output using its own tolerance (bitwise for tile_copy /
dram_roundtrip, exact for relu and the u32 examples, max(0.05, 1%) for
matmul / conv, 0.05 abs for add / bias), printing PASS and returning 0.
"""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROP = os.path.join(REPO, "oracle", "_ref", "droptests")
LIST = os.path.join(REPO, "oracle", "ref", "droptests.txt")
PROGRAMS = os.path.join(REPO, "tt-foil_b200", "programs")


def cases():
    rows = []
    with open(LIST) as f:
        for line in f:
            line = line.strip()
            if line and not line.startswith("#"):
                p = line.split()
                rows.append((p[0], p[2]))
    return rows


@pytest.mark.gpu
@pytest.mark.parametrize("name,program", cases())
def test_reference_test_passes(name, program):
    exe = os.path.join(DROP, name)
    assert os.path.exists(exe), f"{exe} missing: build with python oracle/build.py"
    env = dict(os.environ, TT_FOIL_KERNEL_DIR=os.path.join(PROGRAMS, program), TT_FOIL_DEVICE="0")
    r = subprocess.run([exe], env=env, capture_output=True, text=True, timeout=120)
    out = r.stdout + r.stderr
    assert r.returncode == 0 and "PASS" in out, out
