"""Write the program-descriptor files that stand in for tt-foil's kernel ELFs.

tt-foil tests name their device binaries by convention
(``<kernel_dir>/reader.brisc.elf``, ``writer.ncrisc.elf``,
``compute.trisc{0,1,2}.elf``; the mcast example uses
``reader_producer.brisc.elf`` / ``reader_consumer.brisc.elf``; the scalar
examples use ``add_brisc.elf`` / ``add_ncrisc.elf`` and ``producer.elf`` /
``consumer.elf``) and
``load_kernel`` fails when a file is missing (reference src/kernel.cpp:42-45).
On the B200 there is no per-RISC ELF: each file is a small text descriptor
naming the program and the role, and ``load_kernel`` maps the bundle to the
CUDA kernel that implements the program.

Usage: python make_programs.py [out_dir]   (default: this directory)
One sub-directory per example, laid out like the reference's
``examples/<name>/prebuilt/``.
"""
import os
import sys

MAGIC = "TTFOIL-B200-PROGRAM 1"

# Every example on the accelerated path (reference examples/*/build_kernels.sh).
PROGRAMS = [
    "tile_copy", "matmul_1tile", "matmul_kt", "matmul_mnk", "matmul_dram",
    "matmul_2core", "matmul_2x2", "matmul_4x2", "matmul_2core_mcast",
    "conv_1x1", "conv_3x3", "conv_3x3_2core", "conv_3x3_s2",
    "relu", "add_tiles", "bias_add",
]

# The scalar dispatch examples (examples/add_two_numbers, examples/
# noc_passthrough): one BRISC (or NCRISC) binary each, named as there.
SCALAR_PROGRAMS = {
    "add_two_numbers": {
        "add_brisc.elf": ("reader", ""),
        "add_ncrisc.elf": ("writer", ""),
    },
    "noc_passthrough": {
        "producer.elf": ("reader", "producer"),
        "consumer.elf": ("reader", "consumer"),
    },
}


def descriptor(program, role, variant=""):
    lines = [MAGIC, f"program={program}", f"role={role}"]
    if variant:
        lines.append(f"variant={variant}")
    return "\n".join(lines) + "\n"


def write_file(path, text):
    if not os.path.exists(path) or open(path).read() != text:
        with open(path, "w") as f:
            f.write(text)


def write_all(out_dir):
    for prog, files in SCALAR_PROGRAMS.items():
        d = os.path.join(out_dir, prog)
        os.makedirs(d, exist_ok=True)
        for name, (role, variant) in files.items():
            write_file(os.path.join(d, name), descriptor(prog, role, variant))
    for prog in PROGRAMS:
        d = os.path.join(out_dir, prog)
        os.makedirs(d, exist_ok=True)
        files = {
            "writer.ncrisc.elf": descriptor(prog, "writer"),
            "compute.trisc0.elf": descriptor(prog, "compute"),
            "compute.trisc1.elf": descriptor(prog, "compute"),
            "compute.trisc2.elf": descriptor(prog, "compute"),
        }
        if prog == "matmul_2core_mcast":
            files["reader_producer.brisc.elf"] = descriptor(prog, "reader", "producer")
            files["reader_consumer.brisc.elf"] = descriptor(prog, "reader", "consumer")
        else:
            files["reader.brisc.elf"] = descriptor(prog, "reader")
        for name, text in files.items():
            write_file(os.path.join(d, name), text)


if __name__ == "__main__":
    write_all(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
