// tt-foil host API, B200 edition.
//
// Source-compatible with tt-foil's public header (include/tt_foil/runtime.hpp
// in the reference): the same namespace, types, free functions, default
// arguments and error behaviour (every failure throws std::runtime_error), so
// programs and tests written against tt-foil compile unchanged.  The
// implementation (tt-foil_b200/src/runtime.cpp) forwards every call to the
// C-ABI in include/foil_c.h, which runs the work as sm_100a CUDA kernels on
// an NVIDIA B200 instead of Tensix cores.
//
// Mapping of the reference's concepts:
//   * a logical core is a slot with its own emulated 1.5 MB L1 arena in HBM;
//     L1 addresses stay 32-bit offsets so they fit one runtime-arg word;
//   * DRAM is one growable HBM arena (CUDA virtual memory), 36-bit offsets;
//   * a "kernel" is the set of program-descriptor files the test names as
//     ELFs; execute() launches the CUDA kernel for that program.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <initializer_list>
#include <memory>
#include <span>
#include <string>
#include <vector>

namespace tt::foil {

struct Device;  // opaque
struct Kernel;  // opaque

// Logical core coordinate (same value semantics as the reference).
struct CoreCoord {
    uint32_t x{0};
    uint32_t y{0};
    bool operator==(const CoreCoord& o) const { return x == o.x && y == o.y; }
};

enum class BufferLocation {
    L1,    // the owning core's emulated L1 arena
    DRAM,  // the device DRAM arena
};

// A device allocation.  device_addr is what a kernel receives as a runtime
// argument (L1: 32-bit arena offset; DRAM: arena offset, wrap it with
// make_noc_dram_addr before passing it).
struct Buffer {
    BufferLocation location;
    uint64_t       device_addr{0};
    std::size_t    size_bytes{0};
    CoreCoord      core;  // owning core of an L1 buffer
};

// Open CUDA device `pcie_device_index` and create one L1 arena per listed
// core.  firmware_dir is accepted for compatibility and ignored.
// Throws std::runtime_error on failure.
std::shared_ptr<Device> open_device(
    int pcie_device_index = 0,
    const std::string& firmware_dir = "",
    std::vector<CoreCoord> cores = {{0, 0}});

// Release the device now; the shared_ptr deleter does the same otherwise.
void close_device(std::shared_ptr<Device> device);

// Bump-allocate in a core's L1 arena or in the DRAM arena.
// Throws std::runtime_error when the arena is exhausted or size is 0.
std::shared_ptr<Buffer> allocate_buffer(
    Device& device,
    BufferLocation loc,
    std::size_t size_bytes,
    CoreCoord logical_core = {});

// Bump allocator: nothing is reclaimed until the device is closed.
void free_buffer(std::shared_ptr<Buffer> buffer);

// Blocking host -> device copy.
void write_buffer(Device& device, Buffer& buf, const void* src, std::size_t bytes);

// Blocking device -> host copy.
void read_buffer(Device& device, Buffer& buf, void* dst, std::size_t bytes);

// One program binary of a kernel bundle.
struct RiscBinary {
    enum class RiscId {
        BRISC  = 0,  // reader role
        NCRISC = 1,  // writer role
        TRISC0 = 2,  // compute (unpack)
        TRISC1 = 3,  // compute (math)
        TRISC2 = 4,  // compute (pack)
    };
    RiscId risc;
    std::string elf_path;  // path of a program-descriptor file
};

// Read the program descriptors and bind the kernel to logical_core.
std::shared_ptr<Kernel> load_kernel(
    Device& device,
    std::span<const RiscBinary> binaries,
    CoreCoord logical_core);

// Runtime arguments of one RISC (at most 64 words).
void set_runtime_args(
    Device& device,
    Kernel& kernel,
    RiscBinary::RiscId risc,
    std::span<const uint32_t> args);

// Blocking execution of one kernel (5 s timeout).
void execute(Device& device, Kernel& kernel);

// Blocking execution of several kernels: all are launched before any wait.
void execute(Device& device, std::initializer_list<Kernel*> kernels);

// 64-bit address of an L1 location on another core:
// bits [47:42] = y, [41:36] = x, [35:0] = L1 offset.
uint64_t make_noc_unicast_addr(
    Device& device,
    CoreCoord logical_dst,
    uint64_t local_l1_addr);

// 64-bit address of a DRAM-arena offset (split lo/hi into two runtime args).
uint64_t make_noc_dram_addr(Device& device, uint64_t dram_offset);

}  // namespace tt::foil
