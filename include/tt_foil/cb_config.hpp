// Circular-buffer configuration, B200 edition.
//
// Source-compatible with tt-foil's src/cb_config.hpp (which the reference's
// tests include directly with -I src).  On the B200 the CUDA kernels stage
// tiles in shared memory, so register_cbs only validates the descriptors
// (index < 32, no duplicates, ring inside the core's L1 arena) and records
// them on the kernel; it throws std::runtime_error on the same conditions as
// the reference.
#pragma once

#include <cstdint>
#include <span>

#include "tt_foil/runtime.hpp"

namespace tt::foil {

struct Device;
struct Kernel;

struct CbConfig {
    uint8_t  cb_index;   // 0..31
    uint64_t fifo_addr;  // L1 arena offset of the ring
    uint32_t fifo_size;  // ring bytes (num_pages * page_size)
    uint32_t num_pages;  // slots
    uint32_t page_size;  // bytes per slot
};

void register_cbs(
    Device& dev,
    Kernel& kernel,
    std::span<const CbConfig> cbs);

}  // namespace tt::foil
