// tt-foil C++ API (include/tt_foil/runtime.hpp, include/tt_foil/cb_config.hpp)
// over the C-ABI of libfoil (include/foil_c.h).
//
// Mirrors the reference's delegation layer (src/runtime_impl.cpp:23-131):
// shared_ptr ownership with custom deleters, and every failure surfaces as
// std::runtime_error carrying the C layer's message.
#include "tt_foil/runtime.hpp"

#include <stdexcept>
#include <string>
#include <vector>

#include "foil_c.h"
#include "tt_foil/cb_config.hpp"

namespace tt::foil {

struct Device {
    foil_device* handle{nullptr};
};

struct Kernel {
    foil_kernel* handle{nullptr};
};

namespace {

void check(int status) {
    if (status != FOIL_OK) throw std::runtime_error(foil_last_error());
}

foil_buffer to_c(const Buffer& b) {
    foil_buffer c = {};
    c.location = b.location == BufferLocation::L1 ? FOIL_LOC_L1 : FOIL_LOC_DRAM;
    c.device_addr = b.device_addr;
    c.size_bytes = b.size_bytes;
    c.core = foil_core{b.core.x, b.core.y};
    return c;
}

void close_handle(Device& d) {
    if (d.handle) {
        foil_device* h = d.handle;
        d.handle = nullptr;
        check(foil_close_device(h));
    }
}

}  // namespace

std::shared_ptr<Device> open_device(int pcie_device_index, const std::string& firmware_dir,
                                    std::vector<CoreCoord> cores) {
    std::vector<foil_core> cc;
    cc.reserve(cores.size());
    for (const auto& c : cores) cc.push_back(foil_core{c.x, c.y});
    foil_device* h = nullptr;
    check(foil_open_device(pcie_device_index, firmware_dir.c_str(), cc.data(), cc.size(), &h));
    auto* d = new Device{h};
    return std::shared_ptr<Device>(d, [](Device* p) {
        if (p->handle) foil_close_device(p->handle);
        delete p;
    });
}

void close_device(std::shared_ptr<Device> device) {
    if (device) {
        close_handle(*device);
        device.reset();
    }
}

std::shared_ptr<Buffer> allocate_buffer(Device& device, BufferLocation loc, std::size_t size_bytes,
                                        CoreCoord logical_core) {
    foil_buffer b = {};
    check(foil_allocate_buffer(device.handle,
                               loc == BufferLocation::L1 ? FOIL_LOC_L1 : FOIL_LOC_DRAM, size_bytes,
                               foil_core{logical_core.x, logical_core.y}, &b));
    auto* buf = new Buffer{};
    buf->location = loc;
    buf->device_addr = b.device_addr;
    buf->size_bytes = b.size_bytes;
    buf->core = logical_core;
    return std::shared_ptr<Buffer>(buf);
}

void free_buffer(std::shared_ptr<Buffer> buffer) { (void)buffer; }

void write_buffer(Device& device, Buffer& buf, const void* src, std::size_t bytes) {
    foil_buffer b = to_c(buf);
    check(foil_write_buffer(device.handle, &b, src, bytes));
}

void read_buffer(Device& device, Buffer& buf, void* dst, std::size_t bytes) {
    foil_buffer b = to_c(buf);
    check(foil_read_buffer(device.handle, &b, dst, bytes));
}

std::shared_ptr<Kernel> load_kernel(Device& device, std::span<const RiscBinary> binaries,
                                    CoreCoord logical_core) {
    std::vector<foil_risc_binary> bins;
    bins.reserve(binaries.size());
    for (const auto& b : binaries)
        bins.push_back(foil_risc_binary{static_cast<int32_t>(b.risc), b.elf_path.c_str()});
    foil_kernel* h = nullptr;
    check(foil_load_kernel(device.handle, bins.data(), bins.size(),
                           foil_core{logical_core.x, logical_core.y}, &h));
    return std::shared_ptr<Kernel>(new Kernel{h}, [](Kernel* k) {
        foil_release_kernel(k->handle);
        delete k;
    });
}

void set_runtime_args(Device& device, Kernel& kernel, RiscBinary::RiscId risc,
                      std::span<const uint32_t> args) {
    check(foil_set_runtime_args(device.handle, kernel.handle, static_cast<int32_t>(risc), args.data(),
                                args.size()));
}

void execute(Device& device, Kernel& kernel) {
    foil_kernel* one = kernel.handle;
    check(foil_execute(device.handle, &one, 1, 5000));
}

void execute(Device& device, std::initializer_list<Kernel*> kernels) {
    std::vector<foil_kernel*> v;
    for (Kernel* k : kernels) v.push_back(k ? k->handle : nullptr);
    check(foil_execute(device.handle, v.data(), v.size(), 5000));
}

uint64_t make_noc_unicast_addr(Device& device, CoreCoord logical_dst, uint64_t local_l1_addr) {
    uint64_t out = 0;
    check(foil_make_noc_unicast_addr(device.handle, foil_core{logical_dst.x, logical_dst.y},
                                     local_l1_addr, &out));
    return out;
}

uint64_t make_noc_dram_addr(Device& device, uint64_t dram_offset) {
    uint64_t out = 0;
    check(foil_make_noc_dram_addr(device.handle, dram_offset, &out));
    return out;
}

void register_cbs(Device& dev, Kernel& kernel, std::span<const CbConfig> cbs) {
    std::vector<foil_cb_config> v;
    v.reserve(cbs.size());
    for (const auto& c : cbs)
        v.push_back(foil_cb_config{c.cb_index, c.fifo_addr, c.fifo_size, c.num_pages, c.page_size});
    check(foil_register_cbs(dev.handle, kernel.handle, v.data(), v.size()));
}

}  // namespace tt::foil
