// ORACLE — test infrastructure only.
//
// Link-time stand-in for the tt-foil device API (include/tt_foil/runtime.hpp
// and cb_config.hpp) used when the reference's golden functions are compiled
// into oracle/_ref/libref_golden.so.  The golden wrappers include whole
// reference test files, whose (renamed, never called) main() refers to
// open_device, execute and the rest; those references resolve here instead
// of against the product libraries, so the reference-built checker and the
// CPU baseline map no library of this repository's runtime.  Every function
// throws: nothing in the golden code path may reach the device API.
#include <cstddef>
#include <cstdint>
#include <initializer_list>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

#include "tt_foil/cb_config.hpp"
#include "tt_foil/runtime.hpp"

namespace tt::foil {

struct Device {};
struct Kernel {};

namespace {
[[noreturn]] void unavailable(const char* fn) {
    throw std::runtime_error(std::string("reference golden library: ") + fn +
                             " is not available (device API stubbed out)");
}
}  // namespace

std::shared_ptr<Device> open_device(int, const std::string&, std::vector<CoreCoord>) {
    unavailable("open_device");
}
void close_device(std::shared_ptr<Device>) { unavailable("close_device"); }
std::shared_ptr<Buffer> allocate_buffer(Device&, BufferLocation, std::size_t, CoreCoord) {
    unavailable("allocate_buffer");
}
void free_buffer(std::shared_ptr<Buffer>) { unavailable("free_buffer"); }
void write_buffer(Device&, Buffer&, const void*, std::size_t) { unavailable("write_buffer"); }
void read_buffer(Device&, Buffer&, void*, std::size_t) { unavailable("read_buffer"); }
std::shared_ptr<Kernel> load_kernel(Device&, std::span<const RiscBinary>, CoreCoord) {
    unavailable("load_kernel");
}
void set_runtime_args(Device&, Kernel&, RiscBinary::RiscId, std::span<const uint32_t>) {
    unavailable("set_runtime_args");
}
void execute(Device&, Kernel&) { unavailable("execute"); }
void execute(Device&, std::initializer_list<Kernel*>) { unavailable("execute"); }
uint64_t make_noc_unicast_addr(Device&, CoreCoord, uint64_t) { unavailable("make_noc_unicast_addr"); }
uint64_t make_noc_dram_addr(Device&, uint64_t) { unavailable("make_noc_dram_addr"); }
void register_cbs(Device&, Kernel&, std::span<const CbConfig>) { unavailable("register_cbs"); }

}  // namespace tt::foil
