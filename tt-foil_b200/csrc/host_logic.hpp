// Host-side logic of the B200 tt-foil runtime that needs no GPU: bump
// allocators, the 64-bit core/DRAM address encoding, program descriptors,
// circular-buffer validation and the translation of a program's runtime
// arguments into a launch plan.  foil_runtime.cpp binds these to CUDA; the
// C++ unit test tests/cpp/test_host_logic.cpp exercises them on the CPU.
#pragma once

#include <array>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace foil {

// Error carrying a foil_status code; converted to the C status at the ABI.
struct FoilError : std::runtime_error {
    int status;
    FoilError(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

// ---------------------------------------------------------------- arenas ---
// Emulated per-core L1: offsets [kL1Base, kL1End) of a 1.5 MiB arena.  The
// bottom 128 KiB stays unused so that no buffer sits at offset 0, like the
// firmware-reserved bottom of a Tensix L1.
constexpr uint64_t kL1Size = 1536ull * 1024ull;
constexpr uint64_t kL1Base = 128ull * 1024ull;
constexpr uint64_t kL1End = kL1Size;
constexpr uint32_t kL1Align = 16;    // src/buffer.cpp:20
constexpr uint32_t kDramAlign = 32;  // src/buffer.cpp:24
// DRAM arena: offsets must fit the 36-bit local field of a packed address.
constexpr uint64_t kDramLimit = 1ull << 36;

// Bump allocator with the reference's semantics (src/device.cpp:38-58):
// align up, throw when the request passes the end, never reclaim.
struct BumpAllocator {
    uint64_t base{0};
    uint64_t current{0};
    uint64_t end{0};
    uint64_t alloc(uint64_t bytes, uint32_t alignment, const char* what);
};

// ------------------------------------------------------ address encoding ---
// 64-bit address: bits [47:42] = y, [41:36] = x, [35:0] = offset
// (src/noc_addr.cpp:10-22).  Core coordinates 0..62 address that core's L1
// arena; the node (x = 63, y = 63) addresses the DRAM arena.
constexpr uint32_t kNodeBits = 6;
constexpr uint32_t kLocalBits = 36;
constexpr uint32_t kDramNode = 63;

uint64_t pack_addr(uint32_t x, uint32_t y, uint64_t offset);
struct DecodedAddr {
    bool dram;
    uint32_t x, y;
    uint64_t offset;
};
DecodedAddr decode_addr(uint64_t a);

// ------------------------------------------------------------- programs ---
enum class Program {
    TileCopy,
    Matmul1Tile,
    MatmulKt,
    MatmulMnk,       // L1-resident operands
    MatmulDram,      // DRAM-resident operands (dram, 2core, 2x2, 4x2, conv_*)
    McastProducer,   // matmul_2core_mcast producer core
    McastConsumer,   // matmul_2core_mcast consumer core
    Relu,
    AddTiles,
    BiasAdd,
    AddTwoNumbers,   // add_brisc (BRISC: sum) / add_ncrisc (NCRISC: product)
    NocProducer,     // noc_passthrough producer core
    NocConsumer,     // noc_passthrough consumer core
};

enum class Role { Reader, Writer, Compute };

struct Descriptor {
    std::string program;  // e.g. "matmul_dram"
    std::string role;     // reader | writer | compute
    std::string variant;  // "" | producer | consumer
};

// Parse the text of a program-descriptor file.  Throws FoilError.
Descriptor parse_descriptor(const std::string& text, const std::string& path);

// Program for a set of descriptors (all must name the same program; the
// reader's variant selects the producer / consumer of matmul_2core_mcast and
// noc_passthrough).  Throws FoilError for programs it does not know.
Program resolve_program(const std::vector<Descriptor>& ds);

const char* program_name(Program p);

// Role a RISC id (0..4) must carry.
Role role_of_risc(int risc);
Role parse_role(const std::string& r);

// ---------------------------------------------------------- CB configs ---
struct CbDesc {
    uint8_t cb_index;
    uint64_t fifo_addr;
    uint32_t fifo_size, num_pages, page_size;
};
// Reference checks (src/cb_config.cpp:46-64) plus: the ring lies inside the
// L1 arena.  Returns the mask of registered indices.  Throws FoilError.
uint64_t validate_cbs(const std::vector<CbDesc>& cbs);

// ---------------------------------------------------------- launch plans ---
// An operand location resolved from runtime arguments.
struct Loc {
    bool dram{false};
    uint32_t core_x{0}, core_y{0};  // L1 owner (when !dram)
    uint64_t offset{0};
    uint64_t bytes{0};
};

enum class OpKind { Copy, Relu, Add, BiasAdd, Matmul, McastForward, Word, Send };

// Scalar u32 step of a Word op (wrapping arithmetic, like the RISC-V cores):
// Add out = in0 + in1, Mul out = in0 * in1, Set out = imm, Scale out = in0 * imm.
enum class WordOp : uint8_t { Add, Mul, Set, Scale };

// Sentinel the noc_passthrough producer publishes and its consumer waits for
// (examples/noc_passthrough/kernels/producer.cpp:27, consumer.cpp:20).
constexpr uint32_t kNocFlagValue = 0xCAFEBABEu;

struct PlanOp {
    OpKind kind;
    Loc in0, in1, out;  // operands used by the op kind
    uint32_t Mt{0}, Kt{0}, Nt{0};
    // McastForward: in0 = B in DRAM, in1 = local staging, out = peer staging,
    // flag_src -> flag_dst (4 bytes).  Send: in0 -> out (no staging), then
    // flag_src -> flag_dst.
    Loc flag_src, flag_dst;
    // Word: the step and its immediate.
    WordOp word{WordOp::Add};
    uint32_t imm{0};
    // Gated ops wait until the core's local flag reads gate_value (0: any
    // non-zero value).
    bool gated{false};
    Loc gate_flag;
    uint32_t gate_value{0};
};

constexpr size_t kMaxRtaWords = 64;  // src/kernel.hpp:29
constexpr uint32_t kTileBytes = 2048;

// Translate a kernel's runtime arguments into operations.  `core` is the
// kernel's own core (owner of plain 32-bit L1 addresses).  rta[i] holds the
// args of RISC i; `has_rta[i]` says whether they were set.  Throws FoilError
// when an argument is missing or inconsistent.
std::vector<PlanOp> plan_program(Program prog, uint32_t core_x, uint32_t core_y,
                                 const std::array<std::vector<uint32_t>, 5>& rta,
                                 const std::array<bool, 5>& has_rta);

}  // namespace foil
