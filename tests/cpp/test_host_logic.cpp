// Host-only unit test of tt-foil_b200/csrc/host_logic.cpp (no GPU): bump
// allocators (reference src/device.cpp:38-58, src/buffer.cpp:11-35), the
// 64-bit address packing (src/noc_addr.cpp:10-22), program descriptors,
// CB validation (src/cb_config.cpp:46-64) and runtime-argument planning for
// every program of the accelerated path and of the scalar dispatch examples.
// Prints PASS and returns 0.
#include <cstdio>
#include <cstdlib>
#include <string>

#include "../../tt-foil_b200/csrc/host_logic.hpp"
#include "foil_c.h"

using namespace foil;

static int failures = 0;
#define CHECK(c)                                                        \
    do {                                                                \
        if (!(c)) {                                                     \
            std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #c);    \
            ++failures;                                                 \
        }                                                               \
    } while (0)

template <class F>
static int status_of(F&& f) {
    try {
        f();
    } catch (const FoilError& e) {
        return e.status;
    }
    return 0;
}

static void test_allocators() {
    BumpAllocator l1{kL1Base, kL1Base, kL1End};
    uint64_t a = l1.alloc(10, kL1Align, "L1");
    uint64_t b = l1.alloc(10, kL1Align, "L1");
    CHECK(a == kL1Base && b == kL1Base + 16);
    CHECK(status_of([&] { l1.alloc(0, kL1Align, "L1"); }) == FOIL_ERR_INVALID);
    CHECK(status_of([&] { l1.alloc(kL1End, kL1Align, "L1"); }) == FOIL_ERR_OOM);
    // exhausting exactly to the end is allowed, one more byte is not
    BumpAllocator d{0, 0, 1024};
    CHECK(d.alloc(1000, kDramAlign, "DRAM") == 0);
    CHECK(status_of([&] { d.alloc(1, kDramAlign, "DRAM"); }) == FOIL_ERR_OOM);
    BumpAllocator d2{0, 0, 1024};
    d2.alloc(1, kDramAlign, "DRAM");
    CHECK(d2.alloc(992, kDramAlign, "DRAM") == 32);
    CHECK(status_of([&] { d2.alloc(1, kDramAlign, "DRAM"); }) == FOIL_ERR_OOM);
}

static void test_addresses() {
    uint64_t a = pack_addr(3, 5, 0x12345);
    CHECK(a == ((5ull << 42) | (3ull << 36) | 0x12345));
    DecodedAddr d = decode_addr(a);
    CHECK(!d.dram && d.x == 3 && d.y == 5 && d.offset == 0x12345);
    DecodedAddr dd = decode_addr(pack_addr(kDramNode, kDramNode, (1ull << 36) - 32));
    CHECK(dd.dram && dd.offset == (1ull << 36) - 32);
}

static std::string desc(const char* prog, const char* role, const char* variant = nullptr) {
    std::string s = "TTFOIL-B200-PROGRAM 1\nprogram=";
    s += prog;
    s += "\nrole=";
    s += role;
    s += "\n";
    if (variant) s += std::string("variant=") + variant + "\n";
    return s;
}

static void test_descriptors() {
    Descriptor d = parse_descriptor(desc("matmul_dram", "reader"), "x");
    CHECK(d.program == "matmul_dram" && d.role == "reader");
    CHECK(status_of([] { parse_descriptor("\x7f" "ELF garbage", "x"); }) == FOIL_ERR_INVALID);
    CHECK(status_of([] { parse_descriptor("TTFOIL-B200-PROGRAM 1\nrole=reader\n", "x"); }) ==
          FOIL_ERR_INVALID);
    CHECK(resolve_program({parse_descriptor(desc("conv_3x3_s2", "reader"), "x")}) ==
          Program::MatmulDram);
    CHECK(resolve_program({parse_descriptor(desc("matmul_2core_mcast", "reader", "producer"), "x"),
                           parse_descriptor(desc("matmul_2core_mcast", "writer"), "x")}) ==
          Program::McastProducer);
    CHECK(status_of([] {
              resolve_program({parse_descriptor(desc("relu", "reader"), "x"),
                               parse_descriptor(desc("add_tiles", "writer"), "x")});
          }) == FOIL_ERR_INVALID);
    CHECK(status_of([] { resolve_program({parse_descriptor(desc("erisc_ping", "reader"), "x")}); }) ==
          FOIL_ERR_UNSUPPORTED);
    CHECK(resolve_program({parse_descriptor(desc("add_two_numbers", "reader"), "x"),
                           parse_descriptor(desc("add_two_numbers", "writer"), "x")}) ==
          Program::AddTwoNumbers);
    CHECK(resolve_program({parse_descriptor(desc("noc_passthrough", "reader", "consumer"), "x")}) ==
          Program::NocConsumer);
    CHECK(status_of([] { resolve_program({parse_descriptor(desc("noc_passthrough", "reader"), "x")}); }) ==
          FOIL_ERR_INVALID);
    CHECK(status_of([] { resolve_program({}); }) == FOIL_ERR_INVALID);
    CHECK(role_of_risc(0) == Role::Reader && role_of_risc(1) == Role::Writer &&
          role_of_risc(4) == Role::Compute);
}

static void test_cbs() {
    CHECK(validate_cbs({{0, kL1Base, 2048, 1, 2048}, {16, kL1Base + 2048, 2048, 1, 2048}}) ==
          ((1ull << 0) | (1ull << 16)));
    CHECK(status_of([] { validate_cbs({{32, kL1Base, 2048, 1, 2048}}); }) == FOIL_ERR_INVALID);
    CHECK(status_of([] { validate_cbs({{1, kL1Base, 64, 1, 64}, {1, kL1Base, 64, 1, 64}}); }) ==
          FOIL_ERR_INVALID);
    CHECK(status_of([] { validate_cbs({{1, kL1End - 16, 64, 1, 64}}); }) == FOIL_ERR_INVALID);
}

static void test_plans() {
    std::array<std::vector<uint32_t>, 5> rta;
    std::array<bool, 5> has{};
    // matmul_mnk: reader [a, b, Mt, Kt, Nt], writer [out, Mt*Nt]
    rta[0] = {0x20000, 0x30000, 2, 4, 3};
    rta[1] = {0x40000, 6};
    has[0] = has[1] = true;
    auto ops = plan_program(Program::MatmulMnk, 1, 2, rta, has);
    CHECK(ops.size() == 1 && ops[0].kind == OpKind::Matmul && ops[0].Mt == 2 && ops[0].Kt == 4 &&
          ops[0].Nt == 3);
    CHECK(!ops[0].in0.dram && ops[0].in0.core_x == 1 && ops[0].in0.core_y == 2 &&
          ops[0].in0.bytes == 2u * 4 * 2048 && ops[0].out.bytes == 6u * 2048);
    rta[1] = {0x40000, 5};  // inconsistent tile count
    CHECK(status_of([&] { plan_program(Program::MatmulMnk, 0, 0, rta, has); }) == FOIL_ERR_INVALID);
    // matmul_dram family: lo/hi packed DRAM addresses
    uint64_t a = pack_addr(kDramNode, kDramNode, 0x1000), b = pack_addr(kDramNode, kDramNode, 0x9000),
             c = pack_addr(kDramNode, kDramNode, 0x20000);
    rta[0] = {uint32_t(a), uint32_t(a >> 32), uint32_t(b), uint32_t(b >> 32), 1, 9, 2};
    rta[1] = {uint32_t(c), uint32_t(c >> 32), 2};
    ops = plan_program(Program::MatmulDram, 0, 0, rta, has);
    CHECK(ops.size() == 1 && ops[0].in0.dram && ops[0].in0.offset == 0x1000 &&
          ops[0].in1.offset == 0x9000 && ops[0].out.offset == 0x20000 && ops[0].Kt == 9);
    // zero tile counts are rejected
    rta[0][5] = 0;
    CHECK(status_of([&] { plan_program(Program::MatmulDram, 0, 0, rta, has); }) == FOIL_ERR_INVALID);
    // missing writer args
    has[1] = false;
    CHECK(status_of([&] { plan_program(Program::TileCopy, 0, 0, rta, has); }) == FOIL_ERR_INVALID);
    has[1] = true;
    // mcast producer: forward op then GEMM reading the local staging buffer
    uint64_t st = pack_addr(0, 1, 0x30000), fl = pack_addr(0, 1, 0x40000);
    rta[0] = {uint32_t(a), uint32_t(a >> 32), uint32_t(b), uint32_t(b >> 32), uint32_t(st),
              uint32_t(st >> 32), uint32_t(fl), uint32_t(fl >> 32), 0x25000, 0x26000, 1, 4, 2, 0x27000};
    rta[1] = {uint32_t(c), uint32_t(c >> 32), 2};
    ops = plan_program(Program::McastProducer, 0, 0, rta, has);
    CHECK(ops.size() == 2 && ops[0].kind == OpKind::McastForward && ops[1].kind == OpKind::Matmul);
    CHECK(ops[0].out.core_y == 1 && ops[0].flag_dst.offset == 0x40000 && !ops[1].in1.dram &&
          ops[1].in1.offset == 0x25000);
    // mcast consumer: gated GEMM
    rta[0] = {uint32_t(a), uint32_t(a >> 32), 0x30000, 0x40000, 1, 4, 2};
    ops = plan_program(Program::McastConsumer, 0, 1, rta, has);
    CHECK(ops.size() == 1 && ops[0].gated && ops[0].gate_flag.offset == 0x40000 &&
          ops[0].gate_flag.core_y == 1);
    // eltwise programs are one tile
    rta[0] = {0x20000, 0x20800};
    rta[1] = {0x21000};
    ops = plan_program(Program::BiasAdd, 0, 0, rta, has);
    CHECK(ops.size() == 1 && ops[0].kind == OpKind::BiasAdd && ops[0].in1.offset == 0x20800 &&
          ops[0].out.bytes == 2048);
}

static void test_scalar_plans() {
    std::array<std::vector<uint32_t>, 5> rta;
    std::array<bool, 5> has{};
    // add_two_numbers: BRISC [a, b, sum] -> Add; NCRISC [a, b, prod] -> Mul
    CHECK(status_of([&] { plan_program(Program::AddTwoNumbers, 0, 0, rta, has); }) == FOIL_ERR_INVALID);
    rta[0] = {0x20000, 0x20010, 0x20020};
    has[0] = true;
    auto ops = plan_program(Program::AddTwoNumbers, 0, 1, rta, has);
    CHECK(ops.size() == 1 && ops[0].kind == OpKind::Word && ops[0].word == WordOp::Add &&
          ops[0].in1.offset == 0x20010 && ops[0].out.offset == 0x20020 && ops[0].out.core_y == 1 &&
          ops[0].out.bytes == 4);
    rta[1] = {0x20000, 0x20010, 0x20030};
    has[1] = true;
    ops = plan_program(Program::AddTwoNumbers, 0, 0, rta, has);
    CHECK(ops.size() == 2 && ops[1].word == WordOp::Mul && ops[1].out.offset == 0x20030);
    rta[1] = {0x20000};
    CHECK(status_of([&] { plan_program(Program::AddTwoNumbers, 0, 0, rta, has); }) == FOIL_ERR_INVALID);
    has[1] = false;
    // noc_passthrough producer: sum, sentinel, then send + flag
    uint64_t sd = pack_addr(0, 1, 0x20040), fd = pack_addr(0, 1, 0x20050);
    rta[0] = {0x20000, 0x20010, 0x20020, uint32_t(sd), uint32_t(sd >> 32), 0x20030, uint32_t(fd),
              uint32_t(fd >> 32)};
    ops = plan_program(Program::NocProducer, 0, 0, rta, has);
    CHECK(ops.size() == 3 && ops[0].kind == OpKind::Word && ops[0].word == WordOp::Add &&
          ops[0].out.offset == 0x20020);
    CHECK(ops[1].kind == OpKind::Word && ops[1].word == WordOp::Set && ops[1].imm == kNocFlagValue &&
          ops[1].out.offset == 0x20030);
    CHECK(ops[2].kind == OpKind::Send && ops[2].in0.offset == 0x20020 && ops[2].out.core_y == 1 &&
          ops[2].out.offset == 0x20040 && ops[2].flag_src.offset == 0x20030 &&
          ops[2].flag_dst.offset == 0x20050 && ops[2].flag_dst.core_y == 1);
    rta[0].pop_back();
    CHECK(status_of([&] { plan_program(Program::NocProducer, 0, 0, rta, has); }) == FOIL_ERR_INVALID);
    // noc_passthrough consumer: gated on the sentinel, result = sum * 2
    rta[0] = {0x20050, 0x20040, 0x20060};
    ops = plan_program(Program::NocConsumer, 0, 1, rta, has);
    CHECK(ops.size() == 1 && ops[0].gated && ops[0].gate_value == kNocFlagValue &&
          ops[0].gate_flag.offset == 0x20050 && ops[0].word == WordOp::Scale && ops[0].imm == 2 &&
          ops[0].in0.offset == 0x20040 && ops[0].out.offset == 0x20060);
}

int main() {
    test_allocators();
    test_addresses();
    test_descriptors();
    test_cbs();
    test_plans();
    test_scalar_plans();
    if (failures) {
        std::printf("test_host_logic: FAIL (%d)\n", failures);
        return 1;
    }
    std::printf("test_host_logic: PASS\n");
    return 0;
}
