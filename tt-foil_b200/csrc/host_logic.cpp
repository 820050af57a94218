// GPU-free host logic of the B200 tt-foil runtime (see host_logic.hpp).
#include "host_logic.hpp"

#include <sstream>

#include "../../include/foil_c.h"

namespace foil {

uint64_t BumpAllocator::alloc(uint64_t bytes, uint32_t alignment, const char* what) {
    if (bytes == 0) throw FoilError(FOIL_ERR_INVALID, "tt-foil: buffer size must be > 0");
    const uint64_t aligned = (current + alignment - 1) & ~uint64_t(alignment - 1);
    if (aligned > end || bytes > end - aligned)
        throw FoilError(FOIL_ERR_OOM, std::string("tt-foil: ") + what + " out of memory");
    current = aligned + bytes;
    return aligned;
}

uint64_t pack_addr(uint32_t x, uint32_t y, uint64_t offset) {
    const uint64_t node_mask = (1ull << kNodeBits) - 1;
    const uint64_t local_mask = (1ull << kLocalBits) - 1;
    return ((uint64_t(y) & node_mask) << (kLocalBits + kNodeBits)) |
           ((uint64_t(x) & node_mask) << kLocalBits) | (offset & local_mask);
}

DecodedAddr decode_addr(uint64_t a) {
    const uint64_t node_mask = (1ull << kNodeBits) - 1;
    DecodedAddr d;
    d.y = uint32_t((a >> (kLocalBits + kNodeBits)) & node_mask);
    d.x = uint32_t((a >> kLocalBits) & node_mask);
    d.offset = a & ((1ull << kLocalBits) - 1);
    d.dram = (d.x == kDramNode && d.y == kDramNode);
    return d;
}

static std::string trim(const std::string& s) {
    size_t b = s.find_first_not_of(" \t\r\n");
    if (b == std::string::npos) return "";
    size_t e = s.find_last_not_of(" \t\r\n");
    return s.substr(b, e - b + 1);
}

Descriptor parse_descriptor(const std::string& text, const std::string& path) {
    std::istringstream in(text);
    std::string line;
    if (!std::getline(in, line) || trim(line) != "TTFOIL-B200-PROGRAM 1")
        throw FoilError(FOIL_ERR_INVALID,
                        "tt-foil: not a tt-foil B200 program descriptor: " + path);
    Descriptor d;
    while (std::getline(in, line)) {
        line = trim(line);
        if (line.empty() || line[0] == '#') continue;
        size_t eq = line.find('=');
        if (eq == std::string::npos)
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: malformed descriptor line in " + path);
        std::string k = trim(line.substr(0, eq)), v = trim(line.substr(eq + 1));
        if (k == "program") d.program = v;
        else if (k == "role") d.role = v;
        else if (k == "variant") d.variant = v;
    }
    if (d.program.empty() || d.role.empty())
        throw FoilError(FOIL_ERR_INVALID, "tt-foil: descriptor without program/role: " + path);
    return d;
}

Role parse_role(const std::string& r) {
    if (r == "reader") return Role::Reader;
    if (r == "writer") return Role::Writer;
    if (r == "compute") return Role::Compute;
    throw FoilError(FOIL_ERR_INVALID, "tt-foil: unknown descriptor role '" + r + "'");
}

Role role_of_risc(int risc) {
    switch (risc) {
        case 0: return Role::Reader;
        case 1: return Role::Writer;
        case 2: case 3: case 4: return Role::Compute;
    }
    throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid RISC id " + std::to_string(risc));
}

Program resolve_program(const std::vector<Descriptor>& ds) {
    if (ds.empty()) throw FoilError(FOIL_ERR_INVALID, "tt-foil: no binaries provided to load_kernel");
    const std::string& name = ds[0].program;
    std::string variant;
    for (const auto& d : ds) {
        if (d.program != name)
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: binaries of one kernel name different programs ('" +
                                                  name + "' and '" + d.program + "')");
        if (!d.variant.empty()) variant = d.variant;
    }
    if (name == "tile_copy") return Program::TileCopy;
    if (name == "matmul_1tile") return Program::Matmul1Tile;
    if (name == "matmul_kt") return Program::MatmulKt;
    if (name == "matmul_mnk") return Program::MatmulMnk;
    if (name == "matmul_dram" || name == "matmul_2core" || name == "matmul_2x2" ||
        name == "matmul_4x2" || name == "conv_1x1" || name == "conv_3x3" ||
        name == "conv_3x3_2core" || name == "conv_3x3_s2")
        return Program::MatmulDram;
    if (name == "matmul_2core_mcast") {
        if (variant == "producer") return Program::McastProducer;
        if (variant == "consumer") return Program::McastConsumer;
        throw FoilError(FOIL_ERR_INVALID, "tt-foil: matmul_2core_mcast kernel needs a producer or consumer reader");
    }
    if (name == "relu") return Program::Relu;
    if (name == "add_tiles") return Program::AddTiles;
    if (name == "bias_add") return Program::BiasAdd;
    if (name == "add_two_numbers") return Program::AddTwoNumbers;
    if (name == "noc_passthrough") {
        if (variant == "producer") return Program::NocProducer;
        if (variant == "consumer") return Program::NocConsumer;
        throw FoilError(FOIL_ERR_INVALID, "tt-foil: noc_passthrough kernel needs a producer or consumer binary");
    }
    throw FoilError(FOIL_ERR_UNSUPPORTED, "tt-foil: program '" + name +
                                              "' is not part of the B200 accelerated path");
}

const char* program_name(Program p) {
    switch (p) {
        case Program::TileCopy: return "tile_copy";
        case Program::Matmul1Tile: return "matmul_1tile";
        case Program::MatmulKt: return "matmul_kt";
        case Program::MatmulMnk: return "matmul_mnk";
        case Program::MatmulDram: return "matmul_dram";
        case Program::McastProducer: return "matmul_2core_mcast/producer";
        case Program::McastConsumer: return "matmul_2core_mcast/consumer";
        case Program::Relu: return "relu";
        case Program::AddTiles: return "add_tiles";
        case Program::BiasAdd: return "bias_add";
        case Program::AddTwoNumbers: return "add_two_numbers";
        case Program::NocProducer: return "noc_passthrough/producer";
        case Program::NocConsumer: return "noc_passthrough/consumer";
    }
    return "?";
}

uint64_t validate_cbs(const std::vector<CbDesc>& cbs) {
    uint64_t mask = 0;
    for (const auto& c : cbs) {
        if (c.cb_index >= 32)
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: register_cbs: cb_index must be < 32 (got " +
                                                  std::to_string(c.cb_index) + ")");
        if (mask & (1ull << c.cb_index))
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: register_cbs: cb_index " +
                                                  std::to_string(c.cb_index) + " listed twice");
        if (c.fifo_addr < kL1Base || c.fifo_addr > kL1End || c.fifo_size > kL1End - c.fifo_addr)
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: register_cbs: ring of cb " +
                                                  std::to_string(c.cb_index) + " lies outside L1");
        mask |= 1ull << c.cb_index;
    }
    return mask;
}

namespace {

const std::vector<uint32_t>& need(const std::array<std::vector<uint32_t>, 5>& rta,
                                  const std::array<bool, 5>& has, int risc, size_t n,
                                  Program prog) {
    static const char* names[5] = {"BRISC", "NCRISC", "TRISC0", "TRISC1", "TRISC2"};
    if (!has[risc] || rta[risc].size() < n)
        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + program_name(prog) + " needs " +
                                              std::to_string(n) + " runtime args on " + names[risc]);
    return rta[risc];
}

Loc l1(uint32_t cx, uint32_t cy, uint32_t addr, uint64_t bytes) {
    Loc l;
    l.dram = false;
    l.core_x = cx;
    l.core_y = cy;
    l.offset = addr;
    l.bytes = bytes;
    return l;
}

Loc noc(uint32_t lo, uint32_t hi, uint64_t bytes) {
    DecodedAddr d = decode_addr((uint64_t(hi) << 32) | lo);
    Loc l;
    l.dram = d.dram;
    l.core_x = d.x;
    l.core_y = d.y;
    l.offset = d.offset;
    l.bytes = bytes;
    return l;
}

void check_dims(Program prog, uint64_t Mt, uint64_t Kt, uint64_t Nt) {
    if (Mt == 0 || Kt == 0 || Nt == 0 || Mt > 65535 || Kt > 65535 || Nt > 65535)
        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + program_name(prog) +
                                              ": tile counts must be in 1..65535");
}

void check_count(Program prog, uint64_t got, uint64_t want) {
    if (got != want)
        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + program_name(prog) +
                                              ": writer tile count " + std::to_string(got) +
                                              " != Mt*Nt " + std::to_string(want));
}

PlanOp word(WordOp w, Loc in0, Loc in1, Loc out, uint32_t imm = 0) {
    PlanOp op;
    op.kind = OpKind::Word;
    op.word = w;
    op.in0 = in0;
    op.in1 = in1;
    op.out = out;
    op.imm = imm;
    return op;
}

PlanOp matmul(Loc a, Loc b, Loc c, uint32_t Mt, uint32_t Kt, uint32_t Nt) {
    PlanOp op;
    op.kind = OpKind::Matmul;
    op.in0 = a;
    op.in1 = b;
    op.out = c;
    op.Mt = Mt;
    op.Kt = Kt;
    op.Nt = Nt;
    return op;
}

}  // namespace

std::vector<PlanOp> plan_program(Program prog, uint32_t cx, uint32_t cy,
                                 const std::array<std::vector<uint32_t>, 5>& rta,
                                 const std::array<bool, 5>& has) {
    std::vector<PlanOp> ops;
    const uint64_t T = kTileBytes;
    switch (prog) {
        case Program::TileCopy: {  // examples/tile_copy/kernels/{reader,writer}.cpp
            auto& r = need(rta, has, 0, 1, prog);
            auto& w = need(rta, has, 1, 1, prog);
            PlanOp op;
            op.kind = OpKind::Copy;
            op.in0 = l1(cx, cy, r[0], T);
            op.out = l1(cx, cy, w[0], T);
            ops.push_back(op);
            break;
        }
        case Program::Relu: {  // examples/relu/kernels/*
            auto& r = need(rta, has, 0, 1, prog);
            auto& w = need(rta, has, 1, 1, prog);
            PlanOp op;
            op.kind = OpKind::Relu;
            op.in0 = l1(cx, cy, r[0], T);
            op.out = l1(cx, cy, w[0], T);
            ops.push_back(op);
            break;
        }
        case Program::AddTiles:
        case Program::BiasAdd: {  // examples/{add_tiles,bias_add}/kernels/*
            auto& r = need(rta, has, 0, 2, prog);
            auto& w = need(rta, has, 1, 1, prog);
            PlanOp op;
            op.kind = prog == Program::AddTiles ? OpKind::Add : OpKind::BiasAdd;
            op.in0 = l1(cx, cy, r[0], T);
            op.in1 = l1(cx, cy, r[1], T);
            op.out = l1(cx, cy, w[0], T);
            ops.push_back(op);
            break;
        }
        case Program::Matmul1Tile: {  // examples/matmul_1tile/kernels/*
            auto& r = need(rta, has, 0, 2, prog);
            auto& w = need(rta, has, 1, 1, prog);
            ops.push_back(matmul(l1(cx, cy, r[0], T), l1(cx, cy, r[1], T), l1(cx, cy, w[0], T), 1, 1, 1));
            break;
        }
        case Program::MatmulKt: {  // examples/matmul_kt/kernels/reader.cpp: [a, b, Kt]
            auto& r = need(rta, has, 0, 3, prog);
            auto& w = need(rta, has, 1, 1, prog);
            uint32_t Kt = r[2];
            check_dims(prog, 1, Kt, 1);
            ops.push_back(matmul(l1(cx, cy, r[0], T * Kt), l1(cx, cy, r[1], T * Kt),
                                 l1(cx, cy, w[0], T), 1, Kt, 1));
            break;
        }
        case Program::MatmulMnk: {  // reader [a, b, Mt, Kt, Nt]; writer [out, Mt*Nt]
            auto& r = need(rta, has, 0, 5, prog);
            auto& w = need(rta, has, 1, 2, prog);
            uint32_t Mt = r[2], Kt = r[3], Nt = r[4];
            check_dims(prog, Mt, Kt, Nt);
            check_count(prog, w[1], uint64_t(Mt) * Nt);
            ops.push_back(matmul(l1(cx, cy, r[0], T * Mt * Kt), l1(cx, cy, r[1], T * Kt * Nt),
                                 l1(cx, cy, w[0], T * Mt * Nt), Mt, Kt, Nt));
            break;
        }
        case Program::MatmulDram: {  // reader [a lo/hi, b lo/hi, Mt, Kt, Nt]; writer [out lo/hi, n]
            auto& r = need(rta, has, 0, 7, prog);
            auto& w = need(rta, has, 1, 3, prog);
            uint32_t Mt = r[4], Kt = r[5], Nt = r[6];
            check_dims(prog, Mt, Kt, Nt);
            check_count(prog, w[2], uint64_t(Mt) * Nt);
            ops.push_back(matmul(noc(r[0], r[1], T * Mt * Kt), noc(r[2], r[3], T * Kt * Nt),
                                 noc(w[0], w[1], T * Mt * Nt), Mt, Kt, Nt));
            break;
        }
        case Program::McastProducer: {
            // examples/matmul_2core_mcast/kernels/reader_producer.cpp:13-23
            auto& r = need(rta, has, 0, 13, prog);
            auto& w = need(rta, has, 1, 3, prog);
            uint32_t Mt = r[10], Kt = r[11], Nt = r[12];
            check_dims(prog, Mt, Kt, Nt);
            check_count(prog, w[2], uint64_t(Mt) * Nt);
            const uint64_t b_bytes = T * Kt * Nt;
            PlanOp fwd;
            fwd.kind = OpKind::McastForward;
            fwd.in0 = noc(r[2], r[3], b_bytes);       // B in DRAM
            fwd.in1 = l1(cx, cy, r[8], b_bytes);      // local staging
            fwd.out = noc(r[4], r[5], b_bytes);       // peer staging
            fwd.flag_src = l1(cx, cy, r[9], 4);       // flag source word
            fwd.flag_dst = noc(r[6], r[7], 4);        // peer flag
            ops.push_back(fwd);
            ops.push_back(matmul(noc(r[0], r[1], T * Mt * Kt), l1(cx, cy, r[8], b_bytes),
                                 noc(w[0], w[1], T * Mt * Nt), Mt, Kt, Nt));
            break;
        }
        case Program::McastConsumer: {
            // examples/matmul_2core_mcast/kernels/reader_consumer.cpp:13-19
            auto& r = need(rta, has, 0, 7, prog);
            auto& w = need(rta, has, 1, 3, prog);
            uint32_t Mt = r[4], Kt = r[5], Nt = r[6];
            check_dims(prog, Mt, Kt, Nt);
            check_count(prog, w[2], uint64_t(Mt) * Nt);
            PlanOp op = matmul(noc(r[0], r[1], T * Mt * Kt), l1(cx, cy, r[2], T * Kt * Nt),
                               noc(w[0], w[1], T * Mt * Nt), Mt, Kt, Nt);
            op.gated = true;
            op.gate_flag = l1(cx, cy, r[3], 4);
            ops.push_back(op);
            break;
        }
        case Program::AddTwoNumbers: {
            // examples/add_two_numbers/kernels/add_brisc.cpp:25-37 (BRISC,
            // [a, b, result]: result = a + b) and add_ncrisc.cpp:19-29
            // (NCRISC, same arguments: result = a * b); either or both.
            if (!has[0] && !has[1]) need(rta, has, 0, 3, prog);
            for (int risc : {0, 1}) {
                if (!has[risc]) continue;
                auto& r = need(rta, has, risc, 3, prog);
                ops.push_back(word(risc == 0 ? WordOp::Add : WordOp::Mul, l1(cx, cy, r[0], 4),
                                   l1(cx, cy, r[1], 4), l1(cx, cy, r[2], 4)));
            }
            break;
        }
        case Program::NocProducer: {
            // examples/noc_passthrough/kernels/producer.cpp:29-58: [a, b,
            // sum_scratch, dst_sum lo/hi, flag_scratch, dst_flag lo/hi].  The
            // sum and the sentinel are assembled locally, then the sum is
            // sent and the flag published after it.
            auto& r = need(rta, has, 0, 8, prog);
            ops.push_back(word(WordOp::Add, l1(cx, cy, r[0], 4), l1(cx, cy, r[1], 4), l1(cx, cy, r[2], 4)));
            ops.push_back(word(WordOp::Set, Loc{}, Loc{}, l1(cx, cy, r[5], 4), kNocFlagValue));
            PlanOp send;
            send.kind = OpKind::Send;
            send.in0 = l1(cx, cy, r[2], 4);
            send.out = noc(r[3], r[4], 4);
            send.flag_src = l1(cx, cy, r[5], 4);
            send.flag_dst = noc(r[6], r[7], 4);
            ops.push_back(send);
            break;
        }
        case Program::NocConsumer: {
            // examples/noc_passthrough/kernels/consumer.cpp:22-38: [flag, sum,
            // result]; wait for the sentinel, then result = sum * 2.
            auto& r = need(rta, has, 0, 3, prog);
            PlanOp op = word(WordOp::Scale, l1(cx, cy, r[1], 4), Loc{}, l1(cx, cy, r[2], 4), 2u);
            op.gated = true;
            op.gate_flag = l1(cx, cy, r[0], 4);
            op.gate_value = kNocFlagValue;
            ops.push_back(op);
            break;
        }
    }
    return ops;
}

}  // namespace foil
