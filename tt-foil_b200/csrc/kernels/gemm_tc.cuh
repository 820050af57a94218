// Host-side launcher of the tcgen05 tiled GEMM (gemm_tc.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace foil {
namespace gemm {

// Most peer copies of C one launch writes (8 GPUs per node).
constexpr uint32_t kMaxPeers = 7;

// C = A . B (+bias, relu) on tile-layout operands.  `err` is a device word
// that receives device-side error codes (may be null).  `max_ctas` caps the
// persistent grid (normally the SM count).  `peer_c[0..npeers)`: other GPUs'
// buffers (peer-mapped device pointers, same layout as c) that receive every
// output tile as well.  `mc_c` (instead of peer_c): an NVLink multicast
// address bound to every GPU's copy of C, this one included, at c's offset;
// each output tile is stored once through it.  Returns a foil_status.
int launch(const uint16_t* a, const uint16_t* b, uint16_t* c, uint32_t Mt, uint32_t Kt,
           uint32_t Nt, const uint16_t* bias, int relu, uint32_t* err, cudaStream_t stream,
           int max_ctas, uint16_t* const* peer_c = nullptr, uint32_t npeers = 0, uint16_t* mc_c = nullptr);

// One "core" of a multi-core execute: the work one logical core's program
// does, run by one CTA of a single cluster launch in which every core's CTA
// is resident at the same time, so cores may wait on each other's flags.
// In order: (1) if `gate` is set, wait (bounded) until *gate == gate_value
// (gate_value 0: until *gate != 0); (2) the scalar u32 steps words[0..nwords)
// in order; (3) if fwd_bytes, copy fwd_src -> fwd_stage -> fwd_peer (or
// fwd_src -> fwd_peer when fwd_stage is null) and then publish *flag_dst =
// *flag_src with release semantics (after the copies); (4) if Mt, the tiled
// GEMM c = a . b (Mt x Kt x Nt tiles).
enum WordCode : uint32_t { kWordAdd = 0, kWordMul = 1, kWordSet = 2, kWordScale = 3 };
// out = a + b | a * b | imm | a * imm (wrapping u32).
struct WordStep {
    const uint32_t* a;
    const uint32_t* b;
    uint32_t* out;
    uint32_t imm;
    uint32_t code;
};
constexpr uint32_t kMaxWordSteps = 4;

struct CoreProgram {
    const uint32_t* gate;
    uint32_t gate_value;
    uint32_t nwords;
    WordStep words[kMaxWordSteps];
    const void* fwd_src;
    void* fwd_stage;
    void* fwd_peer;
    uint64_t fwd_bytes;
    const uint32_t* flag_src;
    uint32_t* flag_dst;
    const uint16_t* a;
    const uint16_t* b;
    uint16_t* c;
    uint32_t Mt, Kt, Nt;
};
constexpr uint32_t kMaxCores = 8;

// Launch `ncores` (<= kMaxCores) core programs as one cluster of ncores CTAs
// on `stream`.  A gate wait that runs out after `gate_wait_ns` sets
// kErrWaitTimeout in *err and 1 in core_status[core] (device words, cleared
// by the caller), and that core does nothing else.  Returns a foil_status.
int launch_cores(const CoreProgram* cores, uint32_t ncores, uint32_t* err, uint32_t* core_status,
                 uint64_t gate_wait_ns, cudaStream_t stream);

}  // namespace gemm
}  // namespace foil
