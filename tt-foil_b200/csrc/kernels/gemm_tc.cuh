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
// output tile as well.  Returns a foil_status.
int launch(const uint16_t* a, const uint16_t* b, uint16_t* c, uint32_t Mt, uint32_t Kt,
           uint32_t Nt, const uint16_t* bias, int relu, uint32_t* err, cudaStream_t stream,
           int max_ctas, uint16_t* const* peer_c = nullptr, uint32_t npeers = 0);

}  // namespace gemm
}  // namespace foil
