// Host-side launcher of the tcgen05 tiled GEMM (gemm_tc.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace foil {
namespace gemm {

// C = A . B (+bias, relu) on tile-layout operands.  `err` is a device word
// that receives device-side error codes (may be null).  `max_ctas` caps the
// persistent grid (normally the SM count).  Returns a foil_status.
int launch(const uint16_t* a, const uint16_t* b, uint16_t* c, uint32_t Mt, uint32_t Kt,
           uint32_t Nt, const uint16_t* bias, int relu, uint32_t* err, cudaStream_t stream,
           int max_ctas);

}  // namespace gemm
}  // namespace foil
