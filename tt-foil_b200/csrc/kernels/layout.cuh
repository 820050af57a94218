// Host-side launcher of the batched transpose (layout.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace foil {

// out[b][j][i] = in[b][i][j] for b < in_batch, i < in_rows, j < in_cols and 0
// elsewhere, over b < out_batch, j < out_rows, i < out_cols; 16-bit elements,
// both tensors dense.  Re-lays channel-major activations and weights as
// channel-minor ones (and back), zero-padding the channel counts.  Returns a
// foil_status.
int transpose_u16(const uint16_t* in, uint16_t* out, uint32_t in_batch, uint32_t in_rows, uint32_t in_cols,
                  uint32_t out_batch, uint32_t out_rows, uint32_t out_cols, cudaStream_t stream);

}  // namespace foil
