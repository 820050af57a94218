// Host-side launcher of the implicit-GEMM NHWC convolution (conv_tc.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace foil {
namespace conv {

// y (N, Ho, Wo, Cout) = relu?(conv(x (N, H, W, Cin), w (Cout, KH, KW, Cin)) + bias)
// with Ho = (H + 2 pad - KH) / stride + 1 (likewise Wo).  Requires Cin and
// Cout multiples of 16 and 16-byte aligned pointers (checked by the caller).
int launch(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y, uint32_t N,
           uint32_t H, uint32_t W, uint32_t Cin, uint32_t Cout, uint32_t KH, uint32_t KW,
           uint32_t stride, uint32_t pad, int relu, uint32_t* err, cudaStream_t stream,
           int max_ctas);

}  // namespace conv
}  // namespace foil
