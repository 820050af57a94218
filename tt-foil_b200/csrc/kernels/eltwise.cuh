// Element-wise kernels (tile_copy, relu, add_tiles, bias_add): one streaming
// pipeline on bulk copies, launched through stream::launch.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace foil {
namespace stream {

enum Op : int { kCopy = 0, kRelu = 1, kAdd = 2, kBias = 3 };

// out[0, bytes) = op(a[0, bytes) [, b[0, bytes)]) with the golden
// arithmetic; kBias: a is a tile-layout matrix of Nt tile columns and
// bias_tiles its bias band (row 0 of each tile holds the bias).  bytes: a
// multiple of 16 (of 2048 for kBias); pointers 16-byte aligned; out equal to
// or disjoint from the inputs (all checked by the caller).  Returns a
// cudaError_t value.
int launch(Op op, const void* a, const void* b, void* out, uint64_t bytes, const uint16_t* bias_tiles,
           uint32_t Nt, uint32_t* err, cudaStream_t stream);

}  // namespace stream
}  // namespace foil
