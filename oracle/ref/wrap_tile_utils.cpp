// ORACLE — test infrastructure only.
//
// extern "C" access to the reference's tests/tile_utils.hpp (bf16 rounding
// and the 32x32 / 16x16-face tile permutation), compiled from the reference
// tree by the recipe oracle/build.py.
#include <cstdint>
#include <vector>

#include "tile_utils.hpp"

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

REF_EXPORT uint16_t ref_f32_to_bf16(float f) { return tt::foil::test::f32_to_bf16(f); }
REF_EXPORT float ref_bf16_to_f32(uint16_t b) { return tt::foil::test::bf16_to_f32(b); }

REF_EXPORT void ref_f32_to_bf16_array(const float* in, uint16_t* out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) out[i] = tt::foil::test::f32_to_bf16(in[i]);
}

// One 32x32 row-major block -> one tile (1024 values).
REF_EXPORT void ref_row_major_to_tile(const uint16_t* rm, uint16_t* tile) {
    std::vector<uint16_t> v;
    tt::foil::test::row_major_to_tile(rm, v);
    for (size_t i = 0; i < v.size(); ++i) tile[i] = v[i];
}

REF_EXPORT void ref_tile_to_row_major(const uint16_t* tile, uint16_t* rm) {
    tt::foil::test::tile_to_row_major(tile, rm);
}
