// Layout kernels: tilize, untilize.
//
// Tile layout (the tt-foil wire format, tests/tile_utils.hpp:4-12): a 32x32
// bf16 tile is four 16x16 faces, each row-major; a face row is 16 values =
// 32 bytes = two 16-byte chunks.  Tilize is therefore a permutation of
// 16-byte chunks.  Each CTA moves one "band" of 32 rows x up to 8 tiles
// (16 KiB): global reads and writes are both fully coalesced 16-byte vector
// accesses, and the permutation happens in shared memory.  The shared-memory
// index is XOR-swizzled so that every 8-lane phase of a 16-byte access hits 8
// distinct 4-bank groups (conflict-free on both sides).
#include <cstring>

#include "common.cuh"
#include "layout.cuh"
#include "../../../include/foil_c.h"

namespace foil {
namespace {

constexpr int kBandTiles = 8;                      // tiles per band
constexpr int kChunksPerTile = 128;                // 2 KiB / 16 B
constexpr int kBandChunks = kBandTiles * kChunksPerTile;
constexpr int kLayoutThreads = 256;

// Tile-layout chunk index (inside a band) of row r, 16-byte chunk j of the
// band's row-major slice.  j = tile*4 + (col_in_tile / 8).
__device__ __forceinline__ uint32_t band_tile_chunk(uint32_t r, uint32_t j) {
    uint32_t t = j >> 2;             // tile inside the band
    uint32_t cc = (j & 3u) * 8u;     // column inside the tile
    uint32_t fr = r >> 4, r0 = r & 15u;
    uint32_t fc = cc >> 4, h = (cc >> 3) & 1u;
    return t * kChunksPerTile + (fr * 2u + fc) * 32u + r0 * 2u + h;
}

// Bank-conflict-free placement of a band chunk in shared memory: XOR bits 1
// and 2 of the index with the face-column bit (bit 5) and tile parity
// (bit 7).  Stays inside the same aligned group of 8 chunks (a bijection).
__device__ __forceinline__ uint32_t smem_slot(uint32_t idx) {
    return idx ^ (((idx >> 7) & 1u) << 2) ^ (((idx >> 5) & 1u) << 1);
}

__global__ void __launch_bounds__(kLayoutThreads)
tilize_kernel(const uint4* __restrict__ in, uint4* __restrict__ out,
              uint32_t rows, uint32_t cols) {
    griddep_wait();  // see launch_layout
    griddep_launch_dependents();
    __shared__ uint4 buf[kBandChunks];
    const uint32_t Ct = cols / 32u, Rt = rows / 32u;
    const uint32_t bands_per_row = (Ct + kBandTiles - 1) / kBandTiles;
    const uint64_t num_bands = (uint64_t)Rt * bands_per_row;
    const uint32_t row_chunks = cols / 8u;  // 16-byte chunks per input row

    for (uint64_t band = blockIdx.x; band < num_bands; band += gridDim.x) {
        const uint32_t rt = (uint32_t)(band / bands_per_row);
        const uint32_t ct0 = (uint32_t)(band % bands_per_row) * kBandTiles;
        const uint32_t bw = min((uint32_t)kBandTiles, Ct - ct0);  // tiles
        const uint32_t jn = bw * 4u;                              // chunks/row
        const uint32_t total = 32u * jn;
        // Coalesced row reads -> swizzled tile-order slots.
        for (uint32_t i = threadIdx.x; i < total; i += kLayoutThreads) {
            uint32_t r = i / jn, j = i - r * jn;
            uint4 v = __ldcs(in + (uint64_t)(rt * 32u + r) * row_chunks + ct0 * 4u + j);
            buf[smem_slot(band_tile_chunk(r, j))] = v;
        }
        __syncthreads();
        // Contiguous tile-stream writes.
        uint4* dst = out + ((uint64_t)rt * Ct + ct0) * kChunksPerTile;
        for (uint32_t o = threadIdx.x; o < total; o += kLayoutThreads)
            __stcs(dst + o, buf[smem_slot(o)]);
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kLayoutThreads)
untilize_kernel(const uint4* __restrict__ in, uint4* __restrict__ out,
                uint32_t rows, uint32_t cols) {
    griddep_wait();  // see launch_layout
    griddep_launch_dependents();
    __shared__ uint4 buf[kBandChunks];
    const uint32_t Ct = cols / 32u, Rt = rows / 32u;
    const uint32_t bands_per_row = (Ct + kBandTiles - 1) / kBandTiles;
    const uint64_t num_bands = (uint64_t)Rt * bands_per_row;
    const uint32_t row_chunks = cols / 8u;

    for (uint64_t band = blockIdx.x; band < num_bands; band += gridDim.x) {
        const uint32_t rt = (uint32_t)(band / bands_per_row);
        const uint32_t ct0 = (uint32_t)(band % bands_per_row) * kBandTiles;
        const uint32_t bw = min((uint32_t)kBandTiles, Ct - ct0);
        const uint32_t jn = bw * 4u;
        const uint32_t total = 32u * jn;
        const uint4* src = in + ((uint64_t)rt * Ct + ct0) * kChunksPerTile;
        for (uint32_t o = threadIdx.x; o < total; o += kLayoutThreads)
            buf[smem_slot(o)] = __ldcs(src + o);
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < total; i += kLayoutThreads) {
            uint32_t r = i / jn, j = i - r * jn;
            __stcs(out + (uint64_t)(rt * 32u + r) * row_chunks + ct0 * 4u + j,
                   buf[smem_slot(band_tile_chunk(r, j))]);
        }
        __syncthreads();
    }
}

}  // namespace
}  // namespace foil

extern "C" void foil_set_error(int status, const char* msg);

// Launch with programmatic stream serialization (FOIL_STREAM_PDL=0: plainly):
// the CTAs may be scheduled during the previous kernel's tail and wait
// (griddepcontrol.wait) before touching global memory.
static cudaError_t launch_layout(void (*kernel)(const uint4*, uint4*, uint32_t, uint32_t), unsigned grid,
                                 cudaStream_t stream, const uint4* in, uint4* out, uint32_t rows, uint32_t cols) {
    static const bool pdl = foil::pdl_enabled("FOIL_STREAM_PDL");
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(foil::kLayoutThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = la;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, in, out, rows, cols);
}

static int check_launch(const char* what, cudaError_t launch_err = cudaSuccess) {
    cudaError_t e = cudaGetLastError();
    if (launch_err != cudaSuccess) e = launch_err;
    if (e != cudaSuccess) {
        char buf[256];
        snprintf(buf, sizeof buf, "%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

extern "C" int foil_tilize_dev(const uint16_t* row_major, uint16_t* tiles,
                               uint32_t rows, uint32_t cols, void* stream) {
    if (rows % 32 || cols % 32) {
        foil_set_error(FOIL_ERR_INVALID, "foil_tilize_dev: rows and cols must be multiples of 32");
        return FOIL_ERR_INVALID;
    }
    if (rows == 0 || cols == 0) return FOIL_OK;
    if (!row_major || !tiles || !aligned16(row_major) || !aligned16(tiles)) {
        foil_set_error(FOIL_ERR_INVALID, "foil_tilize_dev: null or misaligned pointer");
        return FOIL_ERR_INVALID;
    }
    uint64_t bands = (uint64_t)(rows / 32) * ((cols / 32 + 7) / 8);
    uint64_t grid = bands < (uint64_t)foil_sm_count() * 8 ? bands : (uint64_t)foil_sm_count() * 8;
    const cudaError_t le = launch_layout(foil::tilize_kernel, (unsigned)grid, (cudaStream_t)stream,
                                         (const uint4*)row_major, (uint4*)tiles, rows, cols);
    return check_launch("foil_tilize_dev", le);
}

extern "C" int foil_untilize_dev(const uint16_t* tiles, uint16_t* row_major,
                                 uint32_t rows, uint32_t cols, void* stream) {
    if (rows % 32 || cols % 32) {
        foil_set_error(FOIL_ERR_INVALID, "foil_untilize_dev: rows and cols must be multiples of 32");
        return FOIL_ERR_INVALID;
    }
    if (rows == 0 || cols == 0) return FOIL_OK;
    if (!row_major || !tiles || !aligned16(row_major) || !aligned16(tiles)) {
        foil_set_error(FOIL_ERR_INVALID, "foil_untilize_dev: null or misaligned pointer");
        return FOIL_ERR_INVALID;
    }
    uint64_t bands = (uint64_t)(rows / 32) * ((cols / 32 + 7) / 8);
    uint64_t grid = bands < (uint64_t)foil_sm_count() * 8 ? bands : (uint64_t)foil_sm_count() * 8;
    const cudaError_t le = launch_layout(foil::untilize_kernel, (unsigned)grid, (cudaStream_t)stream,
                                         (const uint4*)tiles, (uint4*)row_major, rows, cols);
    return check_launch("foil_untilize_dev", le);
}

// ---------------------------------------------------- batched transpose ---
// 32 x 32 element tiles through shared memory (padded rows: no bank
// conflicts on the column reads); reads and writes are 64-byte warp rows.
namespace foil {
namespace {
__global__ void __launch_bounds__(256)
transpose_u16_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out, uint32_t in_batch,
                     uint32_t in_rows, uint32_t in_cols, uint32_t out_rows, uint32_t out_cols) {
    __shared__ uint16_t t[32][34];
    const uint32_t b = blockIdx.z, i0 = blockIdx.x * 32u, j0 = blockIdx.y * 32u;
    const uint32_t tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t i = i0 + ty + 8u * k, j = j0 + tx;
        uint16_t v = 0;
        if (b < in_batch && i < in_rows && j < in_cols) v = in[((uint64_t)b * in_rows + i) * in_cols + j];
        t[ty + 8u * k][tx] = v;
    }
    __syncthreads();
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t j = j0 + ty + 8u * k, i = i0 + tx;
        if (j < out_rows && i < out_cols) out[((uint64_t)b * out_rows + j) * out_cols + i] = t[tx][ty + 8u * k];
    }
}
}  // namespace

int transpose_u16(const uint16_t* in, uint16_t* out, uint32_t in_batch, uint32_t in_rows, uint32_t in_cols,
                  uint32_t out_batch, uint32_t out_rows, uint32_t out_cols, cudaStream_t stream) {
    if (out_batch == 0 || out_rows == 0 || out_cols == 0) return FOIL_OK;
    if (out_batch > 65535u) {
        foil_set_error(FOIL_ERR_INVALID, "transpose: batch too large");
        return FOIL_ERR_INVALID;
    }
    const dim3 grid((out_cols + 31u) / 32u, (out_rows + 31u) / 32u, out_batch);
    transpose_u16_kernel<<<grid, dim3(32, 8), 0, stream>>>(in, out, in_batch, in_rows, in_cols, out_rows, out_cols);
    return check_launch("transpose");
}

}  // namespace foil
