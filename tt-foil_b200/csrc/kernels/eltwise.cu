// Element-wise kernels on bf16 streams: add_tiles, relu, bias_add.
//
// Memory-bound: each thread moves 16-byte vectors (8 bf16) with streaming
// cache hints, several vectors in flight, in a grid-stride loop sized to a
// multiple of the SM count.  The arithmetic is the reference golden's:
// widen to fp32, operate, narrow with the golden's round-to-nearest-even
// integer formula (tests/tile_utils.hpp:33-47), so results are bit-exact.
#include "common.cuh"
#include "../../../include/foil_c.h"

extern "C" void foil_set_error(int status, const char* msg);

namespace foil {
namespace {

__device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b) {
    float lo = host_add_f32(bf16_bits_to_f32(a & 0xffffu), bf16_bits_to_f32(b & 0xffffu));
    float hi = host_add_f32(bf16_bits_to_f32(a >> 16), bf16_bits_to_f32(b >> 16));
    return pack_bf16x2(f32_to_bf16_bits(lo), f32_to_bf16_bits(hi));
}

// max(x, 0) as the golden computes it: `v < 0.0f ? 0.0f : v`
// (tests/test_relu.cpp:54-59).  -0.0 and NaN pass through unchanged.
__device__ __forceinline__ uint32_t relu1(uint32_t b) {
    return bf16_bits_to_f32(b) < 0.0f ? 0u : b;
}
__device__ __forceinline__ uint32_t relu2(uint32_t w) {
    return relu1(w & 0xffffu) | (relu1(w >> 16) << 16);
}

__device__ __forceinline__ uint4 add_v(uint4 a, uint4 b) {
    return make_uint4(add2(a.x, b.x), add2(a.y, b.y), add2(a.z, b.z), add2(a.w, b.w));
}
__device__ __forceinline__ uint4 relu_v(uint4 a) {
    return make_uint4(relu2(a.x), relu2(a.y), relu2(a.z), relu2(a.w));
}

__global__ void __launch_bounds__(256)
add_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
           uint4* __restrict__ out, uint64_t n8) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + stride < n8; i += 2 * stride) {
        uint4 a0 = __ldcs(a + i), b0 = __ldcs(b + i);
        uint4 a1 = __ldcs(a + i + stride), b1 = __ldcs(b + i + stride);
        __stcs(out + i, add_v(a0, b0));
        __stcs(out + i + stride, add_v(a1, b1));
    }
    for (; i < n8; i += stride) __stcs(out + i, add_v(__ldcs(a + i), __ldcs(b + i)));
}

__global__ void __launch_bounds__(256)
relu_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, uint64_t n8) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n8; i += 4 * stride) {
        uint4 x0 = __ldcs(in + i), x1 = __ldcs(in + i + stride);
        uint4 x2 = __ldcs(in + i + 2 * stride), x3 = __ldcs(in + i + 3 * stride);
        __stcs(out + i, relu_v(x0));
        __stcs(out + i + stride, relu_v(x1));
        __stcs(out + i + 2 * stride, relu_v(x2));
        __stcs(out + i + 3 * stride, relu_v(x3));
    }
    for (; i < n8; i += stride) __stcs(out + i, relu_v(__ldcs(in + i)));
}

// Bias add over a tile-layout matrix with Nt tile-columns, one warp per
// 2 KiB tile.  Lane l handles the 16-byte chunks l, l+32, l+64, l+96 of the
// tile: chunk c lies in face c/32 (face column (c/32) & 1) and covers columns
// ((c/32) & 1) * 16 + (l & 1) * 8 + [0, 8) of the tile.  The bias for column n
// is in row 0 of bias tile n/32, i.e. at (n/32) * 1024 + ((n%32)/16) * 256 + n%16,
// so each lane loads its two bias vectors once per tile.
__global__ void __launch_bounds__(256)
bias_kernel(const uint4* __restrict__ in, const uint16_t* __restrict__ bias_tiles,
            uint4* __restrict__ out, uint64_t num_tiles, uint32_t Nt) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t t = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < num_tiles;
         t += warps) {
        const uint32_t nt = (uint32_t)(t % Nt);
        const uint16_t* bt = bias_tiles + (uint64_t)nt * 1024 + (lane & 1u) * 8u;
        const uint4 b0 = __ldg(reinterpret_cast<const uint4*>(bt));        // face column 0
        const uint4 b1 = __ldg(reinterpret_cast<const uint4*>(bt + 256));  // face column 1
        const uint4* src = in + t * 128u + lane;
        uint4* dst = out + t * 128u + lane;
        uint4 x0 = __ldcs(src), x1 = __ldcs(src + 32), x2 = __ldcs(src + 64), x3 = __ldcs(src + 96);
        __stcs(dst, add_v(x0, b0));
        __stcs(dst + 32, add_v(x1, b1));
        __stcs(dst + 64, add_v(x2, b0));
        __stcs(dst + 96, add_v(x3, b1));
    }
}

int grid_for(uint64_t work_items) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    uint64_t want = (work_items + 255) / 256;
    uint64_t cap = (uint64_t)sms * 8;  // 8 x 256-thread CTAs per SM
    return (int)(want < cap ? (want ? want : 1) : cap);
}

int check(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        char buf[256];
        snprintf(buf, sizeof buf, "%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

bool ok16(const void* p) { return p && ((uintptr_t)p & 15u) == 0; }

}  // namespace
}  // namespace foil

extern "C" int foil_add_tiles_dev(const uint16_t* a, const uint16_t* b, uint16_t* out,
                                  uint64_t n, void* stream) {
    if (n % 8) {
        foil_set_error(FOIL_ERR_INVALID, "foil_add_tiles_dev: n must be a multiple of 8");
        return FOIL_ERR_INVALID;
    }
    if (n == 0) return FOIL_OK;
    if (!foil::ok16(a) || !foil::ok16(b) || !foil::ok16(out)) {
        foil_set_error(FOIL_ERR_INVALID, "foil_add_tiles_dev: null or misaligned pointer");
        return FOIL_ERR_INVALID;
    }
    uint64_t n8 = n / 8;
    foil::add_kernel<<<foil::grid_for(n8), 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)a, (const uint4*)b, (uint4*)out, n8);
    return foil::check("foil_add_tiles_dev");
}

extern "C" int foil_relu_tiles_dev(const uint16_t* in, uint16_t* out, uint64_t n, void* stream) {
    if (n % 8) {
        foil_set_error(FOIL_ERR_INVALID, "foil_relu_tiles_dev: n must be a multiple of 8");
        return FOIL_ERR_INVALID;
    }
    if (n == 0) return FOIL_OK;
    if (!foil::ok16(in) || !foil::ok16(out)) {
        foil_set_error(FOIL_ERR_INVALID, "foil_relu_tiles_dev: null or misaligned pointer");
        return FOIL_ERR_INVALID;
    }
    uint64_t n8 = n / 8;
    foil::relu_kernel<<<foil::grid_for(n8), 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)in, (uint4*)out, n8);
    return foil::check("foil_relu_tiles_dev");
}

extern "C" int foil_bias_add_tiles_dev(const uint16_t* in, const uint16_t* bias_tiles,
                                       uint16_t* out, uint32_t rows, uint32_t cols,
                                       void* stream) {
    if (rows % 32 || cols % 32) {
        foil_set_error(FOIL_ERR_INVALID, "foil_bias_add_tiles_dev: rows and cols must be multiples of 32");
        return FOIL_ERR_INVALID;
    }
    if (rows == 0 || cols == 0) return FOIL_OK;
    if (!foil::ok16(in) || !foil::ok16(out) || !foil::ok16(bias_tiles)) {
        foil_set_error(FOIL_ERR_INVALID, "foil_bias_add_tiles_dev: null or misaligned pointer");
        return FOIL_ERR_INVALID;
    }
    const uint64_t tiles = (uint64_t)(rows / 32) * (cols / 32);
    foil::bias_kernel<<<foil::grid_for(tiles * 32), 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)in, bias_tiles, (uint4*)out, tiles, cols / 32);
    return foil::check("foil_bias_add_tiles_dev");
}
