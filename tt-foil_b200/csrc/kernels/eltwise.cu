// Element-wise kernels: tile_copy, relu, add_tiles, bias_add, as one
// streaming pipeline on bulk copies.
//
// An SM-issued 16-byte load/store stream tops out at about 0.9 of the HBM
// copy rate on B200 (each SM keeps only so many LSU requests in flight); the
// bulk copy engine moves whole 8-32 KiB chunks per instruction instead.  Each
// CTA owns chunks blockIdx.x, blockIdx.x + gridDim.x, ... and cycles them
// through BUFS shared-memory buffers:
//
//   producer thread:  bulk load chunk -> buffer b         (full[b], tx bytes)
//   compute warps:    op in place in buffer b              (done[b], per warp)
//   producer thread:  bulk store buffer b -> out, then reload b with the
//                     chunk BUFS steps ahead once the store has read it.
//
// tile_copy has no compute stage (the store follows full[b] directly).  The
// arithmetic is the golden's: bf16 widened to fp32, operated on, narrowed
// with round-to-nearest-even and the x86 host's NaN results
// (tests/tile_utils.hpp:33-47, tests/test_relu.cpp:54-59,
// tests/test_add_tiles.cpp:60), bit-exact.  Every wait is bounded; a timeout
// raises the CTA's abort flag and sets kErrWaitTimeout in the error word.
#include <cstring>

#include "eltwise.cuh"

#include "gemm_ptx.cuh"

namespace foil {
namespace stream {
namespace {

using gemm::bulk_commit;
using gemm::bulk_load;
using gemm::bulk_store;
using gemm::bulk_wait_all;
using gemm::bulk_wait_read;
using gemm::mbar_arrive;
using gemm::mbar_drain;
using gemm::mbar_expect_tx;
using gemm::mbar_init;
using gemm::mbar_wait;
using gemm::smem_u32;

// Pipeline shape of one instantiation: BUFS buffers of CHUNK bytes per input
// stream, CTAS CTAs per SM, WARPS compute warps (none for tile_copy).
template <int OP, int BUFS, uint32_t CHUNK, int CTAS, int WARPS>
struct Cfg {
    static constexpr int kStreams = OP == kAdd ? 2 : 1;
    static constexpr int kWarps = OP == kCopy ? 0 : WARPS;
    static constexpr int kThreads = 32 * (1 + kWarps);
    static constexpr uint32_t kStage = BUFS * CHUNK;             // one stream
    static constexpr uint32_t kBarOff = kStreams * kStage;
    static constexpr uint32_t kSmem = kBarOff + 2 * BUFS * 8 + 16;
    static_assert(CHUNK % 2048 == 0 && BUFS >= 2, "pipeline shape");
    static_assert(OP != kBias || (32 * WARPS) % 128 == 0, "bias: whole tiles per compute pass");
};

__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t add2_golden(uint32_t a, uint32_t b) {
    float lo = host_add_f32(bf16_bits_to_f32(a & 0xffffu), bf16_bits_to_f32(b & 0xffffu));
    float hi = host_add_f32(bf16_bits_to_f32(a >> 16), bf16_bits_to_f32(b >> 16));
    return pack_bf16x2(f32_to_bf16_bits(lo), f32_to_bf16_bits(hi));
}
// The golden rounds twice (exact sum -> fp32 -> bf16, round to nearest
// even); a single bf16 rounding of the exact sum gives the same bits for
// two bf16 operands: their exact sum needs more than 24 significant bits
// only when the exponents differ by more than 16, and then the bits between
// the bf16 rounding position and the smaller operand are all equal (zeros
// or, for a difference, ones), so the fp32 rounding can neither create nor
// cross a bf16 tie.  NaN results (NaN operand or inf - inf) take the golden
// path for the host's NaN bits.
__device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    const uint32_t m = r & 0x7fff7fffu;
    if ((m & 0xffffu) > 0x7f80u || (m >> 16) > 0x7f80u) return add2_golden(a, b);
    return r;
}
// `v < 0.0f ? 0.0f : v` per element: -0.0 and NaN pass through unchanged.
__device__ __forceinline__ uint32_t relu1(uint32_t b) { return bf16_bits_to_f32(b) < 0.0f ? 0u : b; }
__device__ __forceinline__ uint32_t relu2(uint32_t w) {
    return relu1(w & 0xffffu) | (relu1(w >> 16) << 16);
}
__device__ __forceinline__ uint4 add_v(uint4 a, uint4 b) {
    return make_uint4(add2(a.x, b.x), add2(a.y, b.y), add2(a.z, b.z), add2(a.w, b.w));
}
__device__ __forceinline__ uint4 relu_v(uint4 a) {
    return make_uint4(relu2(a.x), relu2(a.y), relu2(a.z), relu2(a.w));
}

template <uint32_t CHUNK>
__device__ __forceinline__ uint32_t chunk_bytes(uint64_t chunk, uint64_t bytes) {
    const uint64_t off = chunk * CHUNK;
    return (uint32_t)(bytes - off < CHUNK ? bytes - off : CHUNK);
}

// One CTA: warp 0 lane 0 is the copy producer, warps 1.. compute in place.
// bias: `a` is a tile-layout matrix with Nt tile columns; a 16-byte vector at
// byte offset o lies in tile o / 2048 (tile column (o / 2048) % Nt) as chunk
// c = (o % 2048) / 16 of the tile, face c / 32, face column (c / 32) & 1,
// half-row c & 1.  Its bias is row 0 of that column's bias tile:
// bias_tiles[nt * 1024 + ((c / 32) & 1) * 256 + (c & 1) * 8 + 0..7].
template <int OP, int BUFS, uint32_t CHUNK, int CTAS, int WARPS>
__global__ void __launch_bounds__(Cfg<OP, BUFS, CHUNK, CTAS, WARPS>::kThreads, CTAS)
stream_kernel(const uint8_t* a, const uint8_t* b, uint8_t* out, uint64_t bytes,
              const uint16_t* __restrict__ bias_tiles, uint32_t Nt, uint32_t* err, uint64_t wait_ns) {
    using C = Cfg<OP, BUFS, CHUNK, CTAS, WARPS>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* done = full + BUFS;
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(done + BUFS);
    const uint32_t base = smem_u32(smem);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    if (threadIdx.x == 0) {
        for (int i = 0; i < BUFS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&done[i], C::kWarps > 0 ? C::kWarps : 1);
        }
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Launched with programmatic stream serialization: the set-up above may
    // overlap the previous kernel's tail; global memory only after it.
    griddep_wait();
    griddep_launch_dependents();

    const uint64_t nchunks = (bytes + CHUNK - 1) / CHUNK;
    const uint64_t first = blockIdx.x, step = gridDim.x;
    if (first >= nchunks) return;
    const uint64_t mine = (nchunks - 1 - first) / step + 1;  // chunks of this CTA

    if (warp == 0) {
        if (lane != 0) return;
        auto load = [&](uint64_t k) {
            const int bi = (int)(k % BUFS);
            const uint64_t chunk = first + k * step;
            const uint32_t n = chunk_bytes<CHUNK>(chunk, bytes);
            mbar_expect_tx(&full[bi], n * C::kStreams);
            bulk_load(base + bi * CHUNK, a + chunk * CHUNK, n, &full[bi]);
            if (OP == kAdd) bulk_load(base + C::kStage + bi * CHUNK, b + chunk * CHUNK, n, &full[bi]);
        };
        const uint64_t pro = mine < (uint64_t)BUFS ? mine : (uint64_t)BUFS;
        for (uint64_t k = 0; k < pro; ++k) load(k);
        // Loads are issued for chunks [0, issued).
        uint64_t issued = pro, k = 0;
        bool ok = true;
        for (; k < mine; ++k) {
            const int bi = (int)(k % BUFS);
            const uint32_t ph = (uint32_t)((k / BUFS) & 1u);
            if (!mbar_wait(OP == kCopy ? &full[bi] : &done[bi], ph, abort_flag, err, wait_ns)) {
                ok = false;
                break;
            }
            const uint64_t chunk = first + k * step;
            bulk_store(out + chunk * CHUNK, base + bi * CHUNK, chunk_bytes<CHUNK>(chunk, bytes));
            bulk_commit();
            if (issued < mine) {
                bulk_wait_read();  // buffer bi has been read by its store
                load(issued++);
            }
        }
        if (!ok) {
            // Loads issued for chunks k .. issued - 1 may still land in
            // shared memory: wait (bounded) for each before the CTA's shared
            // memory is released.
            for (uint64_t j = k; j < issued; ++j)
                mbar_drain(&full[j % BUFS], (uint32_t)((j / BUFS) & 1u), 100000000ull);
        }
        bulk_wait_all();
        return;
    }

    // compute warps
    const uint32_t t = threadIdx.x - 32u;
    constexpr uint32_t kT = 32u * C::kWarps;
    for (uint64_t k = 0; k < mine; ++k) {
        const int bi = (int)(k % BUFS);
        const uint32_t ph = (uint32_t)((k / BUFS) & 1u);
        if (!mbar_wait(&full[bi], ph, abort_flag, err, wait_ns)) return;
        const uint64_t chunk = first + k * step;
        const uint32_t nv = chunk_bytes<CHUNK>(chunk, bytes) / 16u;
        uint4* va = reinterpret_cast<uint4*>(smem + bi * CHUNK);
        if (OP == kRelu) {
#pragma unroll 4
            for (uint32_t v = t; v < nv; v += kT) va[v] = relu_v(va[v]);
        } else if (OP == kAdd) {
            const uint4* vb = reinterpret_cast<const uint4*>(smem + C::kStage + bi * CHUNK);
#pragma unroll 4
            for (uint32_t v = t; v < nv; v += kT) va[v] = add_v(va[v], vb[v]);
        } else if (OP == kBias) {
            // A pass of kT vectors covers kT / 128 whole tiles: thread t
            // handles chunk c = t % 128 of tile t / 128 of each pass.
            constexpr uint32_t kPassTiles = kT / 128u;
            uint32_t nt = (uint32_t)((chunk * (CHUNK / 2048u) + t / 128u) % Nt);
            const uint16_t* bt = bias_tiles + ((t >> 5) & 1u) * 256u + (t & 1u) * 8u;
#pragma unroll 4
            for (uint32_t v = t; v < nv; v += kT) {
                const uint4 bv = __ldg(reinterpret_cast<const uint4*>(bt + (uint64_t)nt * 1024u));
                va[v] = add_v(va[v], bv);
                nt += kPassTiles;
                if (nt >= Nt) nt = kPassTiles < Nt ? nt - Nt : nt % Nt;
            }
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&done[bi]);
    }
}

template <int OP, int BUFS, uint32_t CHUNK, int CTAS, int WARPS>
int launch_op(const void* a, const void* b, void* out, uint64_t bytes, const uint16_t* bias_tiles,
              uint32_t Nt, uint32_t* err, cudaStream_t stream) {
    using C = Cfg<OP, BUFS, CHUNK, CTAS, WARPS>;
    auto kern = stream_kernel<OP, BUFS, CHUNK, CTAS, WARPS>;
    const cudaError_t attr = foil_smem_optin((const void*)kern, (int)C::kSmem);
    if (attr != cudaSuccess) return (int)attr;
    const uint64_t nchunks = (bytes + CHUNK - 1) / CHUNK;
    const uint64_t cap = (uint64_t)foil_sm_count() * CTAS;
    const unsigned grid = (unsigned)(nchunks < cap ? nchunks : cap);
    // add_tiles measured 0.7 % slower with it (6110 against 6155 GB/s); the
    // others 0.7-1.7 % faster.
    static const bool pdl = OP != kAdd && pdl_enabled("FOIL_STREAM_PDL");
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(C::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = la;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<const uint8_t*>(a),
                                             static_cast<const uint8_t*>(b), static_cast<uint8_t*>(out), bytes,
                                             bias_tiles, Nt, err, foil_wait_limit_ns());
    const cudaError_t last = cudaGetLastError();
    return (int)(e != cudaSuccess ? e : last);
}

}  // namespace

int launch(Op op, const void* a, const void* b, void* out, uint64_t bytes, const uint16_t* bias_tiles,
           uint32_t Nt, uint32_t* err, cudaStream_t stream) {
    if (bytes == 0) return 0;
    switch (op) {
        case kCopy: return launch_op<kCopy, 4, 32768, 1, 0>(a, b, out, bytes, bias_tiles, Nt, err, stream);
        case kRelu: return launch_op<kRelu, 6, 16384, 2, 4>(a, b, out, bytes, bias_tiles, Nt, err, stream);
        case kAdd: return launch_op<kAdd, 4, 8192, 2, 12>(a, b, out, bytes, bias_tiles, Nt, err, stream);
        case kBias: return launch_op<kBias, 6, 16384, 2, 12>(a, b, out, bytes, bias_tiles, Nt, err, stream);
    }
    return (int)cudaErrorInvalidValue;
}

}  // namespace stream
}  // namespace foil
