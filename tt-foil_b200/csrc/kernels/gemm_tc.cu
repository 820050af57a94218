// Tiled bf16 GEMM on Blackwell tensor cores (tcgen05 + TMEM + TMA), reading
// and writing the tt-foil tile layout directly (no relayout pass).
//
//   C (Mt x Nt tiles) = A (Mt x Kt tiles) . B (Kt x Nt tiles)
//   fp32 accumulation in TMEM, bf16 output, optional fused bias + relu.
//
// Replaces the reference's matmul pipeline: reader (examples/matmul_mnk/
// kernels/reader.cpp:28-57), compute (compute.cpp:23-53, matmul_tiles with
// fp32 DST accumulation) and writer (writer.cpp:16-34), and — fused into the
// epilogue — bias_add (examples/bias_add/kernels/compute.cpp:19-42) and relu
// (examples/relu/kernels/compute.cpp:19-45).
//
// How the tile layout feeds tcgen05 without a relayout pass
// ---------------------------------------------------------
// A face row is 16 bf16 = 32 bytes, which is exactly one SWIZZLE_32B atom
// row and one UMMA K-step (K = 16).  Both operands are staged so that every
// K-step is a canonical UMMA operand:
//
//  * A (rows = m, contiguous = k: K-major SW32).  K-step (kt, fc) of a stage
//    holds face column fc of the 4 A tiles (mt0..mt0+3, kt): 128 rows x 32 B,
//    8-row groups 256 B apart (SBO = 256 B).
//  * B (rows = k, contiguous = n: MN-major SW32).  K-step (kt, fr) holds face
//    row fr of the 8 B tiles (kt, nt0..nt0+7): 16 atoms of 16 n x 16 k
//    (512 B each, LBO = 512 B between atoms along n, SBO = 256 B along k).
//  A K-step (kt, f) pairs A face column f with B face row f, i.e. the K
//  range kt*32 + f*16 + [0,16).
//
// In both cases a whole 16x16 face (512 contiguous bytes of the tile stream)
// lands as one 512-byte block of shared memory, with the 32-byte swizzle
// (16-byte halves of rows 4..7 of every 8-row group swapped) applied in the
// destination address.  Producer warps therefore copy one face per warp
// instruction with 16-byte cp.async: each warp access is 512 contiguous
// global bytes, i.e. four full 128-byte L2 requests.  (A TMA tensor copy of
// the same operand has a 32-byte inner box — one face row — and costs one L2
// request per 32 bytes, which made L2 tag lookups the limiter.)
//
// Kernel organisation (persistent, warp-specialised, 1 CTA per SM)
// ------------------------------------------------------------------
//  warps 0..3  producers     (4-stage smem ring, 48 KiB per stage, 96 faces)
//  warp 4      MMA issuer    (tcgen05.mma 128x256x16, commits free stages)
//              and TMEM owner
//  warps 5..8  epilogue      (tcgen05.ld -> bf16 (+bias, relu) -> global)
//  TMEM holds two 128x256 fp32 accumulators (512 columns) so the epilogue of
//  tile i overlaps the main loop of tile i+1.  Output tiles of 128x256 are
//  visited in bands of 8 column-blocks for L2 reuse.  Two 2-SM variants
//  follow (cta_group::2, 256x256 and 256x512 pair tiles); launch() picks one
//  by shape.
//
// Multi-GPU: with peer copies of C (other GPUs' buffers, Params::peer_c) the
// kernel is also its own all-gather.  Every output tile goes to the peers over
// NVLink as well, from the epilogue (256-column kernels, whose second TMEM
// accumulator hides the stores) or from four pusher warps that copy finished
// tiles out of L2 (the 512-column kernel, whose epilogue holds TMEM).
//
// Every mbarrier wait is bounded (2 s of wall time); on expiry the kernel
// records kErrWaitTimeout in the error word, all roles leave their loops,
// in-flight copies and MMAs are drained and TMEM is freed.
#include <mutex>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemm_ptx.cuh"
#include "../../../include/foil_c.h"

extern "C" void foil_set_error(int status, const char* msg);

namespace foil {
namespace gemm {

// --------------------------------------------------------------- kernel ---
constexpr int kBM = 128;           // rows per CTA tile (4 tile-rows)
constexpr int kBN = 256;           // cols per CTA tile (8 tile-cols)
constexpr int kBKT = 2;            // K tiles per stage (K = 64)
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBKT * 32 * 2;  // 16 KiB
constexpr int kBBytes = kBN * kBKT * 32 * 2;  // 32 KiB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kProdWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kEpiWarp0 = 5;
constexpr int kThreads = 9 * 32;
static_assert(kThreads / 32 == kEpiWarp0 + 4, "four epilogue warps follow the MMA warp");
constexpr int kFacesPerStage = 96;  // 32 A faces + 64 B faces
constexpr int kTmemCols = 512;
constexpr int kBandN = 8;           // column-blocks per raster band
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;

struct Params {
    const uint16_t* a;
    const uint16_t* b;
    uint16_t* c;
    const uint16_t* bias;
    uint32_t Mt, Kt, Nt;
    uint32_t m_blocks, n_blocks;
    int relu;
    uint32_t* err;
    // Other GPUs' copies of C (peer-mapped, same layout as c): every output
    // tile is also stored there, so the kernel is its own all-gather.
    uint16_t* peer_c[kMaxPeers];
    uint32_t npeers;
    // Or: an NVLink multicast address of C (same layout as c), bound to every
    // GPU's copy; one multimem store per 16 bytes reaches all of them.
    uint16_t* mc_c;
    uint32_t wide_stores;  // c and every peer_c 32-byte aligned: 256-bit stores
    uint64_t wait_ns;      // wall-time limit of each bounded wait
};

__device__ __forceinline__ void tile_coords(uint32_t tile, uint32_t m_blocks, uint32_t n_blocks,
                                            uint32_t& mb, uint32_t& nb, uint32_t bandn = kBandN) {
    const uint32_t band_tiles = m_blocks * bandn;
    const uint32_t band = tile / band_tiles;
    const uint32_t inner = tile - band * band_tiles;
    const uint32_t width = min(bandn, n_blocks - band * bandn);
    mb = inner / width;
    nb = band * bandn + (inner - mb * width);
}

// out = bf16(acc) [+ bias -> bf16] [relu], the composition of the reference
// goldens (matmul, bias_add, relu), per element.
__device__ __forceinline__ uint32_t epi1(uint32_t acc_bits, uint32_t bias_bits, bool has_bias,
                                         bool relu) {
    uint32_t o = f32_to_bf16_bits(__uint_as_float(acc_bits));
    if (has_bias) o = f32_to_bf16_bits(host_add_f32(bf16_bits_to_f32(o), bf16_bits_to_f32(bias_bits)));
    if (relu && bf16_bits_to_f32(o) < 0.0f) o = 0u;
    return o;
}

// Epilogue of one warp: the 32 accumulator rows of TMEM lane quadrant `t_row`
// (tile row mt) x 256 columns (tile columns nt0 .. nt0+7) -> bf16 (+bias,
// relu) -> the tile stream.  Lane = row inside the tile: face row fr = lane/16,
// row r0 = lane%16; each lane writes one 32-byte face row per face.
template <bool kPeers = true>
__device__ __forceinline__ void store_tile_row(const Params& p, uint32_t t_row, uint32_t mt,
                                               uint32_t nt0, uint32_t lane) {
    const uint32_t fr = lane >> 4, r0 = lane & 15u;
    const bool has_bias = p.bias != nullptr;
    const bool relu = p.relu != 0;
#pragma unroll 1
    for (uint32_t nt_l = 0; nt_l < 8; ++nt_l) {
        uint32_t v0[16], v1[16];
        tmem_ld16(t_row + nt_l * 32u, v0);
        tmem_ld16(t_row + nt_l * 32u + 16u, v1);
        tmem_ld_wait();
        const uint32_t nt = nt0 + nt_l;
        if (mt < p.Mt && nt < p.Nt) {
            uint32_t bias_w[16];
            if (has_bias) {
                const uint4* bp = reinterpret_cast<const uint4*>(p.bias + nt * 32u);
                uint4 b0 = __ldg(bp), b1 = __ldg(bp + 1), b2 = __ldg(bp + 2), b3 = __ldg(bp + 3);
                bias_w[0] = b0.x; bias_w[1] = b0.y; bias_w[2] = b0.z; bias_w[3] = b0.w;
                bias_w[4] = b1.x; bias_w[5] = b1.y; bias_w[6] = b1.z; bias_w[7] = b1.w;
                bias_w[8] = b2.x; bias_w[9] = b2.y; bias_w[10] = b2.z; bias_w[11] = b2.w;
                bias_w[12] = b3.x; bias_w[13] = b3.y; bias_w[14] = b3.z; bias_w[15] = b3.w;
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) bias_w[i] = 0u;
            }
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                // face column 0: columns 2i, 2i+1 ; face column 1: 16+2i, 17+2i
                uint32_t bl0 = bias_w[i] & 0xffffu, bh0 = bias_w[i] >> 16;
                uint32_t bl1 = bias_w[8 + i] & 0xffffu, bh1 = bias_w[8 + i] >> 16;
                o[i] = pack_bf16x2(epi1(v0[2 * i], bl0, has_bias, relu),
                                   epi1(v0[2 * i + 1], bh0, has_bias, relu));
                o[8 + i] = pack_bf16x2(epi1(v1[2 * i], bl1, has_bias, relu),
                                       epi1(v1[2 * i + 1], bh1, has_bias, relu));
            }
            // Row r0 of face (fr, 0) at t0 and of face (fr, 1) at t0 + 256
            // (elements): 32 contiguous bytes each, one 256-bit store, so a
            // half-warp writes a whole 512-byte face per instruction (full
            // lines, also over NVLink for the peer copies).
            // (Buffers only 16-byte aligned take two 128-bit stores per row.)
            const uint64_t t0 = ((uint64_t)mt * p.Nt + nt) * 1024u + fr * 512u + r0 * 16u;
            if (kPeers && p.mc_c) {
                st_multimem_v4(p.mc_c + t0, o[0], o[1], o[2], o[3]);
                st_multimem_v4(p.mc_c + t0 + 8u, o[4], o[5], o[6], o[7]);
                st_multimem_v4(p.mc_c + t0 + 256u, o[8], o[9], o[10], o[11]);
                st_multimem_v4(p.mc_c + t0 + 264u, o[12], o[13], o[14], o[15]);
            } else if (p.wide_stores) {
                st_global_v8(p.c + t0, o);
                st_global_v8(p.c + t0 + 256u, o + 8);
#pragma unroll
                for (uint32_t d = 0; d < kMaxPeers; ++d) {
                    if (kPeers && d < p.npeers) {
                        st_global_v8(p.peer_c[d] + t0, o);
                        st_global_v8(p.peer_c[d] + t0 + 256u, o + 8);
                    }
                }
            } else {
                uint4* d0 = reinterpret_cast<uint4*>(p.c + t0);
                uint4* d1 = reinterpret_cast<uint4*>(p.c + t0 + 256u);
                d0[0] = make_uint4(o[0], o[1], o[2], o[3]);
                d0[1] = make_uint4(o[4], o[5], o[6], o[7]);
                d1[0] = make_uint4(o[8], o[9], o[10], o[11]);
                d1[1] = make_uint4(o[12], o[13], o[14], o[15]);
#pragma unroll
                for (uint32_t d = 0; d < kMaxPeers; ++d) {
                    if (kPeers && d < p.npeers) {
                        uint4* e0 = reinterpret_cast<uint4*>(p.peer_c[d] + t0);
                        uint4* e1 = reinterpret_cast<uint4*>(p.peer_c[d] + t0 + 256u);
                        e0[0] = make_uint4(o[0], o[1], o[2], o[3]);
                        e0[1] = make_uint4(o[4], o[5], o[6], o[7]);
                        e1[0] = make_uint4(o[8], o[9], o[10], o[11]);
                        e1[1] = make_uint4(o[12], o[13], o[14], o[15]);
                    }
                }
            }
        }
    }
}

// The single-SM GEMM as a device function: CTA `cta` of `ncta` (persistent
// over the tiles), kThreads threads, kSmemBytes of dynamic shared memory at
// smem_raw.  gemm_tiles_kernel runs it as block blockIdx.x of gridDim.x; the
// multi-core dispatch kernel (below) runs it on one CTA of a cluster.
__device__ __forceinline__ void gemm_tiles_body(const Params& p, uint32_t cta, uint32_t ncta, uint8_t* smem_raw) {
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* tfull = empty + kStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kProdWarps * 32);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched with programmatic stream serialization, the set-up above may
    // overlap the previous kernel's tail; global memory is touched only after
    // that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();

    const uint32_t num_tiles = p.m_blocks * p.n_blocks;
    const uint32_t num_kb = (p.Kt + kBKT - 1) / kBKT;

    if (warp < kProdWarps) {
        // ---------------------------------------------------- producers
        // Lane l copies bytes [16 l, 16 l + 16) of each face: face row
        // r0 = l / 2, half h = l % 2, stored at r0 * 32 + 16 * (h ^ bit 2 of r0).
        const uint32_t src_lane = lane * 16u;
        const uint32_t dst_lane = (lane >> 1) * 32u + ((((lane & 1u) ^ ((lane >> 3) & 1u))) << 4);
        const char* a_g = reinterpret_cast<const char*>(p.a);
        const char* b_g = reinterpret_cast<const char*>(p.b);
        uint32_t stage = 0, phase = 0;
        for (uint32_t tile = cta; tile < num_tiles; tile += ncta) {
            uint32_t mb, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
            bool ok = true;
            for (uint32_t kb = 0; kb < num_kb; ++kb) {
                bool w = true;
                if (lane == 0) w = mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns);
                if (__shfl_sync(0xffffffffu, w ? 1 : 0, 0) == 0) {
                    ok = false;
                    break;
                }
                const uint32_t a_s = smem_u32(smem + stage * kStageBytes);
                const uint32_t b_s = a_s + kABytes;
                const uint32_t kt0 = kb * kBKT;
#pragma unroll
                for (int i = 0; i < kFacesPerStage / kProdWarps; ++i) {
                    const uint32_t f = warp + kProdWarps * i;
                    const char* src;
                    uint32_t dst;
                    bool valid;
                    if (i < 32 / kProdWarps) {  // A face: (mt_l, ktl, fr, fc)
                        const uint32_t mt_l = f >> 3, ktl = (f >> 2) & 1u, fr = (f >> 1) & 1u,
                                       fc = f & 1u;
                        const uint32_t mt = mb * 4u + mt_l, kt = kt0 + ktl;
                        valid = mt < p.Mt && kt < p.Kt;
                        src = a_g + (((uint64_t)mt * p.Kt + kt) * 1024u + (fr * 2u + fc) * 256u) * 2u;
                        dst = a_s + (ktl * 2u + fc) * 4096u + (mt_l * 32u + fr * 16u) * 32u;
                    } else {  // B face: (ktl, nt_l, fr, fc)
                        const uint32_t g = f - 32u;
                        const uint32_t ktl = g >> 5, nt_l = (g >> 2) & 7u, fr = (g >> 1) & 1u,
                                       fc = g & 1u;
                        const uint32_t kt = kt0 + ktl, nt = nb * 8u + nt_l;
                        valid = kt < p.Kt && nt < p.Nt;
                        src = b_g + (((uint64_t)kt * p.Nt + nt) * 1024u + (fr * 2u + fc) * 256u) * 2u;
                        dst = b_s + fr * 16384u + ktl * 8192u + (nt_l * 2u + fc) * 512u;
                    }
                    cp_async16(dst + dst_lane, valid ? src + src_lane : a_g, valid ? 16u : 0u);
                }
                cp_async_arrive(&full[stage]);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            constexpr uint32_t idesc = make_idesc(kBM, kBN);
            constexpr uint64_t a_base = smem_desc_base(16, 256);   // K-major SW32
            constexpr uint64_t b_base = smem_desc_base(512, 256);  // MN-major SW32
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t tile = cta; ok && tile < num_tiles; tile += ncta) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kBN;
                for (uint32_t kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    // The stage was written by cp.async (generic proxy); the MMA
                    // reads it through the async proxy.
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * kStageBytes);
                    const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
                    for (uint32_t s = 0; s < 4; ++s) {
                        const uint32_t a_off = s * 4096u;
                        const uint32_t b_off = (s & 1u) * 16384u + (s >> 1) * 8192u;
                        const uint64_t ad = a_base | (uint64_t)(((a_addr + a_off) >> 4) & 0x3fffu);
                        const uint64_t bd = b_base | (uint64_t)(((b_addr + b_off) >> 4) & 0x3fffu);
                        tc_mma(d_tmem, ad, bd, idesc, (kb | s) != 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tfull[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // Drain all MMAs issued by this thread before TMEM is released.
            tc_commit(drain);
            mbar_drain(drain, 0, 100000000ull);
        }
    } else {
        // ---------------------------------------------------- epilogue
        const uint32_t q = warp & 3u;  // TMEM lane quadrant this warp may access
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t tile = cta; tile < num_tiles; tile += ncta) {
            uint32_t mb, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
            // One lane waits; the warp then proceeds converged (tcgen05.ld is
            // a warp-wide .sync.aligned instruction).
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            store_tile_row(p, tmem_base + ((q * 32u) << 16) + acc * kBN, mb * 4 + q, nb * 8, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        // Peer copies of C: make this thread's remote stores visible
        // system-wide before the kernel's completion is observed.
        if (p.npeers || p.mc_c) __threadfence_system();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols)
                     : "memory");
    }
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_tiles_kernel(const Params p) {
    extern __shared__ uint8_t smem_raw[];
    gemm_tiles_body(p, blockIdx.x, gridDim.x, smem_raw);
}

// ============================================== multi-core dispatch kernel ===
// One CTA per logical core of an execute (CoreProgram), all CTAs of one
// cluster, hence resident together: a consumer core may wait for a flag that
// a producer core of the same launch sets.  Replaces the reference's
// fire-all-then-poll dispatch of several core kernels (src/dispatch.cpp:
// 223-274) for programs that talk to each other (the matmul_2core_mcast
// producer / consumer pair, examples/matmul_2core_mcast/kernels/
// reader_producer.cpp:60-82, reader_consumer.cpp:38-44; the noc_passthrough
// producer / consumer, examples/noc_passthrough/kernels/producer.cpp:29-58,
// consumer.cpp:22-38) and for the scalar add_two_numbers kernels.
struct CoreLaunch {
    CoreProgram core[kMaxCores];
    Params gemm[kMaxCores];  // the GEMM of core i (Mt = 0: none)
    uint32_t* err;
    uint32_t* status;
    uint64_t gate_wait_ns;
};
static_assert(sizeof(CoreLaunch) <= 4096, "multi-core launch parameters must fit the classic 4 KiB limit");

// Bounded acquire poll of a flag in global memory: true once it reads
// `want` (want 0: any non-zero value), false after limit_ns.
__device__ __forceinline__ bool wait_flag_acquire(const uint32_t* flag, uint32_t want, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
#pragma unroll 1
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (want == 0u ? v != 0u : v == want) return true;
        if (global_ns() - t0 > limit_ns) return false;
        __nanosleep(256);
    }
}

// Block-wide copy: 16-byte units when both ends and the size allow, else
// 4-byte words (the host checks 4-byte alignment and size).
__device__ __forceinline__ void copy_block(const void* src, void* dst, uint64_t bytes) {
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | bytes) & 15u) == 0) {
        const uint4* s = static_cast<const uint4*>(src);
        uint4* d = static_cast<uint4*>(dst);
        for (uint64_t i = threadIdx.x; i < bytes / 16u; i += blockDim.x) d[i] = s[i];
    } else {
        const uint32_t* s = static_cast<const uint32_t*>(src);
        uint32_t* d = static_cast<uint32_t*>(dst);
        for (uint64_t i = threadIdx.x; i < bytes / 4u; i += blockDim.x) d[i] = s[i];
    }
}

__global__ void __launch_bounds__(kThreads, 1) cores_kernel(const __grid_constant__ CoreLaunch L) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t go;
    const CoreProgram& c = L.core[blockIdx.x];
    if (threadIdx.x == 0) {
        const bool ok = c.gate == nullptr || wait_flag_acquire(c.gate, c.gate_value, L.gate_wait_ns);
        if (!ok) {
            atomicOr(L.err, kErrWaitTimeout);
            L.status[blockIdx.x] = 1u;
        }
        go = ok ? 1u : 0u;
        // Scalar steps, in program order on one thread, after the gate's
        // acquire (a consumer reads what the producer sent before its flag).
        if (ok) {
            for (uint32_t i = 0; i < c.nwords && i < kMaxWordSteps; ++i) {
                const WordStep& w = c.words[i];
                uint32_t v;
                switch (w.code) {
                    case kWordAdd: v = *w.a + *w.b; break;
                    case kWordMul: v = *w.a * *w.b; break;
                    case kWordSet: v = w.imm; break;
                    default: v = *w.a * w.imm; break;
                }
                *w.out = v;
            }
        }
    }
    __syncthreads();
    if (!go) return;
    if (c.fwd_bytes) {
        // (Stage and) forward to the peer core, then publish its flag: the
        // flag's release store orders every thread's copies (joined by the
        // CTA barrier and made GPU-visible by the fence) before it.
        if (c.fwd_stage) {
            copy_block(c.fwd_src, c.fwd_stage, c.fwd_bytes);
            __syncthreads();
            copy_block(c.fwd_stage, c.fwd_peer, c.fwd_bytes);
        } else {
            copy_block(c.fwd_src, c.fwd_peer, c.fwd_bytes);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            const uint32_t v = *reinterpret_cast<const volatile uint32_t*>(c.flag_src);
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(c.flag_dst), "r"(v) : "memory");
        }
        __syncthreads();
    }
    if (c.Mt) gemm_tiles_body(L.gemm[blockIdx.x], 0, 1, smem_raw);
}

int launch_cores(const CoreProgram* cores, uint32_t ncores, uint32_t* err, uint32_t* core_status,
                 uint64_t gate_wait_ns, cudaStream_t stream) {
    if (ncores == 0 || ncores > kMaxCores) {
        foil_set_error(FOIL_ERR_INVALID, "tt-foil: multi-core execute takes 1 to 8 cores");
        return FOIL_ERR_INVALID;
    }
    if (foil_smem_optin((const void*)cores_kernel, kSmemBytes) != cudaSuccess) {
        foil_set_error(FOIL_ERR_CUDA, "tt-foil: cudaFuncSetAttribute failed (multi-core execute)");
        return FOIL_ERR_CUDA;
    }
    CoreLaunch L;
    memset(&L, 0, sizeof L);
    bool any_gemm = false;
    for (uint32_t i = 0; i < ncores; ++i) {
        if (cores[i].nwords > kMaxWordSteps) {
            foil_set_error(FOIL_ERR_INVALID, "tt-foil: too many scalar steps on one core");
            return FOIL_ERR_INVALID;
        }
        any_gemm |= cores[i].Mt != 0;
        L.core[i] = cores[i];
        Params& p = L.gemm[i];
        p.a = cores[i].a;
        p.b = cores[i].b;
        p.c = cores[i].c;
        p.bias = nullptr;
        p.Mt = cores[i].Mt;
        p.Kt = cores[i].Kt;
        p.Nt = cores[i].Nt;
        p.m_blocks = (p.Mt + 3) / 4;
        p.n_blocks = (p.Nt + 7) / 8;
        p.relu = 0;
        p.err = err;
        p.wait_ns = foil_wait_limit_ns();
        p.npeers = 0;
        p.mc_c = nullptr;
        p.wide_stores = ((uintptr_t)p.c & 31u) == 0 ? 1u : 0u;
    }
    L.err = err;
    L.status = core_status;
    L.gate_wait_ns = gate_wait_ns;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = dim3(ncores, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    // Shared memory only serves the GEMM stages.
    cfg.dynamicSmemBytes = any_gemm ? kSmemBytes : 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ncores;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, cores_kernel, L) != cudaSuccess) {
        char buf[256];
        snprintf(buf, sizeof buf, "tt-foil: multi-core execute launch failed: %s",
                 cudaGetErrorString(cudaGetLastError()));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

// ============================================================ 2-SM kernel ===
// The same tile-layout GEMM on CTA pairs (cluster of 2) with the 2-SM UMMA:
// the even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16)
// whose A rows 0..127 / 128..255 come from the even / odd CTA's shared memory
// and whose B columns 0..127 / 128..255 likewise; each CTA's TMEM receives its
// 128 rows x 256 columns.  Per k-block (K = 64) a CTA stages 16 KiB of A and
// 16 KiB of B (a third less L2 traffic per FLOP than 128x256 on one SM), so
// seven stages fit in shared memory.
//
// Synchronisation: each CTA's producers arrive on their own full[s] through
// cp.async.mbarrier.arrive; in the odd CTA a relay lane waits for it, fences
// the async proxy and arrives (relaxed, cluster scope) on the even CTA's
// full[s], which therefore counts 128 + 1 arrivals.  The even CTA's MMA commits are multicast to both CTAs'
// empty[s] / tfull[b]; both CTAs' epilogue warps arrive on the even CTA's
// tempty[b] (8 arrivals).  A cluster barrier after set-up and before exit
// keeps both CTAs alive while the other may touch their shared memory.
constexpr int kPStages = 7;
constexpr int kPABytes = 128 * kBKT * 32 * 2;  // 16 KiB: 128 rows x K 64
constexpr int kPBBytes = 128 * kBKT * 32 * 2;  // 16 KiB: 128 cols x K 64
constexpr int kPStageBytes = kPABytes + kPBBytes;
constexpr int kPFaces = 64;                    // 32 A + 32 B faces per CTA
constexpr int kPSmemBytes = kPStages * kPStageBytes + 1024 + 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_pair_kernel(const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPStages * kPStageBytes);
    uint64_t* empty = full + kPStages;
    uint64_t* tfull = empty + kPStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t pair_id = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&full[s], kProdWarps * 32 + (leader ? 1 : 0));
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 8);
        }
        mbar_init(drain, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncwarp();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched with programmatic stream serialization, the set-up above may
    // overlap the previous kernel's tail; global memory is touched only after
    // that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();

    const uint32_t num_tiles = p.m_blocks * p.n_blocks;  // m_blocks = 256-row pairs
    const uint32_t num_kb = (p.Kt + kBKT - 1) / kBKT;

    if (warp < kProdWarps) {
        // ---------------------------------------------------- producers
        const uint32_t src_lane = lane * 16u;
        const uint32_t dst_lane = (lane >> 1) * 32u + ((((lane & 1u) ^ ((lane >> 3) & 1u))) << 4);
        const char* a_g = reinterpret_cast<const char*>(p.a);
        const char* b_g = reinterpret_cast<const char*>(p.b);
        uint32_t stage = 0, phase = 0;
        for (uint32_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
            uint32_t mp, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mp, nb);
            const uint32_t mt0 = (mp * 2u + rank) * 4u;  // this CTA's 4 tile rows
            const uint32_t nt0 = nb * 8u + rank * 4u;    // this CTA's 4 B tile columns
            bool ok = true;
            for (uint32_t kb = 0; kb < num_kb; ++kb) {
                bool w = true;
                if (lane == 0) w = mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns);
                if (__shfl_sync(0xffffffffu, w ? 1 : 0, 0) == 0) {
                    ok = false;
                    break;
                }
                const uint32_t a_s = smem_u32(smem + stage * kPStageBytes);
                const uint32_t b_s = a_s + kPABytes;
                const uint32_t kt0 = kb * kBKT;
#pragma unroll
                for (int i = 0; i < kPFaces / kProdWarps; ++i) {
                    const uint32_t f = warp + kProdWarps * i;
                    const char* src;
                    uint32_t dst;
                    bool valid;
                    if (i < 32 / kProdWarps) {  // A face: (mt_l, ktl, fr, fc)
                        const uint32_t mt_l = f >> 3, ktl = (f >> 2) & 1u, fr = (f >> 1) & 1u,
                                       fc = f & 1u;
                        const uint32_t mt = mt0 + mt_l, kt = kt0 + ktl;
                        valid = mt < p.Mt && kt < p.Kt;
                        src = a_g + (((uint64_t)mt * p.Kt + kt) * 1024u + (fr * 2u + fc) * 256u) * 2u;
                        dst = a_s + (ktl * 2u + fc) * 4096u + (mt_l * 32u + fr * 16u) * 32u;
                    } else {  // B face: (ktl, nt_l, fr, fc)
                        const uint32_t g = f - 32u;
                        const uint32_t ktl = g >> 4, nt_l = (g >> 2) & 3u, fr = (g >> 1) & 1u,
                                       fc = g & 1u;
                        const uint32_t kt = kt0 + ktl, nt = nt0 + nt_l;
                        valid = kt < p.Kt && nt < p.Nt;
                        src = b_g + (((uint64_t)kt * p.Nt + nt) * 1024u + (fr * 2u + fc) * 256u) * 2u;
                        dst = b_s + fr * 8192u + ktl * 4096u + (nt_l * 2u + fc) * 512u;
                    }
                    cp_async16(dst + dst_lane, valid ? src + src_lane : a_g, valid ? 16u : 0u);
                }
                cp_async_arrive(&full[stage]);
                if (++stage == kPStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == kMmaWarp) {
        if (lane == 0 && !leader) {
            // ---------------------------------- relay (odd CTA): full -> leader
            const uint32_t remote_full0 = map_to_rank(&full[0], 0);
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (uint32_t tile = pair_id; ok && tile < num_tiles; tile += num_pairs) {
                for (uint32_t kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    // Operands written by cp.async (generic proxy) are read by
                    // the partner's tensor cores (async proxy).
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive_remote_relaxed(remote_full0 + stage * 8u);
                    if (++stage == kPStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        } else if (lane == 0) {
            // ------------------------------------- MMA issuer (even CTA)
            constexpr uint32_t idesc = make_idesc(256, kBN);
            constexpr uint64_t a_base = smem_desc_base(16, 256);   // K-major SW32
            constexpr uint64_t b_base = smem_desc_base(512, 256);  // MN-major SW32
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t tile = pair_id; ok && tile < num_tiles; tile += num_pairs) {
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kBN;
                for (uint32_t kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_cluster(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * kPStageBytes);
                    const uint32_t b_addr = a_addr + kPABytes;
#pragma unroll
                    for (uint32_t s = 0; s < 4; ++s) {
                        const uint32_t a_off = s * 4096u;
                        const uint32_t b_off = (s & 1u) * 8192u + (s >> 1) * 4096u;
                        const uint64_t ad = a_base | (uint64_t)(((a_addr + a_off) >> 4) & 0x3fffu);
                        const uint64_t bd = b_base | (uint64_t)(((b_addr + b_off) >> 4) & 0x3fffu);
                        tc_mma_pair(d_tmem, ad, bd, idesc, (kb | s) != 0u);
                    }
                    tc_commit_pair_mc(&empty[stage], 0x3);
                    if (++stage == kPStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit_pair_mc(&tfull[acc], 0x3);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            tc_commit_pair(drain);
            mbar_drain(drain, 0, 100000000ull);
        }
    } else {
        // ---------------------------------------------------- epilogue
        const uint32_t q = warp & 3u;
        const uint32_t remote_tempty0 = map_to_rank(&tempty[0], 0);
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
            uint32_t mp, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mp, nb);
            bool ok = true;
            if (lane == 0) ok = mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            store_tile_row(p, tmem_base + ((q * 32u) << 16) + acc * kBN, (mp * 2u + rank) * 4u + q,
                           nb * 8u, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(remote_tempty0 + acc * 8u);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        // Peer copies of C: make this thread's remote stores visible
        // system-wide before the kernel's completion is observed.
        if (p.npeers || p.mc_c) __threadfence_system();
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// ------------------------------------------------------------------ host ---
static int check_launch(const char* what, cudaError_t launch_err = cudaSuccess) {
    cudaError_t e = cudaGetLastError();
    if (launch_err != cudaSuccess) e = launch_err;
    if (e != cudaSuccess) {
        char buf[256];
        snprintf(buf, sizeof buf, "%s: launch failed: %s", what, cudaGetErrorString(e));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

// ============================================= 2-SM kernel, 512 columns ===
// The pair tile widened to 256 x 512: per K-step the even CTA issues two
// tcgen05.mma.cta_group::2 of N = 256 (column halves h = 0, 1) on the same A
// rows, into TMEM columns [256 h, 256 h + 256) of both CTAs.  Per k-block a
// CTA stages 16 KiB of A and 32 KiB of B (its 128 columns of each half) for
// twice the MMAs of the 256 x 256 tile: a quarter fewer L2 -> SM bytes per
// FLOP, the operand feed's limit.  The 512 accumulator columns leave no room
// for a second TMEM buffer, so the MMAs of a tile wait for the previous
// tile's epilogue; eight epilogue warps (one per TMEM lane quadrant and
// column half) keep that short, and the producers keep loading meanwhile.
constexpr int kWStages = 4;
constexpr int kWABytes = 128 * kBKT * 32 * 2;      // 16 KiB: 128 rows x K 64
constexpr int kWBBytes = 2 * 128 * kBKT * 32 * 2;  // 32 KiB: 2 halves x 128 cols x K 64
constexpr int kWStageBytes = kWABytes + kWBBytes;
constexpr int kWFaces = 96;                        // 32 A + 64 B faces per CTA
constexpr int kWEpiWarps = 8;
constexpr int kWThreads = (5 + kWEpiWarps) * 32;
// With peer copies of C, four more warps ("pushers") copy each finished tile
// from this GPU's C (still in L2) to every peer copy while the next tile
// computes, so the NVLink stores never hold TMEM.
constexpr int kWPushWarps = 4;
constexpr int kWThreadsPush = kWThreads + kWPushWarps * 32;
constexpr int kWSmemBytes = kWStages * kWStageBytes + 1024 + 256;
constexpr int kWBandN = 4;                         // 512-column blocks per raster band

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kWThreadsPush, 1)
gemm_pair_wide_kernel(const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWStages * kWStageBytes);
    uint64_t* empty = full + kWStages;
    uint64_t* tfull = empty + kWStages;
    uint64_t* tempty = tfull + 1;
    uint64_t* drain = tempty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;
    volatile uint32_t* epi_done = tmem_slot + 2;  // epilogue warp-tiles written to C

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t pair_id = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    const bool pushers = blockDim.x == (uint32_t)kWThreadsPush && (p.npeers > 0 || p.mc_c != nullptr);

    if (threadIdx.x == 0) {
        *epi_done = 0u;
        for (int s = 0; s < kWStages; ++s) {
            mbar_init(&full[s], kProdWarps * 32 + (leader ? 1 : 0));
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(tempty, 2 * kWEpiWarps);
        mbar_init(drain, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched with programmatic stream serialization, the set-up above may
    // overlap the previous kernel's tail; global memory is touched only after
    // that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();

    const uint32_t num_tiles = p.m_blocks * p.n_blocks;  // 256-row x 512-column blocks
    const uint32_t num_kb = (p.Kt + kBKT - 1) / kBKT;

    if (warp < kProdWarps) {
        // ---------------------------------------------------- producers
        const uint32_t src_lane = lane * 16u;
        const uint32_t dst_lane = (lane >> 1) * 32u + ((((lane & 1u) ^ ((lane >> 3) & 1u))) << 4);
        const char* a_g = reinterpret_cast<const char*>(p.a);
        const char* b_g = reinterpret_cast<const char*>(p.b);
        uint32_t stage = 0, phase = 0;
        for (uint32_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
            uint32_t mp, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mp, nb, kWBandN);
            const uint32_t mt0 = (mp * 2u + rank) * 4u;  // this CTA's 4 tile rows
            bool ok = true;
            for (uint32_t kb = 0; kb < num_kb; ++kb) {
                bool w = true;
                if (lane == 0) w = mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns);
                if (__shfl_sync(0xffffffffu, w ? 1 : 0, 0) == 0) {
                    ok = false;
                    break;
                }
                const uint32_t a_s = smem_u32(smem + stage * kWStageBytes);
                const uint32_t b_s = a_s + kWABytes;
                const uint32_t kt0 = kb * kBKT;
#pragma unroll
                for (int i = 0; i < kWFaces / kProdWarps; ++i) {
                    const uint32_t f = warp + kProdWarps * i;
                    const char* src;
                    uint32_t dst;
                    bool valid;
                    if (i < 32 / kProdWarps) {  // A face: (mt_l, ktl, fr, fc)
                        const uint32_t mt_l = f >> 3, ktl = (f >> 2) & 1u, fr = (f >> 1) & 1u,
                                       fc = f & 1u;
                        const uint32_t mt = mt0 + mt_l, kt = kt0 + ktl;
                        valid = mt < p.Mt && kt < p.Kt;
                        src = a_g + (((uint64_t)mt * p.Kt + kt) * 1024u + (fr * 2u + fc) * 256u) * 2u;
                        dst = a_s + (ktl * 2u + fc) * 4096u + (mt_l * 32u + fr * 16u) * 32u;
                    } else {  // B face: (half, ktl, nt_l, fr, fc)
                        const uint32_t g = f - 32u;
                        const uint32_t h = g >> 5, ktl = (g >> 4) & 1u, nt_l = (g >> 2) & 3u,
                                       fr = (g >> 1) & 1u, fc = g & 1u;
                        const uint32_t kt = kt0 + ktl, nt = nb * 16u + h * 8u + rank * 4u + nt_l;
                        valid = kt < p.Kt && nt < p.Nt;
                        src = b_g + (((uint64_t)kt * p.Nt + nt) * 1024u + (fr * 2u + fc) * 256u) * 2u;
                        dst = b_s + h * 16384u + fr * 8192u + ktl * 4096u + (nt_l * 2u + fc) * 512u;
                    }
                    cp_async16(dst + dst_lane, valid ? src + src_lane : a_g, valid ? 16u : 0u);
                }
                cp_async_arrive(&full[stage]);
                if (++stage == kWStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) break;
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == kMmaWarp) {
        if (lane == 0 && !leader) {
            // ---------------------------------- relay (odd CTA): full -> leader
            const uint32_t remote_full0 = map_to_rank(&full[0], 0);
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (uint32_t tile = pair_id; ok && tile < num_tiles; tile += num_pairs) {
                for (uint32_t kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive_remote_relaxed(remote_full0 + stage * 8u);
                    if (++stage == kWStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        } else if (lane == 0) {
            // ------------------------------------- MMA issuer (even CTA)
            constexpr uint32_t idesc = make_idesc(256, 256);
            constexpr uint64_t a_base = smem_desc_base(16, 256);   // K-major SW32
            constexpr uint64_t b_base = smem_desc_base(512, 256);  // MN-major SW32
            uint32_t stage = 0, phase = 0, t_phase = 0;
            bool ok = true;
            for (uint32_t tile = pair_id; ok && tile < num_tiles; tile += num_pairs) {
                if (!mbar_wait_cluster(tempty, t_phase ^ 1u, abort_flag, p.err, p.wait_ns)) break;
                tc_fence_after();
                for (uint32_t kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_cluster(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * kWStageBytes);
                    const uint32_t b_addr = a_addr + kWABytes;
#pragma unroll
                    for (uint32_t s = 0; s < 4; ++s) {
                        const uint64_t ad = a_base | (uint64_t)(((a_addr + s * 4096u) >> 4) & 0x3fffu);
                        const uint32_t b_off = (s & 1u) * 8192u + (s >> 1) * 4096u;
#pragma unroll
                        for (uint32_t h = 0; h < 2; ++h) {
                            const uint64_t bd =
                                b_base | (uint64_t)(((b_addr + h * 16384u + b_off) >> 4) & 0x3fffu);
                            tc_mma_pair(tmem_base + h * 256u, ad, bd, idesc, (kb | s) != 0u);
                        }
                    }
                    tc_commit_pair_mc(&empty[stage], 0x3);
                    if (++stage == kWStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit_pair_mc(tfull, 0x3);
                t_phase ^= 1u;
            }
            tc_commit_pair(drain);
            mbar_drain(drain, 0, 100000000ull);
        }
    } else if (warp < 5u + kWEpiWarps) {
        // ---------------------------------------------------- epilogue
        // Warp e (0..7): TMEM lane quadrant warp % 4, column half e / 4.
        const uint32_t e = warp - 5u, q = warp & 3u, h = e >> 2;
        const uint32_t remote_tempty = map_to_rank(tempty, 0);
        uint32_t t_phase = 0;
        for (uint32_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
            uint32_t mp, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mp, nb, kWBandN);
            bool ok = true;
            if (lane == 0) ok = mbar_wait_cluster(tfull, t_phase, abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            // This GPU's C only; the pusher warps copy it to the peers.
            store_tile_row<false>(p, tmem_base + ((q * 32u) << 16) + h * 256u, (mp * 2u + rank) * 4u + q,
                                  nb * 16u + h * 8u, lane);
            tc_fence_before();
            if (pushers) {
                // Publish this warp's part of the tile (GPU-scope: the
                // pushers read it through L2) BEFORE releasing the
                // accumulator: the next tile's parts can then only be
                // counted after every part of this tile, so the count
                // 8 (k + 1) the pushers wait for means all of tile k.
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(const_cast<uint32_t*>(epi_done), 1u);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(remote_tempty);
            t_phase ^= 1u;
        }
    } else {
        // ---------------------------------------------------- pushers
        // Pusher j copies tile row mt0 + j of each finished tile (its 16
        // tile columns: up to 32 KiB contiguous in the tile layout) from C
        // to every peer copy, 4 x 32 bytes in flight per lane.
        const uint32_t j = warp - (5u + kWEpiWarps);
        uint32_t k = 0;
        for (uint32_t tile = pair_id; pushers && tile < num_tiles; tile += num_pairs, ++k) {
            bool ok = true;
            if (lane == 0) ok = wait_count(epi_done, kWEpiWarps * (k + 1u), abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            __syncwarp();
            __threadfence();
            uint32_t mp, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mp, nb, kWBandN);
            const uint32_t mt = (mp * 2u + rank) * 4u + j, nt0 = nb * 16u;
            if (mt >= p.Mt || nt0 >= p.Nt) continue;
            const uint32_t ntn = min(16u, p.Nt - nt0);
            const uint64_t e0 = ((uint64_t)mt * p.Nt + nt0) * 1024u;  // elements
            const uint32_t n32 = ntn * 64u;                            // 32-byte pieces
#pragma unroll 1
            for (uint32_t i = lane; i < n32; i += 128u) {
                uint32_t w[4][8];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (i + 32u * u < n32) ld_global_cg_v8(p.c + e0 + (uint64_t)(i + 32u * u) * 16u, w[u]);
                if (p.mc_c) {
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (i + 32u * u < n32) {
                            uint16_t* dst = p.mc_c + e0 + (uint64_t)(i + 32u * u) * 16u;
                            st_multimem_v4(dst, w[u][0], w[u][1], w[u][2], w[u][3]);
                            st_multimem_v4(dst + 8, w[u][4], w[u][5], w[u][6], w[u][7]);
                        }
                } else {
#pragma unroll
                    for (uint32_t d = 0; d < kMaxPeers; ++d) {
                        if (d < p.npeers) {
#pragma unroll
                            for (int u = 0; u < 4; ++u)
                                if (i + 32u * u < n32)
                                    st_global_v8(p.peer_c[d] + e0 + (uint64_t)(i + 32u * u) * 16u, w[u]);
                        }
                    }
                }
            }
        }
        if (pushers) __threadfence_system();
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// Launch with programmatic stream serialization (see the kernels' set-up):
// FOIL_GEMM_PDL=0 launches plainly (for comparisons).
static cudaError_t launch_gemm(void (*kernel)(const Params), uint32_t grid, int threads, int smem,
                               cudaStream_t stream, const Params& p) {
    static const bool pdl = pdl_enabled("FOIL_GEMM_PDL");
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

int launch(const uint16_t* a, const uint16_t* b, uint16_t* c, uint32_t Mt, uint32_t Kt,
           uint32_t Nt, const uint16_t* bias, int relu, uint32_t* err, cudaStream_t stream,
           int max_ctas, uint16_t* const* peer_c, uint32_t npeers, uint16_t* mc_c) {
    cudaError_t attr_err = foil_smem_optin((const void*)gemm_tiles_kernel, kSmemBytes);
    if (attr_err == cudaSuccess) attr_err = foil_smem_optin((const void*)gemm_pair_kernel, kPSmemBytes);
    if (attr_err != cudaSuccess) {
        foil_set_error(FOIL_ERR_CUDA, "foil_matmul_tiles: cudaFuncSetAttribute failed");
        return FOIL_ERR_CUDA;
    }
    Params p;
    p.a = a;
    p.b = b;
    p.c = c;
    p.bias = bias;
    p.Mt = Mt;
    p.Kt = Kt;
    p.Nt = Nt;
    p.n_blocks = (Nt + 7) / 8;
    p.relu = relu;
    p.err = err;
    p.wait_ns = foil_wait_limit_ns();
    p.npeers = peer_c ? npeers : 0u;
    for (uint32_t d = 0; d < kMaxPeers; ++d) p.peer_c[d] = d < p.npeers ? peer_c[d] : nullptr;
    p.mc_c = mc_c;
    if (mc_c) p.npeers = 0;  // the multicast address reaches every copy
    bool al32 = ((uintptr_t)c & 31u) == 0 && ((uintptr_t)mc_c & 31u) == 0;
    for (uint32_t d = 0; d < p.npeers; ++d) al32 = al32 && ((uintptr_t)p.peer_c[d] & 31u) == 0;
    p.wide_stores = al32 ? 1u : 0u;
    if (Mt <= 4 || max_ctas < 2) {
        // One 128-row block: the single-SM kernel avoids an idle partner CTA.
        p.m_blocks = (Mt + 3) / 4;
        const uint32_t tiles = p.m_blocks * p.n_blocks;
        const uint32_t grid = tiles < (uint32_t)max_ctas ? tiles : (uint32_t)max_ctas;
        const cudaError_t le = launch_gemm(gemm_tiles_kernel, grid, kThreads, kSmemBytes, stream, p);
        return check_launch("foil_matmul_tiles", le);
    }
    p.m_blocks = (Mt + 7) / 8;  // 256-row blocks, one per CTA pair
    // More than one 256-column block: the 512-column pair kernel (a quarter
    // fewer L2 -> SM bytes per FLOP; 8192^3: 1.17 -> 1.46 PFLOP/s over 50
    // launches, 1.07 -> 1.32 under the power cap over 400).  With peer
    // copies of C it runs with four pusher warps more, which move finished
    // tiles to the peers while later tiles compute (their 256-bit copies need
    // 32-byte aligned buffers; otherwise the 256-column kernel's epilogue
    // stores to the peers itself).
    if (Nt > 8 && ((p.npeers == 0 && p.mc_c == nullptr) || p.wide_stores)) {
        if (foil_smem_optin((const void*)gemm_pair_wide_kernel, kWSmemBytes) != cudaSuccess) {
            foil_set_error(FOIL_ERR_CUDA, "foil_matmul_tiles: cudaFuncSetAttribute failed");
            return FOIL_ERR_CUDA;
        }
        p.n_blocks = (Nt + 15) / 16;  // 512-column blocks
        const uint32_t wtiles = p.m_blocks * p.n_blocks;
        const uint32_t wmax = (uint32_t)max_ctas / 2;
        const uint32_t wpairs = wtiles < wmax ? wtiles : wmax;
        const int threads = (p.npeers || p.mc_c) ? kWThreadsPush : kWThreads;
        const cudaError_t le = launch_gemm(gemm_pair_wide_kernel, wpairs * 2, threads, kWSmemBytes, stream, p);
        return check_launch("foil_matmul_tiles (2-SM, 512 columns)", le);
    }
    const uint32_t tiles = p.m_blocks * p.n_blocks;
    const uint32_t max_pairs = (uint32_t)max_ctas / 2;
    const uint32_t pairs = tiles < max_pairs ? tiles : max_pairs;
    const cudaError_t le = launch_gemm(gemm_pair_kernel, pairs * 2, kThreads, kPSmemBytes, stream, p);
    return check_launch("foil_matmul_tiles (2-SM)", le);
}

}  // namespace gemm
}  // namespace foil
