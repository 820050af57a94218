// Implicit-GEMM NHWC convolution on tcgen05 tensor cores, fused bias + relu.
//
//   y[n, ho, wo, co] = relu( bf16( bf16( sum_{kh,kw,ci} x[n, ho*s+kh-p, wo*s+kw-p, ci]
//                                                       * w[co, kh, kw, ci] ) + bias[co] ) )
//
// The reference runs convolutions as a host im2col followed by its tiled
// matmul (tests/test_conv_3x3.cpp:108-127 and :214-222; stride only changes
// the im2col, tests/test_conv_3x3_s2.cpp:11-15).  Here the im2col is implicit:
// the GEMM rows are output pixels (M = N*Ho*Wo), the columns output channels
// (N = Cout), K = (kh, kw, ci), and the producer warps gather A straight from
// the NHWC input.  Padding taps are zero-filled by the copy itself.
//
// Operands in shared memory (canonical UMMA layouts, SWIZZLE_32B, K-major):
//  * A: a k-block is one tap (kh, kw) x kc channels (kc = 64, 32 or 16).  Each
//    output row's kc channels are one contiguous run of kc*2 bytes of one
//    input pixel, so a warp copying four rows issues full 128-byte requests.
//    K-step j (16 channels) holds 128 rows x 32 B, 8-row groups 256 B apart.
//  * B: the weights, row co = w[co, kh, kw, cb*kc .. +kc] (also contiguous);
//    K-step j holds BN rows x 32 B.
//  Instruction: kind::f16, M = 128, N = BN, K = 16, A and B both K-major.
//
// Two producers fill the same pipeline:
//  * tensor-copy producer (Cin a multiple of 64): one thread issues, per
//    k-block, an im2col tensor copy of A (128 output pixels x 64 channels of
//    tap (kh, kw): the copy engine walks the output pixels of the tile through
//    the bounding box [-pad, dim - 1 + pad - (k - 1)] with the conv stride as
//    traversal stride, reads each at (w + kw, h + kh) and zero-fills padding)
//    and a tiled copy of B (BN rows x 64 channels), both SWIZZLE_128B.  A and
//    B are K-major with 128-byte rows; K-step j starts 32 j bytes into the
//    1024-byte swizzle atom.
//  * gather producer (other Cin): 4 warps of cp.async as described above,
//    SW32 applied in the destination address.
// Organisation otherwise as the tiled GEMM (gemm_tc.cu): 1 MMA warp that owns TMEM
// (2 x BN fp32 accumulator columns, double-buffered).  Convolutions have short
// K loops (9 k-blocks for 3x3x64, 2 for 1x1x128), so the epilogue matters:
// 8 epilogue warps (two per TMEM lane quadrant, each half the columns) read 32
// columns per TMEM load, release the accumulator as soon as their last load
// has landed, and stage their rows for 2-D tensor stores (see epilogue_rows).
//
// Throughput limit measured on B200 that shaped this file: the tensor-copy
// engine of an SM completes about one tiled copy per ~200 ns and one im2col
// copy per ~295 ns, nearly independent of the box size up to 128-256 rows
// and of how many copies are in flight or how many SMs issue them.  So copy
// INSTRUCTIONS are the budget: a 128-row im2col of 16 KiB moves ~56 GB/s per
// SM, a 256-row one twice that.  Hence the weight-stationary pair kernel (no
// weight copies per k-block, 256-row im2col copies).  A per-role trace of
// that kernel (3x3 stride 2, batch 32) showed each 32 KiB stride-2 im2col
// copy taking ~0.9 us from issue to completion, one completing every
// ~0.5 us, so the number of stages in flight sets its pace; its epilogue
// therefore stores from registers and gives the staging buffer to a fourth
// stage.  Every wait is bounded (see gemm_ptx.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "gemm_ptx.cuh"
#include "conv_tc.cuh"
#include "../../../include/foil_c.h"

extern "C" void foil_set_error(int status, const char* msg);

namespace foil {
namespace conv {

using namespace foil::gemm;

constexpr int kProdWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each half of the columns
constexpr int kThreads = (5 + kEpiWarps) * 32;
constexpr int kBarrierBytes = 512;  // mbarriers and flags after the staging area

struct Params {
    const uint16_t* x;
    const uint16_t* w;
    const uint16_t* bias;
    uint16_t* y;
    uint32_t N, H, W, Cin, Cout, KH, KW, stride, pad, Ho, Wo;
    uint32_t M;            // N * Ho * Wo
    uint32_t kc;           // channels per k-block (16, 32 or 64)
    uint32_t cblocks;      // Cin / kc
    uint32_t num_kb;       // KH * KW * cblocks
    uint32_t m_blocks, n_blocks;
    int relu;
    uint32_t box_cols;     // columns of the output tensor map's box (must equal Epi<BN>::kCols)
    uint32_t direct;       // pair kernel: epilogue stores rows from registers (no staging)
    uint32_t wide_y;       // y 32-byte aligned: 256-bit stores in the direct epilogue
    uint32_t* err;
    uint64_t wait_ns;      // wall-time limit of each bounded wait
};

template <int BN, bool kDirect = false>
struct Cfg {
    static constexpr int kABytes = 128 * 128;               // 128 rows x 64 ch x 2 B (max kc)
    static constexpr int kBBytes = BN * 128;                // BN rows x 64 ch x 2 B
    static constexpr int kStageBytes = kABytes + kBBytes;
    // Epilogue staging: 8 warps x 32 rows x BN/2 columns (see Epi); none when
    // the epilogue stores from registers.
    static constexpr int kStagingBytes = kDirect ? 0 : 256 * BN;
    static constexpr int kLimit = 220 * 1024;
    static constexpr int kFit = (kLimit - kStagingBytes - 1024 - kBarrierBytes) / kStageBytes;
    static constexpr int kStages = kFit > 8 ? 8 : kFit;
    static constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 + kBarrierBytes;
    static constexpr int kTmemCols = 2 * BN;                // power of two for BN in {64,128,256}
};

// Epilogue modes: 0 = bf16(acc); 1 = bf16(bf16(acc) + bias);
// 2 = relu(bf16(bf16(acc) + bias)) (bias 0 when absent).
//
// Two accumulators (columns c, c+1 of one row) -> packed bf16x2, the
// composition of the reference goldens (matmul, bias_add, relu).  bf16(acc) is
// one round-to-nearest-even conversion; the bias add is a packed bf16 fma
// r * 1 + bias, rounded once.  That equals the golden's fp32 add followed by
// bf16 rounding: the sum of two bf16 values is either exact in fp32 or
// differs from a bf16 value by far less than half a bf16 ulp, so the fp32
// rounding never creates a bf16 tie.  The .relu form clamps negative results
// to +0 (the golden's float comparison treats -0 and +0 alike).
__device__ __forceinline__ uint32_t epi_pair(uint32_t a0, uint32_t a1, uint32_t bias2, int mode) {
    const uint32_t r = cvt_bf16x2(__uint_as_float(a0), __uint_as_float(a1));
    if (mode == 0) return r;
    uint32_t d;
    if (mode == 1)
        asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(r), "r"(0x3f803f80u), "r"(bias2));
    else
        asm("fma.rn.relu.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(r), "r"(0x3f803f80u), "r"(bias2));
    return d;
}

// 0 = bf16(acc), 1 = + bias, 2 = + bias (if any), relu.
__device__ __forceinline__ int epi_mode(const Params& p) {
    return p.relu ? 2 : (p.bias != nullptr ? 1 : 0);
}

// Bias words (bf16 pairs) of output channels co .. co + 31, or zeros; each
// group of 16 channels is read only if it lies below Cout (a multiple of 16).
__device__ __forceinline__ void load_bias32(const Params& p, uint32_t co, bool want, uint32_t (&bw)[16]) {
    const uint4* bp = reinterpret_cast<const uint4*>(p.bias + co);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 bv = make_uint4(0u, 0u, 0u, 0u);
        if (want && co + 16u * (uint32_t)(i / 2) < p.Cout) bv = __ldg(bp + i);
        bw[4 * i] = bv.x; bw[4 * i + 1] = bv.y; bw[4 * i + 2] = bv.z; bw[4 * i + 3] = bv.w;
    }
}

// Epilogue geometry.  Epilogue warp e covers TMEM lane quadrant e % 4 (32
// rows) and column half e / 4 (BN/2 columns); it stages its 32 x BN/2 share
// in boxes of 32 rows x kCols columns (128-byte rows with SWIZZLE_128B for
// BN >= 128, else 64-byte rows with SWIZZLE_64B) and stores each box with one
// 2-D tensor store.  (Boxes of 128 rows shared by the four warps of a column
// half, synchronised through mbarriers, cut the store instructions by 4 but
// measured 6-37% slower: the warps then wait on each other and on the
// previous store of the shared box.)
template <int BN>
struct Epi {
    static constexpr int kChunks = BN / 64;              // 32-column chunks per warp
    static constexpr int kCols = BN >= 128 ? 64 : 32;    // columns per box
    static constexpr int kCPB = kCols / 32;              // chunks per box
    static constexpr int kBoxes = kChunks / kCPB;        // boxes per warp
    static constexpr uint32_t kRowBytes = kCols * 2;
    static constexpr uint32_t kBoxBytes = 32 * kRowBytes;
    static constexpr uint32_t kWarpBytes = kBoxes * kBoxBytes;  // 32 rows x BN/2 columns
};

// One epilogue warp's share of an accumulator tile: 32 rows (TMEM lane
// quadrant; t_row addresses lane 0 of the quadrant at the warp's first
// column) x BN/2 columns from output channel co0, output rows m0 .. m0 + 31.
// The columns are read 32 at a time (lane = row); the TMEM load and the bias
// load of chunk ci + 1 are in flight while chunk ci is converted.  Chunk ci
// goes to box ci / kCPB at its swizzled position (16-byte piece k of row r at
// k ^ (r & 7), or k ^ ((r >> 1) & 3) for 64-byte rows: conflict-free for
// row-per-lane writes), and each full box is stored by lane 0 (the copy
// engine clips rows >= M and columns >= Cout), one bulk group per box.  Box
// b is rewritten one tile later, after waiting until at most kBoxes - 1 newer
// groups still read shared memory, i.e. box b's previous store has.
// `release` runs after the last TMEM load.  Rows from m_end on are not
// stored (the box of a warp whose first row m0 >= m_end is skipped).
template <int BN, class Release>
__device__ __forceinline__ void epilogue_rows(const Params& p, const CUtensorMap* tmap_y, uint32_t t_row,
                                              uint32_t m0, uint32_t co0, uint32_t stg, int mode, uint32_t lane,
                                              uint32_t m_end, Release release) {
    using E = Epi<BN>;
    const uint32_t row_off = lane * E::kRowBytes;
    const uint32_t sw = E::kCols == 64 ? (lane & 7u) : ((lane >> 1) & 3u);
    const bool want_bias = mode != 0 && p.bias != nullptr;
    uint32_t v[2][32], bw[2][16];
    load_bias32(p, co0, want_bias, bw[0]);
    tmem_ld32(t_row, v[0]);
#pragma unroll
    for (int ci = 0; ci < E::kChunks; ++ci) {
        tmem_ld_wait();  // chunk ci has landed (no other load is in flight)
        if (ci + 1 < E::kChunks) {
            tmem_ld32(t_row + 32u * (ci + 1), v[(ci + 1) & 1]);
            load_bias32(p, co0 + 32u * (ci + 1), want_bias, bw[(ci + 1) & 1]);
        }
        if (ci + 1 == E::kChunks) release();
        const uint32_t* c = v[ci & 1];
        const uint32_t* b = bw[ci & 1];
        uint32_t o[16];
        if (mode == 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = epi_pair(c[2 * i], c[2 * i + 1], 0u, 0);
        } else if (mode == 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = epi_pair(c[2 * i], c[2 * i + 1], b[i], 1);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = epi_pair(c[2 * i], c[2 * i + 1], b[i], 2);
        }
        const int bx = ci / E::kCPB, part = ci % E::kCPB;
        const uint32_t box = stg + bx * E::kBoxBytes;
        if (part == 0) {
            if (lane == 0) bulk_wait_read_n<E::kBoxes - 1>();
            __syncwarp();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t k = (uint32_t)(part * 4 + i);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(box + row_off + ((k ^ sw) << 4)),
                         "r"(o[4 * i]), "r"(o[4 * i + 1]), "r"(o[4 * i + 2]), "r"(o[4 * i + 3])
                         : "memory");
        }
        if (part == E::kCPB - 1) {
            // Generic-proxy writes above, async-proxy (tensor store) reads below.
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                const uint32_t xc = co0 + (uint32_t)(bx * E::kCols);
                if (m0 < m_end && xc < p.Cout) tma_store_2d(tmap_y, (int32_t)xc, (int32_t)m0, box);
                bulk_commit();
            }
        }
    }
}

// The same share of an accumulator tile stored straight from registers: lane
// = output row, each 32-column chunk is 64 contiguous bytes of that row,
// written as two 32-byte stores (whole L2 sectors) or, for a y that is only
// 16-byte aligned, four 16-byte stores.  Needs no staging buffer, so the
// pair kernel can keep one more operand stage in flight.
template <int BN, class Release>
__device__ __forceinline__ void epilogue_rows_direct(const Params& p, uint32_t t_row, uint32_t m0, uint32_t co0,
                                                     int mode, uint32_t lane, uint32_t m_end, Release release) {
    constexpr int kChunks = BN / 64;
    const uint32_t m = m0 + lane;
    const bool row_ok = m < m_end;
    uint16_t* yrow = p.y + (uint64_t)(row_ok ? m : 0u) * p.Cout;
    const bool want_bias = mode != 0 && p.bias != nullptr;
    uint32_t v[2][32], bw[2][16];
    load_bias32(p, co0, want_bias, bw[0]);
    tmem_ld32(t_row, v[0]);
#pragma unroll
    for (int ci = 0; ci < kChunks; ++ci) {
        tmem_ld_wait();
        if (ci + 1 < kChunks) {
            tmem_ld32(t_row + 32u * (ci + 1), v[(ci + 1) & 1]);
            load_bias32(p, co0 + 32u * (ci + 1), want_bias, bw[(ci + 1) & 1]);
        }
        if (ci + 1 == kChunks) release();
        const uint32_t* c = v[ci & 1];
        const uint32_t* b = bw[ci & 1];
        uint32_t o[16];
        if (mode == 0) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = epi_pair(c[2 * i], c[2 * i + 1], 0u, 0);
        } else if (mode == 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = epi_pair(c[2 * i], c[2 * i + 1], b[i], 1);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = epi_pair(c[2 * i], c[2 * i + 1], b[i], 2);
        }
        const uint32_t co = co0 + 32u * (uint32_t)ci;
        if (row_ok) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (co + 16u * h < p.Cout) {
                    uint16_t* dst = yrow + co + 16u * h;
                    if (p.wide_y) {
                        st_global_v8(dst, o + 8 * h);
                    } else {
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
                        d4[0] = make_uint4(o[8 * h], o[8 * h + 1], o[8 * h + 2], o[8 * h + 3]);
                        d4[1] = make_uint4(o[8 * h + 4], o[8 * h + 5], o[8 * h + 6], o[8 * h + 7]);
                    }
                }
            }
        }
    }
}

// Bounded wait for the copies of the last `stages` of `issued` loads (load
// j completes phase (j / stages) & 1 of full[j % stages]); phases that have
// completed return at once.
__device__ __forceinline__ void drain_loads(uint64_t* full, uint32_t issued, uint32_t stages) {
    const uint32_t j0 = issued > stages ? issued - stages : 0u;
#pragma unroll 1
    for (uint32_t j = j0; j < issued; ++j) mbar_drain(&full[j % stages], (j / stages) & 1u, 100000000ull);
}

template <int BN, bool kTma, bool kDirect>
__global__ void __launch_bounds__(kThreads, 1)
    conv_kernel(const Params p, const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_y) {
    using C = Cfg<BN, kDirect>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* staging = smem + C::kStages * C::kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::kStagingBytes);
    uint64_t* empty = full + C::kStages;
    uint64_t* tfull = empty + C::kStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    // The output map's box must be this instantiation's staging box; every
    // thread takes the same early exit otherwise (nothing started yet).
    if (p.box_cols != (uint32_t)Epi<BN>::kCols) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, kErrConfig);
        return;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], kTma ? 1 : kProdWarps * 32);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(C::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Launched with programmatic stream serialization, the set-up above may
    // overlap the previous kernel's tail; global memory is touched only after
    // that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t num_tiles = p.m_blocks * p.n_blocks;
    const uint32_t ksteps = p.kc / 16;  // K-steps (16 channels) per k-block

    if (kTma && warp < kProdWarps) {
        // ------------------------------------- tensor-copy producer (1 thread)
        if (warp == 0 && lane == 0) {
            tma_prefetch_map(&tmap_x);
            tma_prefetch_map(&tmap_w);
            const uint32_t hw = p.Ho * p.Wo;
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                const uint32_t mb = tile / p.n_blocks, nb = tile - mb * p.n_blocks;
                // Base pixel (tap (0, 0)) of the tile's first output pixel.
                const uint32_t m0 = mb * 128u, n = m0 / hw, rem = m0 - n * hw;
                const uint32_t ho = rem / p.Wo, wo = rem - ho * p.Wo;
                const int32_t w0 = (int32_t)(wo * p.stride) - (int32_t)p.pad;
                const int32_t h0 = (int32_t)(ho * p.stride) - (int32_t)p.pad;
                uint32_t kh = 0, kw = 0, cb = 0;
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    const uint32_t a_s = smem_u32(smem + stage * C::kStageBytes);
                    mbar_expect_tx(&full[stage], (uint32_t)C::kStageBytes);
                    tma_load_im2col_4d(a_s, &tmap_x, (int32_t)(cb * 64u), w0, h0, (int32_t)n,
                                       (uint16_t)kw, (uint16_t)kh, &full[stage]);
                    tma_load_2d(a_s + C::kABytes, &tmap_w,
                                (int32_t)((kh * p.KW + kw) * p.Cin + cb * 64u), (int32_t)(nb * BN),
                                &full[stage]);
                    ++issued;
                    if (++stage == C::kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (++cb == p.cblocks) {
                        cb = 0;
                        if (++kw == p.KW) {
                            kw = 0;
                            ++kh;
                        }
                    }
                }
            }
            // After an abort, copies of the last stages may still be landing
            // in shared memory: wait (bounded) for each before the CTA ends
            // (at once when they have all been consumed).
            drain_loads(full, issued, (uint32_t)C::kStages);
        }
    } else if (warp < kProdWarps) {
        // ---------------------------------------------------- producers
        // A: lane covers chunk q = lane & 7 (8 channels) of row (lane >> 3) of
        // each 4-row group; chunk q of a kc-channel run goes to K-step q/2,
        // half q%2.  Rows with q >= kc/8 are idle for kc < 64.
        const uint32_t q = lane & 7u, rsub = lane >> 3;
        const bool chunk_used = q < p.kc / 8u;
        const uint32_t j = q >> 1, h = q & 1u;
        const char* xg = reinterpret_cast<const char*>(p.x);
        const char* wg = reinterpret_cast<const char*>(p.w);
        uint32_t stage = 0, phase = 0;
        for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const uint32_t mb = tile / p.n_blocks, nb = tile - mb * p.n_blocks;
            // Per tile: this lane's 8 A rows r = (warp + 4 i) * 4 + rsub, as the
            // input position of tap (0, 0) and the matching byte pointer; tap
            // (kh, kw), channel block cb then adds one offset common to all rows.
            int32_t ih0[8], iw0[8];
            const char* abase[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t r = (warp + kProdWarps * i) * 4u + rsub;
                const uint32_t m = mb * 128u + r;
                const uint32_t mm = m < p.M ? m : 0u;
                const uint32_t n = mm / (p.Ho * p.Wo), rem = mm - n * p.Ho * p.Wo;
                const uint32_t ho = rem / p.Wo, wo = rem - ho * p.Wo;
                ih0[i] = m < p.M ? (int32_t)(ho * p.stride) - (int32_t)p.pad : INT32_MIN / 2;
                iw0[i] = (int32_t)(wo * p.stride) - (int32_t)p.pad;
                const int64_t pix = (int64_t)n * p.H * p.W + (int64_t)ih0[i] * p.W + iw0[i];
                abase[i] = xg + (pix * p.Cin + q * 8u) * 2;
            }
            const char* bbase[BN / 16];
            bool bvalid[BN / 16];
#pragma unroll
            for (int i = 0; i < BN / 16; ++i) {
                const uint32_t co = nb * BN + (warp + kProdWarps * i) * 4u + rsub;
                bvalid[i] = co < p.Cout;
                bbase[i] = wg + ((uint64_t)(bvalid[i] ? co : 0u) * p.KH * p.KW * p.Cin + q * 8u) * 2u;
            }
            bool ok = true;
            uint32_t kh = 0, kw = 0, cb = 0;
            for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                bool wt = true;
                if (lane == 0) wt = mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns);
                if (__shfl_sync(0xffffffffu, wt ? 1 : 0, 0) == 0) {
                    ok = false;
                    break;
                }
                const uint32_t a_s = smem_u32(smem + stage * C::kStageBytes);
                const uint32_t b_s = a_s + C::kABytes;
                if (chunk_used) {
                    const int64_t a_off = ((int64_t)(kh * p.W + kw) * p.Cin + cb * p.kc) * 2;
                    const uint64_t b_off = ((uint64_t)(kh * p.KW + kw) * p.Cin + cb * p.kc) * 2u;
                    // Row r = (warp + 4 i) * 4 + rsub: bit 2 of r is bit 0 of warp,
                    // so the 32-byte swizzle of this lane's chunk is fixed.
                    const uint32_t row_off = (warp * 4u + rsub) * 32u + ((h ^ (warp & 1u)) << 4);
                    const uint32_t a_dst = a_s + j * 4096u + row_off;
                    const uint32_t b_dst = b_s + j * (uint32_t)(BN * 32) + row_off;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const bool v = (uint32_t)(ih0[i] + (int32_t)kh) < p.H &&
                                       (uint32_t)(iw0[i] + (int32_t)kw) < p.W;
                        cp_async16(a_dst + i * 512u, v ? abase[i] + a_off : xg, v ? 16u : 0u);
                    }
#pragma unroll
                    for (int i = 0; i < BN / 16; ++i)
                        cp_async16(b_dst + i * 512u, bvalid[i] ? bbase[i] + b_off : wg, bvalid[i] ? 16u : 0u);
                }
                cp_async_arrive(&full[stage]);
                if (++stage == C::kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
                // next k-block: channel block, then kw, then kh
                if (++cb == p.cblocks) {
                    cb = 0;
                    if (++kw == p.KW) {
                        kw = 0;
                        ++kh;
                    }
                }
            }
            if (!ok) break;
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            // kind::f16, f32 accumulate, bf16 A and B, both K-major.
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                   ((128u >> 4) << 24);
            constexpr uint64_t kmaj = kTma ? smem_desc_sw128_kmajor() : smem_desc_base(16, 256);
            // Byte step between K-steps: 32 B inside the 128-byte swizzle rows
            // (tensor copies) or one whole SW32 block of rows (gather).
            constexpr uint32_t a_step = kTma ? 32u : 4096u;
            constexpr uint32_t b_step = kTma ? 32u : (uint32_t)(BN * 32);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * C::kStageBytes);
                    const uint32_t b_addr = a_addr + C::kABytes;
                    for (uint32_t s = 0; s < ksteps; ++s) {
                        const uint64_t ad = kmaj | (uint64_t)(((a_addr + s * a_step) >> 4) & 0x3fffu);
                        const uint64_t bd = kmaj | (uint64_t)(((b_addr + s * b_step) >> 4) & 0x3fffu);
                        tc_mma(d_tmem, ad, bd, idesc, (kb | s) != 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == C::kStages) {
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
            tc_commit(drain);
            mbar_drain(drain, 0, 100000000ull);
        }
    } else {
        // ---------------------------------------------------- epilogue
        // Warp e (0..7) drains TMEM lane quadrant warp % 4 (rows qd*32 + lane),
        // columns [half * BN/2, (half + 1) * BN/2).
        const uint32_t e = warp - 5u, qd = warp & 3u, half = e >> 2;
        const uint32_t col0 = half * (uint32_t)(BN / 2);
        const uint32_t stg = smem_u32(staging) + e * Epi<BN>::kWarpBytes;
        const int mode = epi_mode(p);
        if (lane == 0) tma_prefetch_map(&tmap_y);
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const uint32_t mb = tile / p.n_blocks, nb = tile - mb * p.n_blocks;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            uint64_t* te = &tempty[acc];
            auto release = [&] {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(te);
            };
            const uint32_t t_row = tmem_base + ((qd * 32u) << 16) + acc * BN + col0;
            if constexpr (kDirect)
                epilogue_rows_direct<BN>(p, t_row, mb * 128u + qd * 32u, nb * BN + col0, mode, lane, p.M, release);
            else
                epilogue_rows<BN>(p, &tmap_y, t_row, mb * 128u + qd * 32u, nb * BN + col0, stg, mode, lane, p.M,
                                  release);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(C::kTmemCols)
                     : "memory");
    }
}

// ------------------------------------------------------------------------
// Weight-stationary single-CTA variant (tensor copies, one column block):
// the CTA loads all of its BN output channels' weights (every k-block) once,
// with one 3-D tensor copy, and per k-block only the 128-row im2col copy of
// A (16 KiB) into a ring of `stages` A buffers.  For convolutions with few
// k-blocks (the 1x1: 2), where the pair kernel's start-up is not amortised,
// this removes the weight copies of the streaming kernel (2/3 of its copy
// bytes for 128 -> 256 channels) and the freed shared memory holds twice
// the A stages.  Epilogue as in the streaming kernel (staged tensor stores).
constexpr int kResMaxStages = 12;

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    conv_res_kernel(const Params p, const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_y,
                    uint32_t stages) {
    constexpr uint32_t kA = 128u * 128u;             // A bytes per k-block
    constexpr uint32_t kB = (uint32_t)BN * 128u;     // weight bytes per k-block
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* b_res = smem;
    uint8_t* a_st = b_res + p.num_kb * kB;
    uint8_t* staging = a_st + stages * kA;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + 256u * BN);
    uint64_t* empty = full + kResMaxStages;
    uint64_t* tfull = empty + kResMaxStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* bfull = tempty + 2;
    uint64_t* drain = bfull + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    if (p.box_cols != (uint32_t)Epi<BN>::kCols || stages == 0 || stages > (uint32_t)kResMaxStages) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, kErrConfig);
        return;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEpiWarps);
        }
        mbar_init(bfull, 1);
        mbar_init(drain, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(2u * BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Launched with programmatic stream serialization, the set-up above may
    // overlap the previous kernel's tail; global memory is touched only after
    // that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t num_tiles = p.m_blocks;  // one column block

    if (warp == 0) {
        if (lane == 0) {
            // ----------------------------------------- tensor-copy producer
            tma_prefetch_map(&tmap_x);
            tma_prefetch_map(&tmap_w);
            // All weights, once: [k-block][BN rows][64 ch] (encode_weight_map3).
            mbar_expect_tx(bfull, p.num_kb * kB);
            tma_load_3d(smem_u32(b_res), &tmap_w, 0, 0, 0, bfull);
            const uint32_t hw = p.Ho * p.Wo;
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                const uint32_t m0 = tile * 128u, n = m0 / hw, rem = m0 - n * hw;
                const uint32_t ho = rem / p.Wo, wo = rem - ho * p.Wo;
                const int32_t w0 = (int32_t)(wo * p.stride) - (int32_t)p.pad;
                const int32_t h0 = (int32_t)(ho * p.stride) - (int32_t)p.pad;
                uint32_t kh = 0, kw = 0, cb = 0;
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&full[stage], kA);
                    tma_load_im2col_4d(smem_u32(a_st + stage * kA), &tmap_x, (int32_t)(cb * 64u), w0, h0,
                                       (int32_t)n, (uint16_t)kw, (uint16_t)kh, &full[stage]);
                    ++issued;
                    if (++stage == stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (++cb == p.cblocks) {
                        cb = 0;
                        if (++kw == p.KW) {
                            kw = 0;
                            ++kh;
                        }
                    }
                }
            }
            // Copies of the weights and of the last stages may still be in
            // flight after an abort: wait (bounded) for each before the CTA ends.
            mbar_drain(bfull, 0, 100000000ull);
            drain_loads(full, issued, stages);
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                   ((128u >> 4) << 24);
            constexpr uint64_t kmaj = smem_desc_sw128_kmajor();
            const uint32_t a0 = smem_u32(a_st), b0 = smem_u32(b_res);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = mbar_wait(bfull, 0, abort_flag, p.err, p.wait_ns);
            for (uint32_t tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = a0 + stage * kA, b_addr = b0 + kb * kB;
#pragma unroll
                    for (uint32_t s = 0; s < 4; ++s) {
                        const uint64_t ad = kmaj | (uint64_t)(((a_addr + s * 32u) >> 4) & 0x3fffu);
                        const uint64_t bd = kmaj | (uint64_t)(((b_addr + s * 32u) >> 4) & 0x3fffu);
                        tc_mma(d_tmem, ad, bd, idesc, (kb | s) != 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == stages) {
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
            tc_commit(drain);
            mbar_drain(drain, 0, 100000000ull);
        }
    } else if (warp > kMmaWarp) {
        // ---------------------------------------------------- epilogue
        const uint32_t e = warp - 5u, qd = warp & 3u, half = e >> 2;
        const uint32_t col0 = half * (uint32_t)(BN / 2);
        const uint32_t stg = smem_u32(staging) + e * Epi<BN>::kWarpBytes;
        const int mode = epi_mode(p);
        if (lane == 0) tma_prefetch_map(&tmap_y);
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            uint64_t* te = &tempty[acc];
            epilogue_rows<BN>(p, &tmap_y, tmem_base + ((qd * 32u) << 16) + acc * BN + col0,
                              tile * 128u + qd * 32u, col0, stg, mode, lane, p.M, [&] {
                                  tc_fence_before();
                                  __syncwarp();
                                  if (lane == 0) mbar_arrive(te);
                              });
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2u * BN)
                     : "memory");
    }
}

// ------------------------------------------------------------------------
// Weight-stationary 2-SM variant (tensor copies, Cout <= 256).  A CTA pair
// (cluster of 2) computes tiles of 256 kSub rows with tcgen05.mma.cta_group::2
// (M = 256, N = BN): each CTA loads 128 kSub consecutive output pixels of A
// per k-block with ONE im2col copy (kSub = 2 for BN <= 128, 1 for BN = 256,
// bounded by TMEM: 2 buffers x kSub x BN columns <= 512), and keeps its half
// of the weights (BN/2 output channels x all of K) resident in shared memory
// for the whole kernel, loaded once.  Sub-tile s of a stage (rows 128 s ..
// 128 s + 127 of both CTAs) is one M = 256 MMA group into accumulator s.
// Per k-block and CTA the copy engine thus runs one ~295 ns instruction for
// 128 kSub rows, against one im2col plus one weight copy per 128 rows in the
// streaming kernel above.  Both CTAs' copies complete on the leader's
// barriers (cta_group::2 form); the leader issues the MMAs and multicasts
// its commits to both CTAs; each CTA drains its own TMEM rows.
constexpr int kPairMaxStages = 8;

template <int BN>
struct PairCfg {
    static constexpr int kSub = BN <= 128 ? 2 : 1;
    static constexpr uint32_t kHalfB = (BN / 2) * 128;        // this CTA's weight rows of one k-block
    static constexpr uint32_t kABytes = kSub * 128u * 128u;    // A rows of one stage
    static constexpr uint32_t kTmemCols = 2u * kSub * BN;
};

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    conv_pair_kernel(const Params p, const __grid_constant__ CUtensorMap tmap_x,
                     const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_y,
                     uint32_t stages) {
    using PC = PairCfg<BN>;
    constexpr int kSub = PC::kSub;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* b_res = smem;
    uint8_t* a_st = b_res + p.num_kb * PC::kHalfB;
    uint8_t* staging = a_st + stages * PC::kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + (p.direct ? 0u : 256u * BN));
    uint64_t* empty = full + kPairMaxStages;
    uint64_t* tfull = empty + kPairMaxStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* bfull = tempty + 2;
    uint64_t* drain = bfull + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    if (p.box_cols != (uint32_t)Epi<BN>::kCols) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, kErrConfig);
        return;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t pair_id = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * kEpiWarps * kSub);
        }
        mbar_init(bfull, 1);
        mbar_init(drain, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(PC::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    // Launched with programmatic stream serialization, the set-up above may
    // overlap the previous kernel's tail; global memory is touched only after
    // that kernel has completed.
    griddep_wait();
    griddep_launch_dependents();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t num_tiles = p.m_blocks;  // tiles of 256 kSub rows

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------ tensor-copy producer
            tma_prefetch_map(&tmap_x);
            tma_prefetch_map(&tmap_w);
            const uint32_t lead_full0 = map_to_rank(&full[0], 0);
            // Resident weights, once, in one copy: output channels [rank BN/2,
            // (rank + 1) BN/2) of all k-blocks (see encode_weight_map3).
            if (leader) mbar_expect_tx(bfull, 2u * p.num_kb * PC::kHalfB);
            tma_load_3d_pair(smem_u32(b_res), &tmap_w, 0, (int32_t)(rank * (BN / 2)), 0, map_to_rank(bfull, 0));
            const uint32_t hw = p.Ho * p.Wo;
            uint32_t stage = 0, phase = 0, issued = 0;
            bool ok = true;
            for (uint32_t tile = pair_id; ok && tile < num_tiles; tile += num_pairs) {
                // Base pixel (tap (0, 0)) of this CTA's first output pixel; past
                // the last image it lies outside the tensor and reads zeros.
                const uint32_t m0 = (tile * 2u + rank) * (128u * kSub), n = m0 / hw, rem = m0 - n * hw;
                const uint32_t ho = rem / p.Wo, wo = rem - ho * p.Wo;
                const int32_t w0 = (int32_t)(wo * p.stride) - (int32_t)p.pad;
                const int32_t h0 = (int32_t)(ho * p.stride) - (int32_t)p.pad;
                uint32_t kh = 0, kw = 0, cb = 0;
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(&full[stage], 2u * PC::kABytes);
                    tma_load_im2col_4d_pair(smem_u32(a_st + stage * PC::kABytes), &tmap_x, (int32_t)(cb * 64u), w0,
                                            h0, (int32_t)n, (uint16_t)kw, (uint16_t)kh, lead_full0 + stage * 8u);
                    ++issued;
                    if (++stage == stages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (++cb == p.cblocks) {
                        cb = 0;
                        if (++kw == p.KW) {
                            kw = 0;
                            ++kh;
                        }
                    }
                }
            }
            // After an abort: both CTAs' copies complete on the leader's
            // barriers, so the leader waits (bounded) for the weights and the
            // last stages before the pair ends (at once when they have all
            // been consumed); the final cluster barrier keeps the other CTA
            // alive meanwhile.
            if (leader) {
                mbar_drain(bfull, 0, 100000000ull);
                drain_loads(full, issued, stages);
            }
        }
    } else if (warp == kMmaWarp) {
        if (leader && lane == 0) {
            // ------------------------------------------------ MMA issuer
            // kind::f16, f32 accumulate, bf16 A and B, both K-major, M = 256.
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                   ((256u >> 4) << 24);
            constexpr uint64_t kmaj = smem_desc_sw128_kmajor();
            const uint32_t a0 = smem_u32(a_st), b0 = smem_u32(b_res);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = mbar_wait_cluster(bfull, 0, abort_flag, p.err, p.wait_ns);
            for (uint32_t tile = pair_id; ok && tile < num_tiles; tile += num_pairs) {
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * (uint32_t)(kSub * BN);
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait_cluster(&full[stage], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = a0 + stage * PC::kABytes, b_addr = b0 + kb * PC::kHalfB;
#pragma unroll
                    for (int sub = 0; sub < kSub; ++sub) {
#pragma unroll
                        for (uint32_t s = 0; s < 4; ++s) {
                            const uint64_t ad =
                                kmaj | (uint64_t)(((a_addr + sub * 16384u + s * 32u) >> 4) & 0x3fffu);
                            const uint64_t bd = kmaj | (uint64_t)(((b_addr + s * 32u) >> 4) & 0x3fffu);
                            tc_mma_pair(d_tmem + sub * BN, ad, bd, idesc, (kb | s) != 0u);
                        }
                    }
                    tc_commit_pair_mc(&empty[stage], 0x3);
                    if (++stage == stages) {
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
    } else if (warp > kMmaWarp) {
        // ---------------------------------------------------- epilogue
        // As in the streaming kernel, on this CTA's 128 kSub rows of each
        // tile (sub-tile s from accumulator s); the accumulators are released
        // on the leader's barrier.  That arrive only orders TMEM reads before
        // the next MMAs, which the tcgen05 fences do, so it is relaxed.
        const uint32_t e = warp - 5u, qd = warp & 3u, half = e >> 2;
        const uint32_t col0 = half * (uint32_t)(BN / 2);
        const uint32_t stg = smem_u32(staging) + e * Epi<BN>::kWarpBytes;
        const int mode = epi_mode(p);
        const uint32_t lead_tempty0 = map_to_rank(&tempty[0], 0);
        if (lane == 0) tma_prefetch_map(&tmap_y);
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            const uint32_t te = lead_tempty0 + acc * 8u;
#pragma unroll 1
            for (int sub = 0; sub < kSub; ++sub) {
                const uint32_t m0 = (tile * 2u + rank) * (128u * kSub) + 128u * sub + qd * 32u;
                const uint32_t t_row =
                    tmem_base + ((qd * 32u) << 16) + acc * (uint32_t)(kSub * BN) + sub * BN + col0;
                auto release = [&] {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote_relaxed(te);
                };
                if (p.direct)
                    epilogue_rows_direct<BN>(p, t_row, m0, col0, mode, lane, p.M, release);
                else
                    epilogue_rows<BN>(p, &tmap_y, t_row, m0, col0, stg, mode, lane, p.M, release);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(PC::kTmemCols)
                     : "memory");
    }
}

// ------------------------------------------------------------------------
// Plane kernel (2-SM, resident weights, Cin a multiple of 64): every input
// pixel a CTA needs for a window of 128 output pixels is copied into shared
// memory once per "plane", and the KH x KW taps become offsets into it.
//
// Write tap (kh, kw) as kh - pad = s qh + rh and kw - pad = s qw + rw (floor
// division by the stride s, 0 <= rh, rw < s).  Its input pixel for output
// (ho, wo) is x[s (ho + qh) + rh][s (wo + qw) + rw].  For each distinct
// (rh, rw, qw) -- a "plane" -- entry e of a window holds, for output position
// d = a + e (a = the window's first output pixel, d = ho Wo + wo),
// x[s (ho + min_qh) + rh][s (wo + qw) + rw] (zero outside the image), where
// min_qh is the smallest qh of the plane's taps.  Tap (kh, kw) of window row
// j then reads entry j + (qh - min_qh) Wo: the same shift for every row, so
// its A operand is the plane starting at a fixed entry.  A 3x3 stride-1 conv
// has 3 planes (qw = -1, 0, 1), a stride-2 one 6 (row phase x column phase /
// shift), a 1x1 one plane (the input rows themselves).  For the batch-32 3x3
// stride-2 convolution a window reads 936 pixel rows against 1152 for nine
// per-tap im2col copies.
//
// Each plane of a window is ONE im2col tensor copy: base pixel = the window's
// first output position, im2col offsets (s qw + rw + pad, s min_qh + rh +
// pad) -- a tap's kw and the plane's smallest kh -- and 128 + (max_qh -
// min_qh) Wo pixels.  The copy engine walks output positions through the
// bounding box; the box is extended by the planes' largest row span below
// the last output row, so entries past an image's last row are that image's
// (zero-padded) rows, not the next image's.  The copy writes entry e as row e
// of a K-major SWIZZLE_128B operand (channel block cb: one copy each).  Tap
// shifts are multiples of Wo rows and windows start at multiples of 128, so
// with Wo a multiple of 8 every tap's operand starts on an 8-row swizzle
// atom and its descriptor is the usual one.
//
// Windows are 128 consecutive output pixels of one image (the last window of
// an image may be shorter; Ho * Wo must be a multiple of 32 so that each
// epilogue warp's 32-row box is either complete or empty).  A CTA pair takes
// windows 2 t and 2 t + 1 as the 256 rows of one cta_group::2 MMA tile.
// Each CTA keeps its half of the weights (BN/2 output channels x all of K)
// resident, loaded once by tensor copies.
//
// Roles: one producer thread issues each (window, plane)'s copies into a ring
// of `slots` plane buffers (both CTAs' copies complete on the leader's
// barrier, no multicast); the MMA issuer runs the taps of each plane as soon
// as it has landed and frees the slot with a multicast commit; eight
// epilogue warps drain the double-buffered accumulator as in the kernels
// above.
constexpr int kMaxPlanes = 16;
constexpr int kMaxTaps = 25;
constexpr int kPlaneMaxSlots = 12;

struct PlaneGeo {
    uint32_t nplanes, ntaps;
    int32_t rh[kMaxPlanes], rw[kMaxPlanes], qw[kMaxPlanes], min_qh[kMaxPlanes];
    uint32_t entries[kMaxPlanes];    // entries copied per window (the copy's pixel count)
    uint32_t cb_bytes[kMaxPlanes];   // bytes of one channel block of the plane (entries * 128)
    uint32_t map[kMaxPlanes];        // tensor map of the plane's copies (0 or 1: its pixel count)
    uint32_t off_w[kMaxPlanes], off_h[kMaxPlanes];  // im2col offsets of the plane
    uint32_t tap_end[kMaxPlanes];    // taps [tap_end[v - 1], tap_end[v]) read plane v
    uint32_t tap_aoff[kMaxTaps];     // byte offset of the tap's first row: (qh - min_qh) Wo 128
    uint32_t tap_kb[kMaxTaps];       // first weight k-block of the tap: (kh KW + kw) cblocks
    uint32_t slots, slot_bytes;
    uint32_t e_map[2];               // pixels per copy of tensor maps 0 and 1
    uint32_t row_span;               // largest max_qh - min_qh of a plane (bounding-box extension)
    uint32_t P;                      // output pixels per image (Ho * Wo)
    uint32_t wpi;                    // windows per image
    uint32_t windows, tiles;         // N * wpi, ceil(windows / 2)
};

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    conv_plane_kernel(const Params p, const PlaneGeo g, const __grid_constant__ CUtensorMap tmap_x0,
                      const __grid_constant__ CUtensorMap tmap_x1, const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_y) {
    using PC = PairCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* b_res = smem;
    uint8_t* slots = b_res + p.num_kb * PC::kHalfB;
    uint8_t* staging = slots + g.slots * g.slot_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + 256u * BN);
    uint64_t* empty = full + kPlaneMaxSlots;
    uint64_t* tfull = empty + kPlaneMaxSlots;
    uint64_t* tempty = tfull + 2;
    uint64_t* bfull = tempty + 2;
    uint64_t* drain = bfull + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    if (p.box_cols != (uint32_t)Epi<BN>::kCols) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.err, kErrConfig);
        return;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t pair_id = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < g.slots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * kEpiWarps);
        }
        mbar_init(bfull, 1);
        mbar_init(drain, 1);
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(2u * BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // --------------------------------------- tensor-copy producer
            tma_prefetch_map(&tmap_x0);
            tma_prefetch_map(&tmap_x1);
            tma_prefetch_map(&tmap_w);
            // Resident weights, once, in ONE copy: output channels [rank BN/2,
            // (rank + 1) BN/2) of all num_kb k-blocks (a 3-D box over (64
            // channels, Cout, k-block) lands k-block-major, each k-block a
            // K-major SWIZZLE_128B block of BN/2 rows).
            if (leader) mbar_expect_tx(bfull, 2u * p.num_kb * PC::kHalfB);
            tma_load_3d_pair(smem_u32(b_res), &tmap_w, 0, (int32_t)(rank * (BN / 2)), 0, map_to_rank(bfull, 0));
            const uint32_t lead_full0 = map_to_rank(&full[0], 0), slot0 = smem_u32(slots);
            uint32_t slot = 0, phase = 0, issued = 0;
            bool ok = true;
            for (uint32_t tile = pair_id; ok && tile < g.tiles; tile += num_pairs) {
                // This CTA's window; past the last one it copies the last
                // window again (its rows are never stored).
                uint32_t win = tile * 2u + rank;
                if (win >= g.windows) win = g.windows - 1u;
                const uint32_t n = win / g.wpi, a = (win - n * g.wpi) * 128u;
                const uint32_t ho = a / p.Wo, wo = a - ho * p.Wo;
                const int32_t w0 = (int32_t)(wo * p.stride) - (int32_t)p.pad;
                const int32_t h0 = (int32_t)(ho * p.stride) - (int32_t)p.pad;
                for (uint32_t v = 0; v < g.nplanes; ++v) {
                    if (!mbar_wait_cluster(&empty[slot], phase ^ 1u, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    const uint32_t cbb = g.cb_bytes[v];
                    if (leader) mbar_expect_tx(&full[slot], 2u * cbb * p.cblocks);
                    const CUtensorMap* m = g.map[v] ? &tmap_x1 : &tmap_x0;
                    for (uint32_t cb = 0; cb < p.cblocks; ++cb)
                        tma_load_im2col_4d_pair(slot0 + slot * g.slot_bytes + cb * cbb, m, (int32_t)(cb * 64u), w0,
                                                h0, (int32_t)n, (uint16_t)g.off_w[v], (uint16_t)g.off_h[v],
                                                lead_full0 + slot * 8u);
                    ++issued;
                    if (++slot == g.slots) {
                        slot = 0;
                        phase ^= 1u;
                    }
                }
            }
            // After an abort: both CTAs' copies complete on the leader's
            // barriers, so the leader waits (bounded) for the weights and the
            // last slots before the pair ends (at once when they have all
            // been consumed); the final cluster barrier keeps the other CTA
            // alive meanwhile.
            if (leader) {
                mbar_drain(bfull, 0, 100000000ull);
                drain_loads(full, issued, g.slots);
            }
        }
    } else if (warp == kMmaWarp) {
        if (leader && lane == 0) {
            // ------------------------------------------------ MMA issuer
            // kind::f16, f32 accumulate, bf16 A and B, both K-major, M = 256.
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                   ((256u >> 4) << 24);
            constexpr uint64_t kmaj = smem_desc_sw128_kmajor();
            const uint32_t slot0 = smem_u32(slots), b0 = smem_u32(b_res);
            uint32_t slot = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = mbar_wait_cluster(bfull, 0, abort_flag, p.err, p.wait_ns);
            for (uint32_t tile = pair_id; ok && tile < g.tiles; tile += num_pairs) {
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag, p.err, p.wait_ns)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * (uint32_t)BN;
                uint32_t accumulate = 0, t = 0;
                for (uint32_t v = 0; v < g.nplanes; ++v) {
                    if (!mbar_wait_cluster(&full[slot], phase, abort_flag, p.err, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t plane = slot0 + slot * g.slot_bytes, cbb = g.cb_bytes[v];
                    for (; t < g.tap_end[v]; ++t) {
                        const uint32_t a_t = plane + g.tap_aoff[t];
                        for (uint32_t cb = 0; cb < p.cblocks; ++cb) {
                            const uint32_t a_addr = a_t + cb * cbb;
                            const uint32_t b_addr = b0 + (g.tap_kb[t] + cb) * PC::kHalfB;
#pragma unroll
                            for (uint32_t ks = 0; ks < 4; ++ks) {
                                const uint64_t ad = kmaj | (uint64_t)(((a_addr + ks * 32u) >> 4) & 0x3fffu);
                                const uint64_t bd = kmaj | (uint64_t)(((b_addr + ks * 32u) >> 4) & 0x3fffu);
                                tc_mma_pair(d_tmem, ad, bd, idesc, accumulate);
                                accumulate = 1u;
                            }
                        }
                    }
                    tc_commit_pair_mc(&empty[slot], 0x3);
                    if (++slot == g.slots) {
                        slot = 0;
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
    } else if (warp > kMmaWarp) {
        // ---------------------------------------------------- epilogue
        // Warp e (0..7): TMEM lane quadrant warp % 4 (window rows qd 32 ..
        // qd 32 + 31), column half e / 4; the accumulator is released on the
        // leader's barrier.  Rows past the window's end are not stored.
        const uint32_t e = warp - 5u, qd = warp & 3u, half = e >> 2;
        const uint32_t col0 = half * (uint32_t)(BN / 2);
        const uint32_t stg = smem_u32(staging) + e * Epi<BN>::kWarpBytes;
        const int mode = epi_mode(p);
        const uint32_t lead_tempty0 = map_to_rank(&tempty[0], 0);
        if (lane == 0) tma_prefetch_map(&tmap_y);
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t tile = pair_id; tile < g.tiles; tile += num_pairs) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag, p.err, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            const uint32_t win = tile * 2u + rank;
            uint32_t row0 = 0, row_end = 0;  // global output rows of the window
            if (win < g.windows) {
                const uint32_t n = win / g.wpi, a = (win - n * g.wpi) * 128u;
                row0 = n * g.P + a;
                row_end = n * g.P + min(g.P, a + 128u);
            }
            const uint32_t te = lead_tempty0 + acc * 8u;
            epilogue_rows<BN>(p, &tmap_y, tmem_base + ((qd * 32u) << 16) + acc * (uint32_t)BN + col0,
                              row0 + qd * 32u, col0, stg, mode, lane, row_end, [&] {
                                  tc_fence_before();
                                  __syncwarp();
                                  if (lane == 0) mbar_arrive_remote_relaxed(te);
                              });
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(2u * BN)
                     : "memory");
    }
}

// Launch with programmatic stream serialization (the kernels' set-up may
// overlap the previous kernel's tail; they wait for it before touching
// global memory).  FOIL_CONV_PDL=0 launches plainly (for comparisons).
static bool use_pdl() {
    static const bool on = pdl_enabled("FOIL_CONV_PDL");
    return on;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_conv(void (*kernel)(KArgs...), uint32_t grid, size_t smem, cudaStream_t stream,
                               Args&&... args) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = use_pdl() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <int BN, bool kTma, bool kDirect>
static int launch_bn(const Params& p, const CUtensorMap& mx, const CUtensorMap& mw,
                     const CUtensorMap& my, cudaStream_t stream, int max_ctas) {
    using C = Cfg<BN, kDirect>;
    if (foil_smem_optin((const void*)conv_kernel<BN, kTma, kDirect>, C::kSmemBytes) != cudaSuccess) {
        foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: cudaFuncSetAttribute failed");
        return FOIL_ERR_CUDA;
    }
    const uint32_t tiles = p.m_blocks * p.n_blocks;
    const uint32_t grid = tiles < (uint32_t)max_ctas ? tiles : (uint32_t)max_ctas;
    cudaError_t e = launch_conv(conv_kernel<BN, kTma, kDirect>, grid, C::kSmemBytes, stream, p, mx, mw, my);
    if (e != cudaSuccess) {
        char buf[200];
        snprintf(buf, sizeof buf, "foil_conv2d_nhwc: launch failed: %s", cudaGetErrorString(e));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

// Shared memory of the pair kernel: resident weights, `stages` A stages,
// epilogue staging, barriers (+ 1 KiB alignment slack).
static uint32_t pair_smem_bytes(const Params& p, int bn, uint32_t stages) {
    const uint32_t sub = bn <= 128 ? 2u : 1u;
    return p.num_kb * (uint32_t)(bn / 2) * 128u + stages * sub * 16384u + (p.direct ? 0u : 256u * (uint32_t)bn) +
           1024u + (uint32_t)kBarrierBytes;
}

template <int BN>
static int launch_pair(const Params& p, uint32_t stages, const CUtensorMap& mx, const CUtensorMap& mw,
                       const CUtensorMap& my, cudaStream_t stream, int max_ctas, int smem_optin) {
    if (foil_smem_optin((const void*)conv_pair_kernel<BN>, smem_optin) != cudaSuccess) {
        foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: cudaFuncSetAttribute failed");
        return FOIL_ERR_CUDA;
    }
    const uint32_t max_pairs = (uint32_t)max_ctas / 2;
    const uint32_t pairs = p.m_blocks < max_pairs ? p.m_blocks : max_pairs;
    cudaError_t e = launch_conv(conv_pair_kernel<BN>, 2 * pairs, pair_smem_bytes(p, BN, stages), stream, p, mx, mw,
                                my, stages);
    if (e != cudaSuccess) {
        char buf[200];
        snprintf(buf, sizeof buf, "foil_conv2d_nhwc: launch failed: %s", cudaGetErrorString(e));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

// Shared memory of the resident-weight single-CTA kernel.
static uint32_t res_smem_bytes(const Params& p, int bn, uint32_t stages) {
    return p.num_kb * (uint32_t)bn * 128u + stages * 16384u + 256u * (uint32_t)bn + 1024u +
           (uint32_t)kBarrierBytes;
}

template <int BN>
static int launch_res(const Params& p, uint32_t stages, const CUtensorMap& mx, const CUtensorMap& mw,
                      const CUtensorMap& my, cudaStream_t stream, int max_ctas, int smem_optin) {
    if (foil_smem_optin((const void*)conv_res_kernel<BN>, smem_optin) != cudaSuccess) {
        foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: cudaFuncSetAttribute failed");
        return FOIL_ERR_CUDA;
    }
    const uint32_t grid = p.m_blocks < (uint32_t)max_ctas ? p.m_blocks : (uint32_t)max_ctas;
    cudaError_t e = launch_conv(conv_res_kernel<BN>, grid, res_smem_bytes(p, BN, stages), stream, p, mx, mw, my,
                                stages);
    if (e != cudaSuccess) {
        char buf[200];
        snprintf(buf, sizeof buf, "foil_conv2d_nhwc: launch failed: %s", cudaGetErrorString(e));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

// Plane-kernel geometry (see conv_plane_kernel).  False when the shape is
// not served: Cin not a multiple of 64, more than 25 taps or 16 planes, Ho Wo
// not a multiple of 32, Wo not a multiple of 8, a plane span above 256
// pixels, Cout above 256, or fewer than two plane slots fit.
static int floor_div(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

static bool plane_geometry(const Params& p, int bn, uint32_t optin, PlaneGeo& g, uint32_t& smem) {
    memset(&g, 0, sizeof g);
    if (p.Cin % 64 != 0 || p.KH * p.KW > (uint32_t)kMaxTaps || p.stride == 0 || p.stride > 8 || p.pad > 7 ||
        p.Cout > 256 || p.Wo == 0)
        return false;
    const uint32_t P = p.Ho * p.Wo;
    if (P % 32 != 0 || p.Wo % 8 != 0) return false;
    struct Tap {
        uint32_t v, kb;
        int qh;
    } taps[kMaxTaps];
    int max_qh[kMaxPlanes];
    const int s = (int)p.stride;
    uint32_t nt = 0;
    for (uint32_t kh = 0; kh < p.KH; ++kh)
        for (uint32_t kw = 0; kw < p.KW; ++kw) {
            const int dh = (int)kh - (int)p.pad, dw = (int)kw - (int)p.pad;
            const int qh = floor_div(dh, s), rh = dh - qh * s, qw = floor_div(dw, s), rw = dw - qw * s;
            uint32_t v = 0;
            while (v < g.nplanes && !(g.rh[v] == rh && g.rw[v] == rw && g.qw[v] == qw)) ++v;
            if (v == g.nplanes) {
                if (g.nplanes == (uint32_t)kMaxPlanes) return false;
                g.rh[v] = rh;
                g.rw[v] = rw;
                g.qw[v] = qw;
                g.min_qh[v] = qh;
                max_qh[v] = qh;
                ++g.nplanes;
            }
            g.min_qh[v] = g.min_qh[v] < qh ? g.min_qh[v] : qh;
            max_qh[v] = max_qh[v] > qh ? max_qh[v] : qh;
            taps[nt++] = Tap{v, (kh * p.KW + kw) * p.cblocks, qh};
        }
    // Pixel counts of the copies: the smallest and the largest plane span
    // (one im2col tensor map each, at most 256 pixels per copy).
    uint32_t e_lo = ~0u, e_hi = 0, span = 0;
    for (uint32_t v = 0; v < g.nplanes; ++v) {
        const uint32_t e = 128u + (uint32_t)(max_qh[v] - g.min_qh[v]) * p.Wo;
        e_lo = e < e_lo ? e : e_lo;
        e_hi = e > e_hi ? e : e_hi;
        span = (uint32_t)(max_qh[v] - g.min_qh[v]) > span ? (uint32_t)(max_qh[v] - g.min_qh[v]) : span;
    }
    if (e_hi > 256u) return false;
    g.e_map[0] = e_lo;
    g.e_map[1] = e_hi;
    g.row_span = span;
    // Taps grouped by plane (in (kh, kw) order inside a plane).
    uint32_t slot_bytes = 0;
    for (uint32_t v = 0; v < g.nplanes; ++v) {
        const uint32_t e = 128u + (uint32_t)(max_qh[v] - g.min_qh[v]) * p.Wo;
        g.map[v] = e == e_lo ? 0u : 1u;
        g.entries[v] = g.e_map[g.map[v]];
        g.cb_bytes[v] = g.entries[v] * 128u;  // entries: a multiple of 8 (whole 1 KiB swizzle atoms)
        g.off_w[v] = (uint32_t)(s * g.qw[v] + g.rw[v] + (int)p.pad);
        g.off_h[v] = (uint32_t)(s * g.min_qh[v] + g.rh[v] + (int)p.pad);
        const uint32_t bytes = g.cb_bytes[v] * p.cblocks;
        slot_bytes = bytes > slot_bytes ? bytes : slot_bytes;
        for (uint32_t t = 0; t < nt; ++t)
            if (taps[t].v == v) {
                g.tap_aoff[g.ntaps] = (uint32_t)(taps[t].qh - g.min_qh[v]) * p.Wo * 128u;
                g.tap_kb[g.ntaps] = taps[t].kb;
                ++g.ntaps;
            }
        g.tap_end[v] = g.ntaps;
    }
    if (slot_bytes >= (1u << 18)) return false;
    g.slot_bytes = (slot_bytes + 1023u) / 1024u * 1024u;
    const uint32_t fixed = 1024u + p.num_kb * (uint32_t)(bn / 2) * 128u + 256u * (uint32_t)bn + (uint32_t)kBarrierBytes;
    if (fixed >= optin) return false;
    uint32_t slots = (optin - fixed) / g.slot_bytes;
    if (slots > (uint32_t)kPlaneMaxSlots) slots = kPlaneMaxSlots;
    if (slots < 2) return false;
    g.slots = slots;
    g.P = P;
    g.wpi = (P + 127u) / 128u;
    g.windows = p.N * g.wpi;
    g.tiles = (g.windows + 1u) / 2u;
    smem = fixed + slots * g.slot_bytes;
    return true;
}

template <int BN>
static int launch_plane(const Params& p, const PlaneGeo& g, uint32_t smem, const CUtensorMap& mx0,
                        const CUtensorMap& mx1, const CUtensorMap& mw, const CUtensorMap& my,
                        cudaStream_t stream, int max_ctas) {
    if (foil_smem_optin((const void*)conv_plane_kernel<BN>, (int)smem) != cudaSuccess) {
        foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: cudaFuncSetAttribute failed");
        return FOIL_ERR_CUDA;
    }
    const uint32_t max_pairs = (uint32_t)max_ctas / 2;
    const uint32_t pairs = g.tiles < max_pairs ? g.tiles : max_pairs;
    conv_plane_kernel<BN><<<2 * pairs, kThreads, smem, stream>>>(p, g, mx0, mx1, mw, my);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        char buf[200];
        snprintf(buf, sizeof buf, "foil_conv2d_nhwc: launch failed: %s", cudaGetErrorString(e));
        foil_set_error(FOIL_ERR_CUDA, buf);
        return FOIL_ERR_CUDA;
    }
    foil_count_launch();
    return FOIL_OK;
}

template <bool kTma>
static int launch_tiles(const Params& p, int bn, const CUtensorMap& mx, const CUtensorMap& mw,
                        const CUtensorMap& my, cudaStream_t stream, int max_ctas) {
    if (p.direct) {
        switch (bn) {
            case 64: return launch_bn<64, kTma, true>(p, mx, mw, my, stream, max_ctas);
            case 128: return launch_bn<128, kTma, true>(p, mx, mw, my, stream, max_ctas);
            default: return launch_bn<256, kTma, true>(p, mx, mw, my, stream, max_ctas);
        }
    }
    switch (bn) {
        case 64: return launch_bn<64, kTma, false>(p, mx, mw, my, stream, max_ctas);
        case 128: return launch_bn<128, kTma, false>(p, mx, mw, my, stream, max_ctas);
        default: return launch_bn<256, kTma, false>(p, mx, mw, my, stream, max_ctas);
    }
}

// ------------------------------------------------- tensor-map encoding ---
struct Encoders {
    PFN_cuTensorMapEncodeIm2col im2col = nullptr;
    PFN_cuTensorMapEncodeTiled tiled = nullptr;
};

static const Encoders& encoders() {
    static Encoders e;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", (void**)&e.im2col, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            e.im2col = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&e.tiled, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            e.tiled = nullptr;
    });
    return e;
}

// The plane kernel serves Cin a multiple of 64, Cout <= 256, Ho Wo a
// multiple of 32 and up to 9 taps.  Otherwise the tensor-copy producer
// serves Cin a multiple of 64 (one 128-byte channel run per k-block) with a
// traversal stride the copy engine supports (<= 8) and byte strides below
// 2^40, and the gather producer the rest.  FOIL_CONV_PRODUCER=gather selects
// the gather producer for every shape, =single the tensor-copy producer in
// the single-CTA kernel, =pair the im2col pair kernel wherever it can run,
// and =plane the plane kernel, failing with FOIL_ERR_UNSUPPORTED where it
// cannot (A/B comparisons: the first three agree bit for bit; the plane
// kernel sums the same products in plane order, so it agrees within the
// tolerance).
static const char* producer_override() {
    static const char* v = getenv("FOIL_CONV_PRODUCER");
    return v ? v : "";
}

static bool use_tensor_copies(const Params& p) {
    return strcmp(producer_override(), "gather") != 0 && p.Cin % 64 == 0 && p.stride <= 8 &&
           (uint64_t)p.H * p.W * p.Cin * 2 < (1ull << 40);
}

// Output y as an M x Cout matrix, stored in boxes of 32 rows x p.box_cols
// columns: 64 (SWIZZLE_128B) or 32 (SWIZZLE_64B), the epilogue's staging
// boxes (Epi<BN>::kCols, which the kernels check against p.box_cols).
static bool encode_output_map(const Params& p, CUtensorMap* my) {
    const Encoders& e = encoders();
    if (!e.tiled) return false;
    const bool wide = p.box_cols == 64;
    const cuuint64_t ydim[2] = {p.Cout, p.M};
    const cuuint64_t ystr[1] = {(cuuint64_t)p.Cout * 2};
    const cuuint32_t box[2] = {wide ? 64u : 32u, 32};
    const cuuint32_t one[2] = {1, 1};
    return e.tiled(my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.y, ydim, ystr, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_weight_map(const Params& p, uint32_t w_rows, CUtensorMap* mw);

// All weights of one CTA in one box: the K x Cout weight matrix viewed as
// (64 channels, Cout, num_kb k-blocks) with byte strides (K * 2, 128), box
// (64, w_rows, num_kb), SWIZZLE_128B: the box lands k-block-major.
static bool encode_weight_map3(const Params& p, uint32_t w_rows, CUtensorMap* mw) {
    const Encoders& e = encoders();
    if (!e.tiled || p.num_kb > 256) return false;
    const cuuint64_t dim[3] = {64, p.Cout, p.num_kb};
    const cuuint64_t str[2] = {(cuuint64_t)p.KH * p.KW * p.Cin * 2, 128};
    const cuuint32_t box[3] = {64, w_rows, p.num_kb};
    const cuuint32_t one[3] = {1, 1, 1};
    return e.tiled(mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(p.w), dim, str, box, one,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// im2col map of the plane kernel's copies: `pixels` output positions per
// copy, 64 channels, traversal stride = the conv stride, and the bounding
// box of base pixels [-pad, dim - 1 + pad - (k - 1)] extended below the last
// output row by the planes' largest row span (g.row_span output rows), so a
// copy that runs past an image's last output row reads that image's
// zero-padded rows rather than the next image.
static bool encode_plane_map(const Params& p, const PlaneGeo& g, uint32_t pixels, CUtensorMap* mx) {
    const Encoders& e = encoders();
    if (!e.im2col) return false;
    const cuuint64_t xdim[4] = {p.Cin, p.W, p.H, p.N};
    const cuuint64_t xstr[3] = {(cuuint64_t)p.Cin * 2, (cuuint64_t)p.W * p.Cin * 2,
                                (cuuint64_t)p.H * p.W * p.Cin * 2};
    const int lower[2] = {-(int)p.pad, -(int)p.pad};
    const int upper[2] = {(int)p.pad - (int)(p.KW - 1),
                          (int)p.pad - (int)(p.KH - 1) + (int)(p.stride * g.row_span)};
    const cuuint32_t trav[4] = {1, p.stride, p.stride, 1};
    return e.im2col(mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(p.x), xdim, xstr, lower, upper,
                    64, pixels, trav, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A (im2col of x) and weights as a K x Cout matrix read in boxes of 64
// channels x `w_rows` output channels (BN, or BN/2 per CTA of a pair).
static bool encode_maps(const Params& p, uint32_t w_rows, uint32_t pixels, CUtensorMap* mx, CUtensorMap* mw) {
    const Encoders& e = encoders();
    if (!e.im2col || !e.tiled) return false;
    // Dims and byte strides innermost first: C, W, H, N.
    const cuuint64_t xdim[4] = {p.Cin, p.W, p.H, p.N};
    const cuuint64_t xstr[3] = {(cuuint64_t)p.Cin * 2, (cuuint64_t)p.W * p.Cin * 2,
                                (cuuint64_t)p.H * p.W * p.Cin * 2};
    // Bounding box of the base pixels (tap (0, 0)) per spatial dim, W first:
    // [-pad, dim - 1 + pad - (k - 1)].
    const int lower[2] = {-(int)p.pad, -(int)p.pad};
    const int upper[2] = {(int)p.pad - (int)(p.KW - 1), (int)p.pad - (int)(p.KH - 1)};
    const cuuint32_t trav[4] = {1, p.stride, p.stride, 1};
    if (e.im2col(mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(p.x), xdim, xstr, lower,
                 upper, 64, pixels, trav, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    return encode_weight_map(p, w_rows, mw);
}

// Weights as a K x Cout matrix (K = KH * KW * Cin contiguous per row), read
// in boxes of 64 channels x `w_rows` output channels, SWIZZLE_128B.
static bool encode_weight_map(const Params& p, uint32_t w_rows, CUtensorMap* mw) {
    const Encoders& e = encoders();
    if (!e.tiled) return false;
    const cuuint64_t wdim[2] = {(cuuint64_t)p.KH * p.KW * p.Cin, p.Cout};
    const cuuint64_t wstr[1] = {(cuuint64_t)p.KH * p.KW * p.Cin * 2};
    const cuuint32_t box[2] = {64, w_rows};
    const cuuint32_t one[2] = {1, 1};
    return e.tiled(mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(p.w), wdim, wstr, box,
                   one, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y, uint32_t N,
           uint32_t H, uint32_t W, uint32_t Cin, uint32_t Cout, uint32_t KH, uint32_t KW,
           uint32_t stride, uint32_t pad, int relu, uint32_t* err, cudaStream_t stream,
           int max_ctas) {
    Params p;
    p.x = x;
    p.w = w;
    p.bias = bias;
    p.y = y;
    p.N = N;
    p.H = H;
    p.W = W;
    p.Cin = Cin;
    p.Cout = Cout;
    p.KH = KH;
    p.KW = KW;
    p.stride = stride;
    p.pad = pad;
    p.Ho = (H + 2 * pad - KH) / stride + 1;
    p.Wo = (W + 2 * pad - KW) / stride + 1;
    p.M = N * p.Ho * p.Wo;
    p.kc = Cin % 64 == 0 ? 64 : (Cin % 32 == 0 ? 32 : 16);
    p.cblocks = Cin / p.kc;
    p.num_kb = KH * KW * p.cblocks;
    p.relu = relu;
    p.err = err;
    p.wait_ns = foil_wait_limit_ns();
    p.m_blocks = (p.M + 127) / 128;
    // Epilogue store path: the pair kernel stores rows from registers by
    // default (its staging buffer then holds a fourth operand stage: 3x3
    // stride-2 batch 32, L2 flushed, 27.7-27.9 against 28.9-29.3 us), the
    // single-CTA kernel stages for tensor stores (1x1 batch 32: 20.5-20.7
    // against 27.2-27.5 us from registers).  FOIL_CONV_EPILOGUE=direct or
    // staged forces one path (tests compare both).
    const char* ep = getenv("FOIL_CONV_EPILOGUE");
    const bool force_direct = ep != nullptr && strcmp(ep, "direct") == 0;
    const bool force_staged = ep != nullptr && strcmp(ep, "staged") == 0;
    p.wide_y = ((uintptr_t)y & 31u) == 0 ? 1u : 0u;
    p.direct = force_staged ? 0u : 1u;  // the pair kernel's default
    // Column tile: the smallest of 64 / 128 / 256 covering Cout, else 256.
    const int bn = Cout <= 64 ? 64 : (Cout <= 128 ? 128 : 256);
    p.n_blocks = (Cout + bn - 1) / bn;
    alignas(64) CUtensorMap mx, mw, my;
    memset(&mx, 0, sizeof mx);
    memset(&mw, 0, sizeof mw);
    const bool tc = use_tensor_copies(p);
    p.box_cols = bn >= 128 ? 64u : 32u;  // Epi<bn>::kCols
    if (!encode_output_map(p, &my)) {
        foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: tensor-map encoding failed");
        return FOIL_ERR_CUDA;
    }
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
        foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: device query failed");
        return FOIL_ERR_CUDA;
    }
    // Plane kernel (2-SM, resident weights, taps as offsets into one copy
    // per plane): only on request.  Measured on the batch-32 configurations
    // (L2 flushed) it trails the im2col kernels below: 3x3 stride 2 36.7
    // against 29.3 us, 1x1 23.5 against 21.9 us, and the N = 1 3x3 14.1
    // against 13.9 us; it moves fewer operand bytes but issues more copies.
    const char* ov = producer_override();
    if (max_ctas >= 2 && strcmp(ov, "plane") == 0) {
        PlaneGeo g;
        uint32_t smem = 0;
        if (plane_geometry(p, bn, (uint32_t)optin, g, smem)) {
            alignas(64) CUtensorMap mx1;
            if (!encode_weight_map3(p, (uint32_t)bn / 2, &mw) || !encode_plane_map(p, g, g.e_map[0], &mx) ||
                !encode_plane_map(p, g, g.e_map[1], &mx1)) {
                foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: tensor-map encoding failed");
                return FOIL_ERR_CUDA;
            }
            switch (bn) {
                case 64: return launch_plane<64>(p, g, smem, mx, mx1, mw, my, stream, max_ctas);
                case 128: return launch_plane<128>(p, g, smem, mx, mx1, mw, my, stream, max_ctas);
                default: return launch_plane<256>(p, g, smem, mx, mx1, mw, my, stream, max_ctas);
            }
        }
    }
    if (strcmp(ov, "plane") == 0) {
        foil_set_error(FOIL_ERR_UNSUPPORTED, "foil_conv2d_nhwc: FOIL_CONV_PRODUCER=plane but the plane kernel "
                                             "does not serve this shape");
        return FOIL_ERR_UNSUPPORTED;
    }
    if (!tc) {
        p.direct = force_direct ? 1u : 0u;
        return launch_tiles<false>(p, bn, mx, mw, my, stream, max_ctas);
    }
    // Weight-stationary pair kernel: one column block, more than one 128-row
    // block, and at least 3 A stages beside the resident weights.
    uint32_t stages = 0;
    while (stages < (uint32_t)kPairMaxStages && pair_smem_bytes(p, bn, stages + 1) <= (uint32_t)optin) ++stages;
    // The pair kernel pays ~1 us more start-up (cluster launch, resident
    // weights); it needs one column block and at least 3 A stages beside the
    // resident weights.
    const bool pair_ok = p.n_blocks == 1 && p.M > 128 && stages >= 3 && max_ctas >= 2;
    // Measured: the pair kernel wins on the 3x3 stride-2 batch-32 convolution
    // (9 k-blocks; 23.5 against 31.5 us) and loses on the 1x1 one (2
    // k-blocks; 18.8 against 16.8 us), where weights are a small share of the
    // operand copies and the start-up is not amortised.
    const bool pair = pair_ok && strcmp(producer_override(), "single") != 0 &&
                      strcmp(producer_override(), "resident") != 0 &&
                      (strcmp(producer_override(), "pair") == 0 ||
                       (p.num_kb >= 4 && p.m_blocks >= (uint32_t)max_ctas));
    const uint32_t sub = bn <= 128 ? 2u : 1u;
    if (!encode_maps(p, pair ? (uint32_t)bn / 2 : (uint32_t)bn, pair ? 128u * sub : 128u, &mx, &mw) ||
        (pair && !encode_weight_map3(p, (uint32_t)bn / 2, &mw))) {
        foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: tensor-map encoding failed");
        return FOIL_ERR_CUDA;
    }
    if (pair) {
        Params q = p;
        q.m_blocks = (p.M + 256u * sub - 1u) / (256u * sub);
        switch (bn) {
            case 64: return launch_pair<64>(q, stages, mx, mw, my, stream, max_ctas, optin);
            case 128: return launch_pair<128>(q, stages, mx, mw, my, stream, max_ctas, optin);
            default: return launch_pair<256>(q, stages, mx, mw, my, stream, max_ctas, optin);
        }
    }
    // Resident-weight single-CTA kernel: one column block, at least 4 A
    // stages beside the weights.  Measured (L2 flushed, three alternating
    // rounds): 1x1 batch 32 128 -> 256 18.9-19.0 against 20.1-20.4 us for the
    // streaming kernel, 3x3 N = 1 64 -> 64 11.4-11.9 against 12.9-13.2 us.
    uint32_t rstages = 0;
    while (rstages < (uint32_t)kResMaxStages && res_smem_bytes(p, bn, rstages + 1) <= (uint32_t)optin) ++rstages;
    const bool res = p.n_blocks == 1 && rstages >= 4 && strcmp(producer_override(), "single") != 0;
    if (res) {
        if (!encode_weight_map3(p, (uint32_t)bn, &mw)) {
            foil_set_error(FOIL_ERR_CUDA, "foil_conv2d_nhwc: tensor-map encoding failed");
            return FOIL_ERR_CUDA;
        }
        p.direct = 0u;
        switch (bn) {
            case 64: return launch_res<64>(p, rstages, mx, mw, my, stream, max_ctas, optin);
            case 128: return launch_res<128>(p, rstages, mx, mw, my, stream, max_ctas, optin);
            default: return launch_res<256>(p, rstages, mx, mw, my, stream, max_ctas, optin);
        }
    }
    if (strcmp(producer_override(), "resident") == 0) {
        foil_set_error(FOIL_ERR_UNSUPPORTED, "foil_conv2d_nhwc: FOIL_CONV_PRODUCER=resident but the resident-weight "
                                             "kernel does not serve this shape");
        return FOIL_ERR_UNSUPPORTED;
    }
    p.direct = force_direct ? 1u : 0u;
    return launch_tiles<true>(p, bn, mx, mw, my, stream, max_ctas);
}

}  // namespace conv
}  // namespace foil
