// PTX wrappers shared by the tcgen05 GEMM kernels (sm_100a): mbarriers with
// bounded waits, cp.async, tcgen05 MMA / commit / TMEM loads, cluster
// helpers, and the shared-memory / instruction descriptor encodings.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace foil {
namespace gemm {

// ---------------------------------------------------------------- PTX ---
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Suspend hint of the waiting forms below: the thread sleeps until the phase
// completes or about this many nanoseconds pass, so a warp waiting for a
// barrier leaves the issue slots to the warps that do the work (a plain
// try_wait returns at once and the wait loop would spin).
constexpr uint32_t kSuspendNs = 10000u;

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return done != 0;
}

// Default wall-time limit of one bounded wait (the kernels take the limit
// as a launch parameter; foil_set_wait_limit_ns changes it).
constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;  // 2 s per wait

// Wait for completion of phase `parity`.  Returns false if the CTA is
// aborting or this wait exceeded `limit_ns` of wall time (then it raises the
// abort flag and records the error).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile uint32_t* abort_flag, uint32_t* err,
                                          uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
#pragma unroll 1
    while (true) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > limit_ns) {
            *abort_flag = 1u;
            if (err) atomicOr(err, kErrWaitTimeout);
            return false;
        }
    }
}

// Bounded drain wait used on the way out (ignores the abort flag).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
#pragma unroll 1
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (global_ns() - t0 > limit_ns) return;
    }
}

// 16-byte global->shared copy; src_bytes = 0 writes zeros (out-of-range
// tiles).  .cg: cached in L2 only.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}

// Arrive on `bar` once every cp.async issued so far by this thread is done
// (counts toward the barrier's expected arrivals).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 format): start >> 4 in [0,14),
// LBO >> 4 in [16,30), SBO >> 4 in [32,46), fixed version bit 46, layout type
// in [61,64) (6 = SWIZZLE_32B).
__host__ __device__ constexpr uint64_t smem_desc_base(uint32_t lbo, uint32_t sbo) {
    return ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) | ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) |
           (1ull << 46) | (6ull << 61);
}

// K-major operand written by a SWIZZLE_128B tensor copy: rows of 128 bytes,
// 8-row atoms 1024 bytes apart (SBO), layout type 2 = SWIZZLE_128B.  A
// K-step of 16 bf16 (32 bytes) inside the atom advances the start address.
__host__ __device__ constexpr uint64_t smem_desc_sw128_kmajor() {
    return (1ull << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// ------------------------------------------------ tensor copies (no multicast)
// The tensor map is a __grid_constant__ kernel parameter; its generic address
// is the operand.  Completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_prefetch_map(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load: box origin (x = inner element index, y = row).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* map, int32_t x, int32_t y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 4-D im2col load of an NHWC tensor (dims C, W, H, N): pixelsPerColumn
// pixels, traversed from the base pixel (c, w, h, n) through the map's
// bounding box, each read at (w + off_w, h + off_h); out-of-range pixels are
// zero-filled.
__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const void* map, int32_t c,
                                                   int32_t w, int32_t h, int32_t n, uint16_t off_w,
                                                   uint16_t off_h, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n), "r"(smem_u32(bar)),
        "h"(off_w), "h"(off_h)
        : "memory");
}

// 3-D tiled load: box origin (x, y, z).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Pair (cta_group::2) forms, no multicast: the destination is this CTA's
// shared memory and completion is signalled on the mbarrier at shared::cluster
// address `bar_cluster`, which may be the pair leader's.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* map, int32_t x, int32_t y,
                                                 uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}

// 3-D tiled load, pair form (see tma_load_2d_pair).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* map, int32_t x, int32_t y, int32_t z,
                                                 uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar_cluster)
        : "memory");
}

__device__ __forceinline__ void tma_load_im2col_4d_pair(uint32_t dst, const void* map, int32_t c,
                                                        int32_t w, int32_t h, int32_t n, uint16_t off_w,
                                                        uint16_t off_h, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.4d.im2col.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n), "r"(bar_cluster),
        "h"(off_w), "h"(off_h)
        : "memory");
}

// 2-D tiled store from shared memory (bulk group of this thread); elements of
// the box outside the tensor are not written.  Coordinates must be >= 0.
__device__ __forceinline__ void tma_store_2d(const void* map, int32_t x, int32_t y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}

// Instruction descriptor for kind::f16: f32 accumulate (bits 4-5 = 1), bf16
// A and B (bits 7-9, 10-12 = 1), A K-major (bit 15 = 0), B MN-major (bit 16
// = 1), N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t m, uint32_t n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (0u << 15) | (1u << 16) | ((n >> 3) << 17) |
           ((m >> 4) << 24);
}

// 32 consecutive TMEM columns of this warp's 32 lanes (one row per lane).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr));
}

// 256-bit global store of w[0..7] (address 32-byte aligned).
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t* w) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
}

// 16-byte store through an NVLink multicast address (multimem): the one
// store reaches the same offset of every GPU's buffer bound to the multicast
// object, replicated by the NVSwitch.  16-byte aligned; the words are bf16
// pairs, stored unchanged.
__device__ __forceinline__ void st_multimem_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
}

// 256-bit global load through L2 only (no L1 allocation), 32-byte aligned.
__device__ __forceinline__ void ld_global_cg_v8(const void* p, uint32_t* w) {
    asm volatile("ld.global.cg.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]),
                   "=r"(w[7])
                 : "l"(p)
                 : "memory");
}

// Wait (bounded, like mbar_wait) until the shared-memory counter reaches
// `target`.  Returns false on abort or timeout.
__device__ __forceinline__ bool wait_count(const volatile uint32_t* counter, uint32_t target,
                                           volatile uint32_t* abort_flag, uint32_t* err,
                                           uint64_t limit_ns) {
    if (*counter >= target) return true;
    const uint64_t t0 = global_ns();
#pragma unroll 1
    while (*counter < target) {
        if (*abort_flag) return false;
        if (global_ns() - t0 > limit_ns) {
            *abort_flag = 1u;
            if (err) atomicOr(err, kErrWaitTimeout);
            return false;
        }
    }
    return true;
}

// Bulk (non-tensor) global -> shared copy of `bytes` (multiple of 16, both
// addresses 16-byte aligned), completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bulk (non-tensor) shared -> global copy of `bytes` (multiple of 16, both
// addresses 16-byte aligned), tracked by this thread's bulk groups.
__device__ __forceinline__ void bulk_store(void* gdst, uint32_t ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
                 "r"(ssrc), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until this thread's bulk copies no longer read their shared source.
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until at most N of this thread's most recent bulk groups still read
// their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read_n() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until this thread's bulk copies are complete.
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ------------------------------------------------------- cluster (pairs) ---
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

// Arrive on an mbarrier of another CTA of the cluster (release, cluster scope).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

// Relaxed remote arrive, for the per-stage "operands landed" relay.  The
// release form makes the arriving thread wait for a cluster-scope fence,
// which measured ~35% of GEMM throughput when issued once per k-block; the
// relay publishes no data of its own (the operands are already complete in
// shared memory when its local barrier fires), so relaxed ordering suffices.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_try_wait_cluster_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return done != 0;
}

// Bounded wait (acquire at cluster scope) for barriers that receive arrivals
// from the other CTA of the pair.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile uint32_t* abort_flag, uint32_t* err,
                                                  uint64_t limit_ns) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_ns();
#pragma unroll 1
    while (true) {
        if (mbar_try_wait_cluster_sleep(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > limit_ns) {
            *abort_flag = 1u;
            if (err) atomicOr(err, kErrWaitTimeout);
            return false;
        }
    }
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

// 2-SM MMA: D (256 x N, rows split over the pair's TMEM) += A . B, issued by
// the even CTA; operands are read from both CTAs' shared memory at the same
// offsets.
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on the barrier at this offset in every CTA of `mask` once all prior
// 2-SM MMAs of this thread have completed.
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t* bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
        "[%0], %1;" ::"r"(smem_u32(bar)),
        "h"(mask)
        : "memory");
}

__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

}  // namespace gemm
}  // namespace foil
