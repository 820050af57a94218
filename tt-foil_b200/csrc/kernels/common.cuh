// Shared device helpers for the sm_100a kernels of libfoil.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>

namespace foil {

// bf16 <-> fp32 with the exact arithmetic of the tt-foil CPU golden
// (tests/tile_utils.hpp:33-47): widening is a 16-bit shift; narrowing adds
// 0x7fff plus the lowest kept bit and truncates (round to nearest even, no
// NaN special case).  Using the same integer formula keeps every
// element-wise kernel bit-identical to the golden, NaN payloads included.
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) {
    return __uint_as_float(b << 16);
}

__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return u >> 16;
}

// fp32 addition with the NaN results of the x86-64 build of the reference
// golden (`f(a) + f(b)` compiled to SSE addss / addps): a NaN operand
// propagates quieted, the SECOND operand winning when both are NaN; an
// invalid sum (inf - inf) yields the default NaN 0xffc00000.  The GPU's adder
// returns one canonical NaN instead, so without this the narrowed bf16 of a
// NaN result would differ from the golden.
__device__ __forceinline__ float host_add_f32(float a, float b) {
    const float sum = __fadd_rn(a, b);
    if (sum == sum) return sum;  // no NaN operand and no invalid operation
    const uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    const bool na = (ua & 0x7fffffffu) > 0x7f800000u;
    const bool nb = (ub & 0x7fffffffu) > 0x7f800000u;
    if (nb) return __uint_as_float(ub | 0x00400000u);
    if (na) return __uint_as_float(ua | 0x00400000u);
    return __uint_as_float(0xffc00000u);
}

// Round two fp32 values to bf16 (round to nearest even) and pack them, low
// half = lo.  The hardware conversion gives the golden formula's result for
// every non-NaN input (NaN becomes the canonical NaN); used where parity is
// checked with a tolerance (GEMM / conv epilogues).
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Two bf16 in one 32-bit word (low half = first element).
__device__ __forceinline__ uint32_t pack_bf16x2(uint32_t lo, uint32_t hi) {
    return (lo & 0xffffu) | (hi << 16);
}

// Device-side error codes written to the error word.
enum : uint32_t {
    kErrWaitTimeout = 1u,  // a bounded mbarrier wait gave up
    kErrConfig = 4u,       // launch parameters inconsistent with the kernel instantiation (nothing ran)
    kErrBadShape = 2u,     // kernel saw a shape it cannot handle
};

// Wall-clock nanoseconds (for bounded waits).
// Programmatic dependent launch.  griddep_wait: block until the grids this
// one depends on (the previous kernel in the stream, when launched with
// programmatic stream serialization) have completed and their memory is
// visible; a no-op otherwise.  griddep_launch_dependents: allow the next
// such kernel to start launching (its own griddep_wait still waits for this
// grid to complete).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch attribute for programmatic stream serialization, on unless the
// environment variable `env` is "0" (read once per variable by the caller).
inline bool pdl_enabled(const char* env) {
    const char* v = getenv(env);
    return v == nullptr || v[0] != '0' || v[1] != '\0';
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

}  // namespace foil

// Host-side launch accounting shared by every entry point (defined in
// foil_runtime.cpp).
void foil_count_launch();

// Per-device host caches (defined in foil_runtime.cpp).  A kernel's dynamic
// shared-memory opt-in (cudaFuncSetAttribute) belongs to the current
// device's context, so it is set once per (kernel, device ordinal), not once
// per process; likewise the SM count is read once per device.  Both act on
// the calling thread's current device.
cudaError_t foil_smem_optin(const void* kernel, int bytes);
int foil_sm_count();

// Wall-time limit (ns) of each bounded device-side wait, passed to every
// kernel launch; process-wide, set by foil_set_wait_limit_ns (default 2 s).
uint64_t foil_wait_limit_ns();
