// Allocation-free entry point of the tiled tcgen05 GEMM.
//
// Who it is for: callers that must not allocate device memory at the point
// where they launch the GEMM.  Examples are code running inside an allocator
// or memory-pool callback (where calling back into cudaMalloc can deadlock or
// recurse), a process whose device memory is owned up front by another
// allocator (a framework's caching allocator that has reserved the GPU, so a
// fresh cudaMalloc fails), and latency-bound loops that forbid allocation
// after start-up.  foil_matmul_tiles_dev allocates its 256-byte device error
// word with cudaMalloc on the first call on each device; this variant keeps
// that scratch in an array compiled into the library instead, and otherwise
// launches exactly the same kernel.
//
// Scratch: g_noalloc_scratch is a file-scope __device__ array of
// kNoAllocScratchBytes (256) bytes; word 0 is the GEMM's device error word
// (set when a bounded wait inside the kernel expires).  A call needs 4 bytes;
// a call whose scratch need exceeded the array would be rejected with
// FOIL_ERR_INVALID.  Every GPU that loads libfoil holds the array until the
// process exits.
//
// Set-up: host code cannot use the array's name as a device address (it is a
// host-side shadow symbol).  The first call on each device — with that device
// current — resolves the address with cudaGetSymbolAddress and caches it; make
// that first call before any stream capture begins.
//
// Sharing: every call on a device uses the same array and it keeps the last
// call's contents.  Each call clears the error word on its stream before the
// launch, so calls that overlap on the GPU (for example on two streams) race
// on the word: one may clear or report the other's status.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "../../../include/foil_c.h"

extern "C" void foil_set_error(int status, const char* msg);

namespace {

constexpr size_t kNoAllocScratchBytes = 256;
constexpr size_t kGemmScratchBytes = sizeof(uint32_t);  // the device error word

static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocScratchBytes / 4];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint32_t* g_scratch[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};

int fail(int status, const char* msg) {
    foil_set_error(status, msg);
    return status;
}

}  // namespace

extern "C" int foil_matmul_tiles_noalloc_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                                             uint32_t Mt, uint32_t Kt, uint32_t Nt,
                                             const uint16_t* bias, int32_t relu, void* stream,
                                             uint32_t* status_out) {
    if (status_out) *status_out = 0;
    if (Mt == 0 || Kt == 0 || Nt == 0) return FOIL_OK;
    if (Mt > 65535 || Kt > 65535 || Nt > 65535)
        return fail(FOIL_ERR_INVALID, "foil_matmul_tiles_noalloc_dev: tile counts must be <= 65535");
    auto aligned = [](const void* p) { return p && ((uintptr_t)p & 15u) == 0; };
    if (!aligned(a) || !aligned(b) || !aligned(c) || (bias && !aligned(bias)))
        return fail(FOIL_ERR_INVALID, "foil_matmul_tiles_noalloc_dev: null or misaligned pointer");
    if (kGemmScratchBytes > kNoAllocScratchBytes)
        return fail(FOIL_ERR_INVALID,
                    "foil_matmul_tiles_noalloc_dev: scratch need exceeds the 256-byte static array");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(FOIL_ERR_CUDA, "foil_matmul_tiles_noalloc_dev: no current CUDA device");
    uint32_t* scratch = nullptr;
    int sms = 0;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch[dev]) {
            // Once per device, with the device current: device address of the
            // static array (the host-side name is only a shadow symbol).
            void* ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess || !ptr) {
                char buf[200];
                snprintf(buf, sizeof buf, "foil_matmul_tiles_noalloc_dev: cudaGetSymbolAddress failed: %s",
                         cudaGetErrorString(e));
                return fail(FOIL_ERR_CUDA, buf);
            }
            int n = 0;
            if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
                n = 148;
            g_sms[dev] = n;
            g_scratch[dev] = static_cast<uint32_t*>(ptr);
        }
        scratch = g_scratch[dev];
        sms = g_sms[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The array keeps the previous call's contents: the error word must start at 0.
    if (cudaMemsetAsync(scratch, 0, kGemmScratchBytes, s) != cudaSuccess)
        return fail(FOIL_ERR_CUDA, "foil_matmul_tiles_noalloc_dev: clearing the scratch failed");
    int st = foil::gemm::launch(a, b, c, Mt, Kt, Nt, bias, relu, scratch, s, sms);
    if (st != FOIL_OK) return st;
    if (status_out) {
        if (cudaMemcpyAsync(status_out, scratch, sizeof(uint32_t), cudaMemcpyDeviceToHost, s) !=
                cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess)
            return fail(FOIL_ERR_CUDA, "foil_matmul_tiles_noalloc_dev: reading the status failed");
        if (*status_out != 0)
            return fail(FOIL_ERR_DEVICE,
                        "foil_matmul_tiles_noalloc_dev: a bounded wait in the kernel expired");
    }
    return FOIL_OK;
}
