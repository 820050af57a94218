// C-ABI of the B200 tt-foil runtime (include/foil_c.h) bound to CUDA.
//
// The reference re-backed here: device open/close and bump allocators
// (src/device.cpp, src/buffer.cpp), blocking host transfers
// (src/runtime_impl.cpp:52-78), kernel load and runtime args
// (src/kernel.cpp), CB registration (src/cb_config.cpp) and dispatch
// (src/dispatch.cpp).  Where the reference cold-boots Tensix cores and writes
// ELFs into L1, this file creates HBM arenas and launches CUDA kernels:
//
//  * DRAM arena: a 64 GiB virtual range (cuMemAddressReserve) backed on
//    demand by physical chunks (cuMemCreate / cuMemMap) as the bump pointer
//    grows, so a DRAM offset maps to base + offset with no table.
//  * L1 arenas: one 1.5 MiB device allocation per opened core.
//  * execute: runtime args -> launch plan (host_logic.cpp) -> range-checked
//    device pointers -> CUDA launches on the device's stream -> bounded wait
//    (cudaEventQuery against the caller's deadline) -> device error word.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "../../include/foil_c.h"
#include "host_logic.hpp"
#include "kernels/gemm_tc.cuh"
#include "kernels/conv_tc.cuh"
#include "kernels/eltwise.cuh"
#include "kernels/layout.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

}  // namespace

extern "C" void foil_set_error(int /*status*/, const char* msg) { g_last_error = msg ? msg : ""; }
void foil_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Per-(kernel, device) shared-memory opt-in and per-device SM count; see
// kernels/common.cuh.
namespace {
struct OptinEntry {
    const void* kernel;
    int device;
    int bytes;
};
std::mutex g_optin_mu;
std::vector<OptinEntry> g_optin;
int g_sm_counts[64] = {};
}  // namespace

cudaError_t foil_smem_optin(const void* kernel, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(g_optin_mu);
    for (OptinEntry& x : g_optin)
        if (x.kernel == kernel && x.device == dev) {
            if (x.bytes >= bytes) return cudaSuccess;
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
            if (e == cudaSuccess) x.bytes = bytes;
            return e;
        }
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) g_optin.push_back(OptinEntry{kernel, dev, bytes});
    return e;
}

int foil_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lk(g_optin_mu);
    if (g_sm_counts[dev] <= 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
        g_sm_counts[dev] = n;
    }
    return g_sm_counts[dev];
}

namespace {
constexpr uint64_t kDefaultWaitNs = 2000000000ull;
std::atomic<uint64_t> g_wait_ns{kDefaultWaitNs};
}  // namespace

uint64_t foil_wait_limit_ns() { return g_wait_ns.load(std::memory_order_relaxed); }

extern "C" uint64_t foil_set_wait_limit_ns(uint64_t ns) {
    return g_wait_ns.exchange(ns ? ns : kDefaultWaitNs, std::memory_order_relaxed);
}

extern "C" const char* foil_last_error(void) { return g_last_error.c_str(); }
extern "C" uint64_t foil_launch_count(void) { return g_launches.load(); }
extern "C" const char* foil_version(void) { return "tt-foil-b200 1.0 (sm_100a, tcgen05)"; }

namespace {

using foil::FoilError;

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        throw FoilError(FOIL_ERR_CUDA, std::string("tt-foil: ") + what + ": " + cudaGetErrorString(e));
}

// Makes `device` current for the scope and restores the caller's device.
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int32_t device) {
        cuda_check(cudaGetDevice(&prev), "cudaGetDevice");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
    }
    ~DeviceScope() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// ------------------------------------------------ driver VMM entry points ---
struct Vmm {
    PFN_cuMemAddressReserve reserve = nullptr;
    PFN_cuMemAddressFree addr_free = nullptr;
    PFN_cuMemCreate create = nullptr;
    PFN_cuMemRelease release = nullptr;
    PFN_cuMemMap map = nullptr;
    PFN_cuMemUnmap unmap = nullptr;
    PFN_cuMemSetAccess set_access = nullptr;
    PFN_cuMemGetAllocationGranularity granularity = nullptr;
};

const Vmm& vmm() {
    static Vmm v;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* name, void** fn) {
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) != cudaSuccess ||
                q != cudaDriverEntryPointSuccess)
                *fn = nullptr;
        };
        get("cuMemAddressReserve", (void**)&v.reserve);
        get("cuMemAddressFree", (void**)&v.addr_free);
        get("cuMemCreate", (void**)&v.create);
        get("cuMemRelease", (void**)&v.release);
        get("cuMemMap", (void**)&v.map);
        get("cuMemUnmap", (void**)&v.unmap);
        get("cuMemSetAccess", (void**)&v.set_access);
        get("cuMemGetAllocationGranularity", (void**)&v.granularity);
    });
    return v;
}

constexpr uint64_t kDramReserve = 64ull << 30;  // virtual range (= 36-bit limit)
constexpr uint64_t kDramChunkMin = 64ull << 20;  // physical growth step

// ----------------------------------------- per-device scratch error word ---
std::mutex g_err_mu;
uint32_t* g_err_words[64] = {};

uint32_t* error_word_for_current_device() {
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= 64) throw FoilError(FOIL_ERR_INVALID, "tt-foil: device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (!g_err_words[dev]) {
        void* p = nullptr;
        cuda_check(cudaMalloc(&p, 256), "cudaMalloc(error word)");
        cuda_check(cudaMemset(p, 0, 256), "cudaMemset(error word)");
        g_err_words[dev] = static_cast<uint32_t*>(p);
    }
    return g_err_words[dev];
}

int sm_count_current() { return foil_sm_count(); }

template <class F>
int guarded(F&& f) {
    try {
        f();
        return FOIL_OK;
    } catch (const FoilError& e) {
        g_last_error = e.what();
        return e.status;
    } catch (const std::bad_alloc&) {
        g_last_error = "tt-foil: host out of memory";
        return FOIL_ERR_OOM;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return FOIL_ERR_INVALID;
    }
}

void throw_status(int st) {
    if (st != FOIL_OK) throw FoilError(st, g_last_error);
}

}  // namespace

// ====================================================================== ====
struct foil_device {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    std::mutex mu;
    bool closed = false;
    // DRAM arena
    CUdeviceptr dram_base = 0;
    uint64_t dram_mapped = 0;
    size_t granularity = 2u << 20;
    std::vector<std::pair<CUmemGenericAllocationHandle, uint64_t>> chunks;
    foil::BumpAllocator dram_alloc;
    // L1 arenas
    struct CoreArena {
        uint32_t x, y;
        char* base;
        foil::BumpAllocator alloc;
    };
    std::vector<CoreArena> cores;
    uint32_t* err_word = nullptr;

    CoreArena* core(uint32_t x, uint32_t y) {
        for (auto& c : cores)
            if (c.x == x && c.y == y) return &c;
        return nullptr;
    }
};

struct foil_kernel {
    foil_device* dev = nullptr;
    uint32_t core_x = 0, core_y = 0;
    foil::Program prog = foil::Program::TileCopy;
    std::array<bool, 5> present{};
    std::array<std::vector<uint32_t>, 5> rta;
    std::array<bool, 5> has_rta{};
    std::vector<foil::CbDesc> cbs;
    uint64_t cb_mask = 0;
};

namespace {


void release_device(foil_device* d) {
    if (d->closed) return;
    d->closed = true;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(d->ordinal);
    if (d->stream) cudaStreamSynchronize(d->stream);
    const Vmm& v = vmm();
    if (d->dram_base) {
        uint64_t off = 0;
        for (auto& ch : d->chunks) {
            if (v.unmap) v.unmap(d->dram_base + off, ch.second);
            if (v.release) v.release(ch.first);
            off += ch.second;
        }
        d->chunks.clear();
        if (v.addr_free) v.addr_free(d->dram_base, kDramReserve);
        d->dram_base = 0;
    }
    for (auto& c : d->cores)
        if (c.base) cudaFree(c.base);
    d->cores.clear();
    if (d->err_word) cudaFree(d->err_word);
    d->err_word = nullptr;
    if (d->done) cudaEventDestroy(d->done);
    if (d->stream) cudaStreamDestroy(d->stream);
    d->done = nullptr;
    d->stream = nullptr;
    if (prev >= 0) cudaSetDevice(prev);
}

// Back the DRAM arena with physical memory up to `needed` bytes.
void grow_dram(foil_device* d, uint64_t needed) {
    if (needed <= d->dram_mapped) return;
    const Vmm& v = vmm();
    uint64_t want = needed - d->dram_mapped;
    if (want < kDramChunkMin) want = kDramChunkMin;
    want = (want + d->granularity - 1) / d->granularity * d->granularity;
    if (d->dram_mapped + want > kDramReserve) want = kDramReserve - d->dram_mapped;
    CUmemAllocationProp prop = {};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = d->ordinal;
    CUmemGenericAllocationHandle h;
    if (v.create(&h, want, &prop, 0) != CUDA_SUCCESS)
        throw FoilError(FOIL_ERR_OOM, "tt-foil: DRAM out of memory (cuMemCreate failed)");
    if (v.map(d->dram_base + d->dram_mapped, want, 0, h, 0) != CUDA_SUCCESS) {
        v.release(h);
        throw FoilError(FOIL_ERR_CUDA, "tt-foil: cuMemMap failed");
    }
    CUmemAccessDesc acc = {};
    acc.location = prop.location;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    if (v.set_access(d->dram_base + d->dram_mapped, want, &acc, 1) != CUDA_SUCCESS) {
        v.unmap(d->dram_base + d->dram_mapped, want);
        v.release(h);
        throw FoilError(FOIL_ERR_CUDA, "tt-foil: cuMemSetAccess failed");
    }
    d->chunks.emplace_back(h, want);
    d->dram_mapped += want;
}

// Device pointer of a buffer-shaped region; checks it lies in allocated
// memory of the right arena.
char* region_ptr(foil_device* d, bool dram, uint32_t x, uint32_t y, uint64_t off, uint64_t bytes,
                 const char* what) {
    if (dram) {
        if (off > d->dram_alloc.current || bytes > d->dram_alloc.current - off)
            throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + what +
                                                  ": DRAM range outside allocated DRAM");
        return reinterpret_cast<char*>(d->dram_base) + off;
    }
    auto* c = d->core(x, y);
    if (!c)
        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + what + ": core (" +
                                              std::to_string(x) + "," + std::to_string(y) +
                                              ") was not opened");
    if (off < foil::kL1Base || off > c->alloc.current || bytes > c->alloc.current - off)
        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + what + ": L1 range outside allocated L1 of core (" +
                                              std::to_string(x) + "," + std::to_string(y) + ")");
    return c->base + off;
}

char* loc_ptr(foil_device* d, const foil::Loc& l, const char* what) {
    return region_ptr(d, l.dram, l.core_x, l.core_y, l.offset, l.bytes, what);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Element-wise stages (tile_copy / relu / add_tiles / bias_add) on the bulk
// streaming pipeline.  `out` may equal an input (in place) but must not
// partially overlap one: chunks are processed in no fixed order.  err: the
// device error word (null: this device's scratch word).
void launch_eltwise(const char* what, foil::stream::Op op, const void* a, const void* b, void* out,
                    uint64_t bytes, const uint16_t* bias_tiles, uint32_t Nt, uint32_t* err,
                    cudaStream_t stream) {
    if (bytes == 0) return;
    if (bytes % (op == foil::stream::kBias ? 2048 : 16))
        throw FoilError(FOIL_ERR_INVALID, std::string(what) + ": size is not a whole number of vectors / tiles");
    auto overlaps = [&](const void* in, uint64_t in_bytes) {
        if (!in || in == out) return false;
        const uintptr_t i0 = (uintptr_t)in, o0 = (uintptr_t)out;
        return i0 < o0 + bytes && o0 < i0 + in_bytes;
    };
    if (!a || !out || !aligned16(a) || !aligned16(out) || (op == foil::stream::kAdd && (!b || !aligned16(b))) ||
        (op == foil::stream::kBias && (!bias_tiles || !aligned16(bias_tiles))))
        throw FoilError(FOIL_ERR_INVALID, std::string(what) + ": null or misaligned pointer");
    if (overlaps(a, bytes) || (op == foil::stream::kAdd && overlaps(b, bytes)))
        throw FoilError(FOIL_ERR_INVALID, std::string(what) + ": output partially overlaps an input");
    if (op == foil::stream::kBias && (bias_tiles == out || overlaps(bias_tiles, (uint64_t)Nt * 2048)))
        throw FoilError(FOIL_ERR_INVALID, std::string(what) + ": output overlaps the bias band");
    if (!err) err = error_word_for_current_device();
    const int e = foil::stream::launch(op, a, b, out, bytes, bias_tiles, Nt, err, stream);
    if (e != 0)
        throw FoilError(FOIL_ERR_CUDA, std::string(what) + ": CUDA launch failed: " +
                                           cudaGetErrorString(static_cast<cudaError_t>(e)));
    foil_count_launch();
}

// Wait for the device stream with a deadline; throws on timeout.
void wait_stream(foil_device* d, std::chrono::steady_clock::time_point deadline,
                 uint32_t core_x, uint32_t core_y) {
    cuda_check(cudaEventRecord(d->done, d->stream), "cudaEventRecord");
    int spins = 0;
    while (true) {
        cudaError_t q = cudaEventQuery(d->done);
        if (q == cudaSuccess) return;
        if (q != cudaErrorNotReady) cuda_check(q, "kernel execution");
        if (std::chrono::steady_clock::now() > deadline)
            throw FoilError(FOIL_ERR_TIMEOUT,
                            "tt-foil: timeout waiting for kernel completion on core (" +
                                std::to_string(core_x) + "," + std::to_string(core_y) + ")");
        if (++spins > 2000) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

void check_error_word(foil_device* d) {
    uint32_t w = 0;
    cuda_check(cudaMemcpyAsync(&w, d->err_word, 4, cudaMemcpyDeviceToHost, d->stream), "read error word");
    cuda_check(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
    if (w != 0) {
        cudaMemsetAsync(d->err_word, 0, 4, d->stream);
        cudaStreamSynchronize(d->stream);
        throw FoilError(FOIL_ERR_DEVICE, "tt-foil: a kernel reported device error 0x" +
                                             [&] { std::ostringstream s; s << std::hex << w; return s.str(); }() +
                                             " (bounded wait expired)");
    }
}

}  // namespace

// ============================================================ C-ABI ======

extern "C" int foil_open_device(int idx, const char* /*firmware_dir*/, const foil_core* cores,
                                size_t num_cores, foil_device** out) {
    return guarded([&] {
        if (!out) throw FoilError(FOIL_ERR_INVALID, "tt-foil: null output pointer");
        *out = nullptr;
        if (num_cores == 0 || !cores)
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: device_open requires at least one Tensix core to boot");
        int count = 0;
        cuda_check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        if (idx < 0 || idx >= count)
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: no CUDA device with index " + std::to_string(idx));
        for (size_t i = 0; i < num_cores; ++i) {
            if (cores[i].x >= foil::kDramNode || cores[i].y >= foil::kDramNode)
                throw FoilError(FOIL_ERR_INVALID, "tt-foil: core coordinate out of range");
            for (size_t j = 0; j < i; ++j)
                if (cores[j].x == cores[i].x && cores[j].y == cores[i].y)
                    throw FoilError(FOIL_ERR_INVALID, "tt-foil: core listed twice in open_device");
        }
        const Vmm& v = vmm();
        if (!v.reserve || !v.create || !v.map || !v.set_access)
            throw FoilError(FOIL_ERR_CUDA, "tt-foil: CUDA virtual-memory entry points unavailable");
        auto d = std::make_unique<foil_device>();
        d->ordinal = idx;
        DeviceScope scope(idx);
        cuda_check(cudaFree(nullptr), "CUDA context init");
        try {
            cuda_check(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "cudaStreamCreate");
            cuda_check(cudaEventCreateWithFlags(&d->done, cudaEventDisableTiming), "cudaEventCreate");
            CUmemAllocationProp prop = {};
            prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
            prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
            prop.location.id = idx;
            size_t gran = 0;
            if (v.granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) == CUDA_SUCCESS && gran)
                d->granularity = gran;
            if (v.reserve(&d->dram_base, kDramReserve, 0, 0, 0) != CUDA_SUCCESS)
                throw FoilError(FOIL_ERR_CUDA, "tt-foil: cuMemAddressReserve failed");
            d->dram_alloc = foil::BumpAllocator{0, 0, foil::kDramLimit};
            for (size_t i = 0; i < num_cores; ++i) {
                void* p = nullptr;
                cuda_check(cudaMalloc(&p, foil::kL1Size), "cudaMalloc(L1 arena)");
                foil_device::CoreArena ca{cores[i].x, cores[i].y, static_cast<char*>(p),
                                          foil::BumpAllocator{foil::kL1Base, foil::kL1Base, foil::kL1End}};
                d->cores.push_back(ca);
                cuda_check(cudaMemsetAsync(p, 0, foil::kL1Size, d->stream), "cudaMemset(L1 arena)");
            }
            void* e = nullptr;
            cuda_check(cudaMalloc(&e, 256), "cudaMalloc(error word)");
            d->err_word = static_cast<uint32_t*>(e);
            cuda_check(cudaMemsetAsync(e, 0, 256, d->stream), "cudaMemset(error word)");
            cuda_check(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
        } catch (...) {
            release_device(d.get());
            throw;
        }
        *out = d.release();
    });
}

extern "C" int foil_close_device(foil_device* d) {
    return guarded([&] {
        if (!d) return;
        release_device(d);
        delete d;
    });
}

extern "C" int foil_allocate_buffer(foil_device* d, int32_t loc, uint64_t size, foil_core core,
                                    foil_buffer* out) {
    return guarded([&] {
        if (!d || !out || d->closed) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device");
        std::lock_guard<std::mutex> lk(d->mu);
        if (size == 0) throw FoilError(FOIL_ERR_INVALID, "tt-foil: buffer size must be > 0");
        foil_buffer b = {};
        b.location = loc;
        b.size_bytes = size;
        b.core = core;
        if (loc == FOIL_LOC_L1) {
            auto* c = d->core(core.x, core.y);
            if (!c)
                throw FoilError(FOIL_ERR_INVALID, "tt-foil: L1 allocation on core (" + std::to_string(core.x) +
                                                      "," + std::to_string(core.y) + ") which was not opened");
            b.device_addr = c->alloc.alloc(size, foil::kL1Align, "L1");
        } else if (loc == FOIL_LOC_DRAM) {
            const uint64_t saved = d->dram_alloc.current;
            b.device_addr = d->dram_alloc.alloc(size, foil::kDramAlign, "DRAM");
            DeviceScope scope(d->ordinal);
            try {
                grow_dram(d, d->dram_alloc.current);
            } catch (...) {
                d->dram_alloc.current = saved;
                throw;
            }
        } else {
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: unknown buffer location");
        }
        *out = b;
    });
}

extern "C" int foil_free_buffer(foil_device*, const foil_buffer*) { return FOIL_OK; }

static char* buffer_ptr(foil_device* d, const foil_buffer* b, uint64_t bytes, const char* what) {
    if (!d || !b || d->closed) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device or buffer");
    if (bytes > b->size_bytes)
        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + what + " size exceeds allocation");
    return region_ptr(d, b->location == FOIL_LOC_DRAM, b->core.x, b->core.y, b->device_addr,
                      b->size_bytes, what);
}

extern "C" int foil_write_buffer(foil_device* d, const foil_buffer* b, const void* src, uint64_t bytes) {
    return guarded([&] {
        if (!d || d->closed) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device");
        std::lock_guard<std::mutex> lk(d->mu);
        char* p = buffer_ptr(d, b, bytes, "write_buffer");
        if (bytes == 0) return;
        if (!src) throw FoilError(FOIL_ERR_INVALID, "tt-foil: write_buffer from null pointer");
        DeviceScope scope(d->ordinal);
        cuda_check(cudaMemcpyAsync(p, src, bytes, cudaMemcpyHostToDevice, d->stream), "cudaMemcpy H2D");
        cuda_check(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
    });
}

extern "C" int foil_read_buffer(foil_device* d, const foil_buffer* b, void* dst, uint64_t bytes) {
    return guarded([&] {
        if (!d || d->closed) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device");
        std::lock_guard<std::mutex> lk(d->mu);
        char* p = buffer_ptr(d, b, bytes, "read_buffer");
        if (bytes == 0) return;
        if (!dst) throw FoilError(FOIL_ERR_INVALID, "tt-foil: read_buffer into null pointer");
        DeviceScope scope(d->ordinal);
        cuda_check(cudaMemcpyAsync(dst, p, bytes, cudaMemcpyDeviceToHost, d->stream), "cudaMemcpy D2H");
        cuda_check(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize");
    });
}

extern "C" int foil_buffer_device_ptr(foil_device* d, const foil_buffer* b, void** out) {
    return guarded([&] {
        if (!out) throw FoilError(FOIL_ERR_INVALID, "tt-foil: null output pointer");
        *out = buffer_ptr(d, b, 0, "buffer_device_ptr");
    });
}

extern "C" int foil_load_kernel(foil_device* d, const foil_risc_binary* bins, size_t n,
                                foil_core core, foil_kernel** out) {
    return guarded([&] {
        if (!d || !out || d->closed) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device");
        *out = nullptr;
        if (n == 0 || !bins) throw FoilError(FOIL_ERR_INVALID, "tt-foil: no binaries provided to load_kernel");
        if (!d->core(core.x, core.y))
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: load_kernel on core (" + std::to_string(core.x) + "," +
                                                  std::to_string(core.y) + ") which was not opened");
        auto k = std::make_unique<foil_kernel>();
        k->dev = d;
        k->core_x = core.x;
        k->core_y = core.y;
        std::vector<foil::Descriptor> ds;
        for (size_t i = 0; i < n; ++i) {
            const std::string path = bins[i].elf_path ? bins[i].elf_path : "";
            std::ifstream f(path, std::ios::binary);
            if (!f) throw FoilError(FOIL_ERR_NOT_FOUND, "tt-foil: ELF not found: " + path);
            std::stringstream ss;
            ss << f.rdbuf();
            foil::Descriptor desc = foil::parse_descriptor(ss.str(), path);
            int risc = bins[i].risc;
            if (foil::role_of_risc(risc) != foil::parse_role(desc.role))
                throw FoilError(FOIL_ERR_INVALID, "tt-foil: " + path + " has role '" + desc.role +
                                                      "' which does not match its RISC");
            k->present[risc] = true;
            ds.push_back(desc);
        }
        k->prog = foil::resolve_program(ds);
        *out = k.release();
    });
}

extern "C" int foil_release_kernel(foil_kernel* k) {
    delete k;
    return FOIL_OK;
}

extern "C" int foil_set_runtime_args(foil_device*, foil_kernel* k, int32_t risc, const uint32_t* args,
                                     size_t n) {
    return guarded([&] {
        if (!k) throw FoilError(FOIL_ERR_INVALID, "tt-foil: null kernel");
        if (risc < 0 || risc > 4 || !k->present[risc])
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: set_runtime_args called for a RISC not in this kernel");
        if (n > foil::kMaxRtaWords)
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: too many runtime args (max " +
                                                  std::to_string(foil::kMaxRtaWords) + ")");
        k->rta[risc].assign(args, args + n);
        k->has_rta[risc] = true;
    });
}

extern "C" int foil_register_cbs(foil_device*, foil_kernel* k, const foil_cb_config* cbs, size_t n) {
    return guarded([&] {
        if (!k) throw FoilError(FOIL_ERR_INVALID, "tt-foil: null kernel");
        std::vector<foil::CbDesc> v;
        for (size_t i = 0; i < n; ++i)
            v.push_back({cbs[i].cb_index, cbs[i].fifo_addr, cbs[i].fifo_size, cbs[i].num_pages,
                         cbs[i].page_size});
        uint64_t mask = foil::validate_cbs(v);
        k->cbs = v;
        k->cb_mask = mask;
    });
}

extern "C" int foil_make_noc_unicast_addr(foil_device* d, foil_core dst, uint64_t off, uint64_t* out) {
    return guarded([&] {
        if (!d || !out) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device");
        if (!d->core(dst.x, dst.y))
            throw FoilError(FOIL_ERR_INVALID, "tt-foil: make_noc_unicast_addr to core that was not opened");
        *out = foil::pack_addr(dst.x, dst.y, off);
    });
}

extern "C" int foil_make_noc_dram_addr(foil_device* d, uint64_t off, uint64_t* out) {
    return guarded([&] {
        if (!d || !out) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device");
        if (off >= foil::kDramLimit) throw FoilError(FOIL_ERR_INVALID, "tt-foil: DRAM offset too large");
        *out = foil::pack_addr(foil::kDramNode, foil::kDramNode, off);
    });
}

namespace {

struct ResolvedOp {
    foil::PlanOp op;
    const foil_kernel* k;
    char *p0 = nullptr, *p1 = nullptr, *po = nullptr;
    char *flag_src = nullptr, *flag_dst = nullptr, *gate = nullptr;
};

void run_op(foil_device* d, ResolvedOp& r) {
    cudaStream_t s = d->stream;
    switch (r.op.kind) {
        case foil::OpKind::Copy:
            launch_eltwise("tile_copy", foil::stream::kCopy, r.p0, nullptr, r.po, r.op.in0.bytes, nullptr, 0,
                           d->err_word, s);
            break;
        case foil::OpKind::Relu:
            launch_eltwise("relu", foil::stream::kRelu, r.p0, nullptr, r.po, r.op.in0.bytes, nullptr, 0,
                           d->err_word, s);
            break;
        case foil::OpKind::Add:
            launch_eltwise("add_tiles", foil::stream::kAdd, r.p0, r.p1, r.po, r.op.in0.bytes, nullptr, 0,
                           d->err_word, s);
            break;
        case foil::OpKind::BiasAdd:
            launch_eltwise("bias_add", foil::stream::kBias, r.p0, nullptr, r.po, 2048, (const uint16_t*)r.p1, 1,
                           d->err_word, s);
            break;
        case foil::OpKind::Matmul:
            throw_status(foil::gemm::launch((const uint16_t*)r.p0, (const uint16_t*)r.p1, (uint16_t*)r.po,
                                            r.op.Mt, r.op.Kt, r.op.Nt, nullptr, 0, d->err_word, s,
                                            sm_count_current()));
            break;
        case foil::OpKind::McastForward:
        case foil::OpKind::Word:
        case foil::OpKind::Send:
            break;  // run by the multi-core launch
    }
}

}  // namespace

extern "C" int foil_execute(foil_device* d, foil_kernel* const* kernels, size_t n, int32_t timeout_ms) {
    return guarded([&] {
        if (!d || d->closed) throw FoilError(FOIL_ERR_INVALID, "tt-foil: invalid device");
        if (n == 0 || !kernels) throw FoilError(FOIL_ERR_INVALID, "tt-foil: dispatch_execute_multi: no kernels");
        std::lock_guard<std::mutex> lk(d->mu);
        DeviceScope scope(d->ordinal);
        const auto deadline = std::chrono::steady_clock::now() +
                              std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 5000);
        // 1. Plan and resolve every operand before launching anything.
        std::vector<ResolvedOp> ops;
        for (size_t i = 0; i < n; ++i) {
            const foil_kernel* k = kernels[i];
            if (!k || k->dev != d) throw FoilError(FOIL_ERR_INVALID, "tt-foil: kernel belongs to another device");
            for (auto& op : foil::plan_program(k->prog, k->core_x, k->core_y, k->rta, k->has_rta)) {
                ResolvedOp r;
                r.op = op;
                r.k = k;
                const char* what = foil::program_name(k->prog);
                switch (op.kind) {
                    case foil::OpKind::Copy:
                    case foil::OpKind::Relu:
                        r.p0 = loc_ptr(d, op.in0, what);
                        r.po = loc_ptr(d, op.out, what);
                        break;
                    case foil::OpKind::Add:
                    case foil::OpKind::BiasAdd:
                    case foil::OpKind::Matmul:
                        r.p0 = loc_ptr(d, op.in0, what);
                        r.p1 = loc_ptr(d, op.in1, what);
                        r.po = loc_ptr(d, op.out, what);
                        break;
                    case foil::OpKind::McastForward:
                        r.p0 = loc_ptr(d, op.in0, what);
                        r.p1 = loc_ptr(d, op.in1, what);
                        r.po = loc_ptr(d, op.out, what);
                        r.flag_src = loc_ptr(d, op.flag_src, what);
                        r.flag_dst = loc_ptr(d, op.flag_dst, what);
                        break;
                    case foil::OpKind::Word:
                        if (op.word != foil::WordOp::Set) r.p0 = loc_ptr(d, op.in0, what);
                        if (op.word == foil::WordOp::Add || op.word == foil::WordOp::Mul)
                            r.p1 = loc_ptr(d, op.in1, what);
                        r.po = loc_ptr(d, op.out, what);
                        break;
                    case foil::OpKind::Send:
                        r.p0 = loc_ptr(d, op.in0, what);
                        r.po = loc_ptr(d, op.out, what);
                        r.flag_src = loc_ptr(d, op.flag_src, what);
                        r.flag_dst = loc_ptr(d, op.flag_dst, what);
                        break;
                }
                if (op.gated) r.gate = loc_ptr(d, op.gate_flag, what);
                const bool scalar = op.kind == foil::OpKind::Word || op.kind == foil::OpKind::Send;
                for (char* p : {r.p0, r.p1, r.po})
                    if (p && (scalar ? (reinterpret_cast<uintptr_t>(p) & 3u) != 0 : !aligned16(p)))
                        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + what +
                                                              (scalar ? ": word operands must be 4-byte aligned"
                                                                      : ": tile operands must be 16-byte aligned"));
                for (char* p : {r.flag_src, r.flag_dst, r.gate})
                    if (p && (reinterpret_cast<uintptr_t>(p) & 3u) != 0)
                        throw FoilError(FOIL_ERR_INVALID, std::string("tt-foil: ") + what +
                                                              ": flag words must be 4-byte aligned");
                ops.push_back(r);
            }
        }
        // 2. Programs that talk to each other (the mcast producer forwards B
        //    and sets the consumer's ready flag; the consumer waits for it,
        //    reader_consumer.cpp:40-44; likewise noc_passthrough) and the
        //    scalar add_two_numbers kernels run as ONE cluster launch, one
        //    CTA per core, so they are resident together and a consumer's
        //    bounded device-side wait sees its producer's flag.  The other
        //    programs of the execute follow in stream order.
        bool interacting = false;
        for (auto& r : ops)
            interacting |= r.gate != nullptr || r.op.kind == foil::OpKind::McastForward ||
                           r.op.kind == foil::OpKind::Word || r.op.kind == foil::OpKind::Send;
        if (interacting) {
            std::vector<foil::gemm::CoreProgram> cores;
            std::vector<const foil_kernel*> core_kernel;
            std::vector<bool> in_cluster(ops.size(), false);
            for (size_t i = 0; i < n; ++i) {
                foil::gemm::CoreProgram c = {};
                bool any = false, plain = true;
                for (size_t j = 0; j < ops.size(); ++j) {
                    if (ops[j].k != kernels[i]) continue;
                    const auto& r = ops[j];
                    if ((r.op.kind == foil::OpKind::McastForward || r.op.kind == foil::OpKind::Send) &&
                        !c.fwd_bytes) {
                        c.fwd_src = r.p0;
                        c.fwd_stage = r.op.kind == foil::OpKind::McastForward ? r.p1 : nullptr;
                        c.fwd_peer = r.po;
                        c.fwd_bytes = r.op.in0.bytes;
                        c.flag_src = reinterpret_cast<const uint32_t*>(r.flag_src);
                        c.flag_dst = reinterpret_cast<uint32_t*>(r.flag_dst);
                        any = true;
                    } else if (r.op.kind == foil::OpKind::Matmul && c.Mt == 0) {
                        c.a = reinterpret_cast<const uint16_t*>(r.p0);
                        c.b = reinterpret_cast<const uint16_t*>(r.p1);
                        c.c = reinterpret_cast<uint16_t*>(r.po);
                        c.Mt = r.op.Mt;
                        c.Kt = r.op.Kt;
                        c.Nt = r.op.Nt;
                    } else if (r.op.kind == foil::OpKind::Word && c.nwords < foil::gemm::kMaxWordSteps) {
                        foil::gemm::WordStep& w = c.words[c.nwords++];
                        w.a = reinterpret_cast<const uint32_t*>(r.p0);
                        w.b = reinterpret_cast<const uint32_t*>(r.p1);
                        w.out = reinterpret_cast<uint32_t*>(r.po);
                        w.imm = r.op.imm;
                        switch (r.op.word) {
                            case foil::WordOp::Add: w.code = foil::gemm::kWordAdd; break;
                            case foil::WordOp::Mul: w.code = foil::gemm::kWordMul; break;
                            case foil::WordOp::Set: w.code = foil::gemm::kWordSet; break;
                            case foil::WordOp::Scale: w.code = foil::gemm::kWordScale; break;
                        }
                        any = true;
                    } else {
                        plain = false;
                    }
                    if (r.gate) {
                        c.gate = reinterpret_cast<const uint32_t*>(r.gate);
                        c.gate_value = r.op.gate_value;
                    }
                }
                if (c.gate || any || (plain && c.Mt)) {
                    if (!plain)
                        throw FoilError(FOIL_ERR_UNSUPPORTED,
                                        "tt-foil: a core that waits, forwards or runs scalar steps runs at most "
                                        "one matmul and no tile programs");
                    for (size_t j = 0; j < ops.size(); ++j)
                        if (ops[j].k == kernels[i]) in_cluster[j] = true;
                    cores.push_back(c);
                    core_kernel.push_back(kernels[i]);
                }
            }
            if (cores.size() > foil::gemm::kMaxCores)
                throw FoilError(FOIL_ERR_UNSUPPORTED, "tt-foil: at most 8 cores that wait on each other per execute");
            uint32_t* status = d->err_word + 16;  // per-core gate status (bytes 64 .. 95 of the word block)
            cuda_check(cudaMemsetAsync(status, 0, 4 * foil::gemm::kMaxCores, d->stream), "clear core status");
            const auto left = std::chrono::duration_cast<std::chrono::nanoseconds>(
                deadline - std::chrono::steady_clock::now());
            const uint64_t gate_ns = left.count() > 0 ? (uint64_t)left.count() : 1u;
            throw_status(foil::gemm::launch_cores(cores.data(), (uint32_t)cores.size(), d->err_word, status, gate_ns,
                                                  d->stream));
            for (size_t j = 0; j < ops.size(); ++j)
                if (!in_cluster[j]) run_op(d, ops[j]);
            // The device-side gate wait ends by the deadline; allow the launch
            // a grace period beyond it before the host gives up.
            wait_stream(d, deadline + std::chrono::seconds(2), kernels[0]->core_x, kernels[0]->core_y);
            uint32_t st[foil::gemm::kMaxCores] = {};
            cuda_check(cudaMemcpy(st, status, sizeof st, cudaMemcpyDeviceToHost), "read core status");
            for (size_t i = 0; i < cores.size(); ++i)
                if (st[i]) {
                    cudaMemsetAsync(d->err_word, 0, 4, d->stream);
                    cudaStreamSynchronize(d->stream);
                    throw FoilError(FOIL_ERR_TIMEOUT, "tt-foil: timeout waiting for kernel completion on core (" +
                                                          std::to_string(core_kernel[i]->core_x) + "," +
                                                          std::to_string(core_kernel[i]->core_y) +
                                                          "): ready flag never set");
                }
            check_error_word(d);
            return;
        }
        // 3. Compute launches.
        for (auto& r : ops) run_op(d, r);
        // 4. Bounded wait, then the device error word.
        wait_stream(d, deadline, kernels[0]->core_x, kernels[0]->core_y);
        check_error_word(d);
    });
}

// --------------------------------------------- device-resident GEMM entry ---
extern "C" int foil_matmul_tiles_dev(const uint16_t* a, const uint16_t* b, uint16_t* c, uint32_t Mt,
                                     uint32_t Kt, uint32_t Nt, const uint16_t* bias, int32_t relu,
                                     void* stream) {
    return guarded([&] {
        if (Mt == 0 || Kt == 0 || Nt == 0) return;
        if (Mt > 65535 || Kt > 65535 || Nt > 65535)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_dev: tile counts must be <= 65535");
        if (!a || !b || !c || !aligned16(a) || !aligned16(b) || !aligned16(c) ||
            (bias && !aligned16(bias)))
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_dev: null or misaligned pointer");
        uint32_t* err = error_word_for_current_device();
        throw_status(foil::gemm::launch(a, b, c, Mt, Kt, Nt, bias, relu, err, (cudaStream_t)stream,
                                        sm_count_current()));
    });
}

// ---------------------------------- GEMM with its own all-gather (NVLink) ---
extern "C" int foil_matmul_tiles_gather_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                                            uint16_t* const* peer_c, uint32_t npeers, uint32_t Mt,
                                            uint32_t Kt, uint32_t Nt, const uint16_t* bias, int32_t relu,
                                            void* stream) {
    return guarded([&] {
        if (npeers > foil::gemm::kMaxPeers)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_dev: at most 7 peer copies");
        if (npeers && !peer_c)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_dev: null peer list");
        for (uint32_t i = 0; i < npeers; ++i)
            if (!peer_c[i] || !aligned16(peer_c[i]))
                throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_dev: null or misaligned peer buffer");
        if (Mt == 0 || Kt == 0 || Nt == 0) return;
        if (Mt > 65535 || Kt > 65535 || Nt > 65535)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_dev: tile counts must be <= 65535");
        if (!a || !b || !c || !aligned16(a) || !aligned16(b) || !aligned16(c) || (bias && !aligned16(bias)))
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_dev: null or misaligned pointer");
        uint32_t* err = error_word_for_current_device();
        throw_status(foil::gemm::launch(a, b, c, Mt, Kt, Nt, bias, relu, err, (cudaStream_t)stream,
                                        sm_count_current(), peer_c, npeers));
    });
}

// ------------------------------- GEMM whose tiles go out through multicast ---
extern "C" int foil_matmul_tiles_gather_mc_dev(const uint16_t* a, const uint16_t* b, uint16_t* c, uint16_t* mc_c,
                                               uint32_t Mt, uint32_t Kt, uint32_t Nt, const uint16_t* bias,
                                               int32_t relu, void* stream) {
    return guarded([&] {
        if (!mc_c || !aligned16(mc_c))
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_mc_dev: null or misaligned multicast address");
        if (Mt == 0 || Kt == 0 || Nt == 0) return;
        if (Mt > 65535 || Kt > 65535 || Nt > 65535)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_mc_dev: tile counts must be <= 65535");
        if (!a || !b || !c || !aligned16(a) || !aligned16(b) || !aligned16(c) || (bias && !aligned16(bias)))
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_mc_dev: null or misaligned pointer");
        uint32_t* err = error_word_for_current_device();
        throw_status(foil::gemm::launch(a, b, c, Mt, Kt, Nt, bias, relu, err, (cudaStream_t)stream,
                                        sm_count_current(), nullptr, 0, mc_c));
    });
}

// ------------------------ GEMM in row chunks, copy engines push to the peers ---
// Per device: one copy stream per peer and the events that order each copy
// after the GEMM launch of its chunk (reused under the device's lock).
namespace {

struct CopyPipe {
    std::mutex mu;
    int device = -1;
    cudaStream_t copy[foil::gemm::kMaxPeers] = {};
    cudaEvent_t done[foil::gemm::kMaxPeers] = {};
    std::vector<cudaEvent_t> chunk_ev;
};

CopyPipe& copy_pipe(int device) {
    static std::mutex mu;
    static std::vector<std::unique_ptr<CopyPipe>> pipes;
    std::lock_guard<std::mutex> lk(mu);
    for (auto& p : pipes)
        if (p->device == device) return *p;
    auto p = std::make_unique<CopyPipe>();
    p->device = device;
    for (uint32_t i = 0; i < foil::gemm::kMaxPeers; ++i) {
        cuda_check(cudaStreamCreateWithFlags(&p->copy[i], cudaStreamNonBlocking), "cudaStreamCreate(copy)");
        cuda_check(cudaEventCreateWithFlags(&p->done[i], cudaEventDisableTiming), "cudaEventCreate");
    }
    pipes.push_back(std::move(p));
    return *pipes.back();
}

}  // namespace

extern "C" int foil_matmul_tiles_gather_ce_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                                               uint16_t* const* peer_c, uint32_t npeers, uint32_t Mt,
                                               uint32_t Kt, uint32_t Nt, const uint16_t* bias, int32_t relu,
                                               uint32_t chunks, void* stream) {
    return guarded([&] {
        if (npeers > foil::gemm::kMaxPeers)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_ce_dev: at most 7 peer copies");
        if (npeers && !peer_c)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_ce_dev: null peer list");
        for (uint32_t i = 0; i < npeers; ++i)
            if (!peer_c[i] || !aligned16(peer_c[i]))
                throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_ce_dev: null or misaligned peer buffer");
        if (chunks == 0 || chunks > 64)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_ce_dev: chunks must be in 1..64");
        if (Mt == 0 || Kt == 0 || Nt == 0) return;
        if (Mt > 65535 || Kt > 65535 || Nt > 65535)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_ce_dev: tile counts must be <= 65535");
        if (!a || !b || !c || !aligned16(a) || !aligned16(b) || !aligned16(c) || (bias && !aligned16(bias)))
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_gather_ce_dev: null or misaligned pointer");
        int dev = 0;
        cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
        uint32_t* err = error_word_for_current_device();
        cudaStream_t s = (cudaStream_t)stream;
        // Chunks of whole 256-row pair tiles (8 tile rows), the last one shorter.
        uint32_t per = (Mt + chunks - 1) / chunks;
        per = (per + 7u) / 8u * 8u;
        CopyPipe& cp = copy_pipe(dev);
        std::lock_guard<std::mutex> lk(cp.mu);
        const uint32_t nchunks = (Mt + per - 1) / per;
        while (cp.chunk_ev.size() < nchunks) {
            cudaEvent_t e;
            cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
            cp.chunk_ev.push_back(e);
        }
        // The copy streams start after everything already queued on `s`
        // (earlier readers of the peers' buffers are ordered by the caller's
        // collective on `s`).
        for (uint32_t d = 0; d < npeers; ++d) {
            cuda_check(cudaEventRecord(cp.done[d], s), "cudaEventRecord");
            cuda_check(cudaStreamWaitEvent(cp.copy[d], cp.done[d], 0), "cudaStreamWaitEvent");
        }
        const int sms = sm_count_current();
        for (uint32_t k = 0; k < nchunks; ++k) {
            const uint32_t m0 = k * per, mt = std::min(per, Mt - m0);
            const uint64_t c_off = (uint64_t)m0 * Nt * 1024u, a_off = (uint64_t)m0 * Kt * 1024u;
            throw_status(foil::gemm::launch(a + a_off, b, c + c_off, mt, Kt, Nt, bias, relu, err, s, sms));
            if (npeers == 0) continue;
            cuda_check(cudaEventRecord(cp.chunk_ev[k], s), "cudaEventRecord");
            for (uint32_t d = 0; d < npeers; ++d) {
                cuda_check(cudaStreamWaitEvent(cp.copy[d], cp.chunk_ev[k], 0), "cudaStreamWaitEvent");
                cuda_check(cudaMemcpyAsync(peer_c[d] + c_off, c + c_off, (uint64_t)mt * Nt * 2048u,
                                           cudaMemcpyDeviceToDevice, cp.copy[d]),
                           "cudaMemcpyAsync(peer chunk)");
            }
        }
        // `s` continues after every chunk has reached every peer.
        for (uint32_t d = 0; d < npeers; ++d) {
            cuda_check(cudaEventRecord(cp.done[d], cp.copy[d]), "cudaEventRecord");
            cuda_check(cudaStreamWaitEvent(s, cp.done[d], 0), "cudaStreamWaitEvent");
        }
    });
}

// Inter-process device buffers: allocated here, exported as a 64-byte handle,
// opened by the other processes of the node as peer-mapped pointers.
static_assert(sizeof(cudaIpcMemHandle_t) == FOIL_PEER_HANDLE_BYTES, "IPC handle size");


extern "C" int foil_peer_alloc(int32_t device, uint64_t bytes, void** ptr, uint8_t* handle) {
    return guarded([&] {
        if (!ptr || !handle || bytes == 0) throw FoilError(FOIL_ERR_INVALID, "foil_peer_alloc: bad arguments");
        DeviceScope scope(device);
        void* p = nullptr;
        cuda_check(cudaMalloc(&p, bytes), "cudaMalloc(peer buffer)");
        cudaIpcMemHandle_t h;
        const cudaError_t e = cudaIpcGetMemHandle(&h, p);
        if (e != cudaSuccess) {
            cudaFree(p);
            cuda_check(e, "cudaIpcGetMemHandle");
        }
        std::memcpy(handle, &h, sizeof h);
        *ptr = p;
    });
}

extern "C" int foil_peer_open(int32_t device, const uint8_t* handle, void** ptr) {
    return guarded([&] {
        if (!ptr || !handle) throw FoilError(FOIL_ERR_INVALID, "foil_peer_open: bad arguments");
        DeviceScope scope(device);
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle, sizeof h);
        void* p = nullptr;
        cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        *ptr = p;
    });
}

extern "C" int foil_peer_close(int32_t device, void* ptr) {
    return guarded([&] {
        if (!ptr) return;
        DeviceScope scope(device);
        cuda_check(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
    });
}

extern "C" int foil_peer_free(int32_t device, void* ptr) {
    return guarded([&] {
        if (!ptr) return;
        DeviceScope scope(device);
        cuda_check(cudaFree(ptr), "cudaFree(peer buffer)");
    });
}

extern "C" int foil_conv2d_nhwc_dev(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                                    uint16_t* y, uint32_t N, uint32_t H, uint32_t W, uint32_t Cin,
                                    uint32_t Cout, uint32_t KH, uint32_t KW, uint32_t stride,
                                    uint32_t pad, int32_t relu, void* stream) {
    return guarded([&] {
        if (N == 0 || Cout == 0) return;
        if (Cin == 0 || Cin % 16 || Cout % 16)
            throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_nhwc_dev: Cin and Cout must be non-zero multiples of 16");
        if (H == 0 || W == 0 || KH == 0 || KW == 0 || stride == 0 || KH > 16 || KW > 16 || stride > 16 ||
            pad >= KH || pad >= KW || H + 2 * pad < KH || W + 2 * pad < KW)
            throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_nhwc_dev: unsupported kernel / stride / padding");
        const uint64_t Ho = (H + 2 * pad - KH) / stride + 1, Wo = (W + 2 * pad - KW) / stride + 1;
        if ((uint64_t)N * H * W * Cin >= (1ull << 40) || (uint64_t)N * Ho * Wo >= (1ull << 31) ||
            (uint64_t)N * H * W >= (1ull << 32))
            throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_nhwc_dev: tensor too large");
        if (!x || !w || !y || !aligned16(x) || !aligned16(w) || !aligned16(y) || (bias && !aligned16(bias)))
            throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_nhwc_dev: null or misaligned pointer");
        uint32_t* err = error_word_for_current_device();
        throw_status(foil::conv::launch(x, w, bias, y, N, H, W, Cin, Cout, KH, KW, stride, pad, relu, err,
                                        (cudaStream_t)stream, sm_count_current()));
    });
}

// ----------------------------------- conv in the reference's convention ---
extern "C" int foil_conv2d_chw_dev(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                                   uint32_t N, uint32_t Cin, uint32_t H, uint32_t W, uint32_t Cout, uint32_t KH,
                                   uint32_t KW, uint32_t stride, uint32_t pad, int32_t relu, void* stream) {
    return guarded([&] {
        if (N == 0 || Cout == 0) return;
        if (Cin == 0 || H == 0 || W == 0 || KH == 0 || KW == 0 || stride == 0 || KH > 16 || KW > 16 ||
            stride > 16 || pad >= KH || pad >= KW || H + 2 * pad < KH || W + 2 * pad < KW)
            throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_chw_dev: unsupported kernel / stride / padding");
        if (!x || !w || !y) throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_chw_dev: null pointer");
        const uint64_t Ho = (H + 2 * pad - KH) / stride + 1, Wo = (W + 2 * pad - KW) / stride + 1;
        const uint32_t cin_p = (Cin + 15u) / 16u * 16u, cout_p = (Cout + 15u) / 16u * 16u;
        const uint64_t hw = (uint64_t)H * W, howo = Ho * Wo, k = (uint64_t)KH * KW;
        if (N > 65535 || Cout > 65535 || hw >= (1ull << 31) || (uint64_t)N * hw * cin_p >= (1ull << 40) ||
            (uint64_t)N * howo >= (1ull << 31))
            throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_chw_dev: tensor too large");
        auto up = [](uint64_t b) { return (b + 255u) / 256u * 256u; };
        const uint64_t bx = up((uint64_t)N * hw * cin_p * 2), bw = up((uint64_t)cout_p * k * cin_p * 2),
                       bb = up((uint64_t)cout_p * 2), by = up((uint64_t)N * howo * cout_p * 2);
        cudaStream_t s = (cudaStream_t)stream;
        char* ws = nullptr;
        if (cudaMallocAsync((void**)&ws, bx + bw + bb + by, s) != cudaSuccess) {
            cudaGetLastError();
            throw FoilError(FOIL_ERR_OOM, "foil_conv2d_chw_dev: out of device memory for the re-laid operands");
        }
        struct Free {
            char* p;
            cudaStream_t s;
            ~Free() { cudaFreeAsync(p, s); }
        } release{ws, s};
        uint16_t* xn = reinterpret_cast<uint16_t*>(ws);
        uint16_t* wn = reinterpret_cast<uint16_t*>(ws + bx);
        uint16_t* bn = reinterpret_cast<uint16_t*>(ws + bx + bw);
        uint16_t* yn = reinterpret_cast<uint16_t*>(ws + bx + bw + bb);
        // x (N, Cin, H W) -> (N, H W, Cin_p); w (Cout, Cin, KH KW) -> (Cout_p, KH KW, Cin_p);
        // zero-padded channels contribute nothing.
        throw_status(foil::transpose_u16(x, xn, N, Cin, (uint32_t)hw, N, (uint32_t)hw, cin_p, s));
        throw_status(foil::transpose_u16(w, wn, Cout, Cin, (uint32_t)k, cout_p, (uint32_t)k, cin_p, s));
        if (bias) {
            cuda_check(cudaMemsetAsync(bn, 0, (size_t)cout_p * 2, s), "clear bias");
            cuda_check(cudaMemcpyAsync(bn, bias, (size_t)Cout * 2, cudaMemcpyDeviceToDevice, s), "copy bias");
        }
        uint32_t* err = error_word_for_current_device();
        throw_status(foil::conv::launch(xn, wn, bias ? bn : nullptr, yn, N, H, W, cin_p, cout_p, KH, KW, stride,
                                        pad, relu, err, s, sm_count_current()));
        // y (N, Ho Wo, Cout_p) -> (N, Cout, Ho Wo)
        throw_status(foil::transpose_u16(yn, y, N, (uint32_t)howo, cout_p, N, Cout, (uint32_t)howo, s));
    });
}

// ------------------------------------------------ element-wise entries ---
extern "C" int foil_tile_copy_dev(const void* src, void* dst, uint64_t bytes, void* stream) {
    return guarded([&] {
        if (bytes % 16) throw FoilError(FOIL_ERR_INVALID, "foil_tile_copy_dev: bytes must be a multiple of 16");
        if (bytes == 0) return;
        launch_eltwise("foil_tile_copy_dev", foil::stream::kCopy, src, nullptr, dst, bytes, nullptr, 0,
                       nullptr, (cudaStream_t)stream);
    });
}

extern "C" int foil_add_tiles_dev(const uint16_t* a, const uint16_t* b, uint16_t* out, uint64_t n,
                                  void* stream) {
    return guarded([&] {
        if (n % 8) throw FoilError(FOIL_ERR_INVALID, "foil_add_tiles_dev: n must be a multiple of 8");
        if (n == 0) return;
        if (n > (1ull << 62)) throw FoilError(FOIL_ERR_INVALID, "foil_add_tiles_dev: n too large");
        launch_eltwise("foil_add_tiles_dev", foil::stream::kAdd, a, b, out, 2 * n, nullptr, 0,
                       nullptr, (cudaStream_t)stream);
    });
}

extern "C" int foil_relu_tiles_dev(const uint16_t* in, uint16_t* out, uint64_t n, void* stream) {
    return guarded([&] {
        if (n % 8) throw FoilError(FOIL_ERR_INVALID, "foil_relu_tiles_dev: n must be a multiple of 8");
        if (n == 0) return;
        if (n > (1ull << 62)) throw FoilError(FOIL_ERR_INVALID, "foil_relu_tiles_dev: n too large");
        launch_eltwise("foil_relu_tiles_dev", foil::stream::kRelu, in, nullptr, out, 2 * n, nullptr, 0,
                       nullptr, (cudaStream_t)stream);
    });
}

extern "C" int foil_bias_add_tiles_dev(const uint16_t* in, const uint16_t* bias_tiles, uint16_t* out,
                                       uint32_t rows, uint32_t cols, void* stream) {
    return guarded([&] {
        if (rows % 32 || cols % 32)
            throw FoilError(FOIL_ERR_INVALID, "foil_bias_add_tiles_dev: rows and cols must be multiples of 32");
        if (rows == 0 || cols == 0) return;
        launch_eltwise("foil_bias_add_tiles_dev", foil::stream::kBias, in, nullptr, out,
                       (uint64_t)rows * cols * 2, bias_tiles, cols / 32, nullptr, (cudaStream_t)stream);
    });
}

// ------------------------------------------------ host-buffer pipelines ---
// One set of streams, events and grow-only device buffers per device: h2d
// (inputs), comp (kernels) and d2h (outputs), so that the copy of chunk i + 1
// and the read-back of chunk i - 1 overlap the kernel of chunk i, and H2D and
// D2H run at the same time on the full-duplex link.
namespace {
struct HostPipe {
    std::mutex mu;
    cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
    std::vector<cudaEvent_t> ev;
    void* buf[4] = {};
    size_t cap[4] = {};
};
HostPipe g_pipes[64];

HostPipe& pipe_for(int32_t device) {
    if (device < 0 || device >= 64) throw FoilError(FOIL_ERR_INVALID, "tt-foil: device ordinal out of range");
    int count = 0;
    cuda_check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device >= count) throw FoilError(FOIL_ERR_INVALID, "tt-foil: no such CUDA device");
    return g_pipes[device];
}

void pipe_init(HostPipe& hp) {
    if (hp.h2d) return;
    cuda_check(cudaStreamCreateWithFlags(&hp.h2d, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaStreamCreateWithFlags(&hp.comp, cudaStreamNonBlocking), "cudaStreamCreate");
    cuda_check(cudaStreamCreateWithFlags(&hp.d2h, cudaStreamNonBlocking), "cudaStreamCreate");
}

void* pipe_buffer(HostPipe& hp, int slot, size_t bytes) {
    if (hp.cap[slot] < bytes) {
        if (hp.buf[slot]) cuda_check(cudaFree(hp.buf[slot]), "cudaFree");
        hp.buf[slot] = nullptr;
        hp.cap[slot] = 0;
        if (cudaMalloc(&hp.buf[slot], bytes) != cudaSuccess) {
            cudaGetLastError();
            throw FoilError(FOIL_ERR_OOM, "tt-foil: out of device memory for the host pipeline");
        }
        hp.cap[slot] = bytes;
    }
    return hp.buf[slot];
}

cudaEvent_t pipe_event(HostPipe& hp, size_t i) {
    while (hp.ev.size() <= i) {
        cudaEvent_t e;
        cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        hp.ev.push_back(e);
    }
    return hp.ev[i];
}

// Waits for the pipeline's last read-back, then reads and clears the device
// error word (bounded waits that expired in any chunk's kernel).
void pipe_finish(HostPipe& hp, const char* what) {
    cuda_check(cudaStreamSynchronize(hp.d2h), "cudaStreamSynchronize");
    cuda_check(cudaStreamSynchronize(hp.comp), "cudaStreamSynchronize");
    uint32_t* err = error_word_for_current_device();
    uint32_t word = 0;
    cuda_check(cudaMemcpy(&word, err, 4, cudaMemcpyDeviceToHost), "read error word");
    if (word) {
        cuda_check(cudaMemset(err, 0, 4), "clear error word");
        throw FoilError(FOIL_ERR_DEVICE, std::string(what) + ": a bounded device wait expired");
    }
}
}  // namespace

extern "C" int foil_matmul_tiles_host(int32_t device, const uint16_t* a, const uint16_t* b, uint16_t* c,
                                      uint32_t Mt, uint32_t Kt, uint32_t Nt, const uint16_t* bias, int32_t relu,
                                      uint32_t chunk_rows) {
    return guarded([&] {
        if (Mt == 0 || Kt == 0 || Nt == 0) return;
        if (Mt > 65535 || Kt > 65535 || Nt > 65535)
            throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_host: tile counts must be <= 65535");
        if (!a || !b || !c) throw FoilError(FOIL_ERR_INVALID, "foil_matmul_tiles_host: null pointer");
        HostPipe& hp = pipe_for(device);
        DeviceScope scope(device);  // the caller's current device is restored on return
        std::lock_guard<std::mutex> lk(hp.mu);
        pipe_init(hp);
        const size_t tile = 1024;  // elements per 32 x 32 tile
        uint16_t* dA = static_cast<uint16_t*>(pipe_buffer(hp, 0, (size_t)Mt * Kt * tile * 2));
        uint16_t* dB = static_cast<uint16_t*>(pipe_buffer(hp, 1, (size_t)Kt * Nt * tile * 2));
        uint16_t* dC = static_cast<uint16_t*>(pipe_buffer(hp, 2, (size_t)Mt * Nt * tile * 2));
        uint16_t* dBias = bias ? static_cast<uint16_t*>(pipe_buffer(hp, 3, (size_t)Nt * 32 * 2)) : nullptr;
        uint32_t* err = error_word_for_current_device();
        const int sms = sm_count_current();
        // Chunks of 8 tile rows (one 2-SM row block) or more, about 32 chunks:
        // the GEMM and read-back of the last chunk are the part that does not
        // overlap the input copies (8192^3: 5.95 ms with 8 chunks, 5.74 with
        // 32, against 4.85 ms for the 256 MiB of input alone).
        uint32_t chunk = chunk_rows ? chunk_rows : std::max<uint32_t>(8u, (Mt / 32u + 7u) / 8u * 8u);
        cuda_check(cudaMemcpyAsync(dB, b, (size_t)Kt * Nt * tile * 2, cudaMemcpyHostToDevice, hp.h2d), "copy B");
        if (bias) cuda_check(cudaMemcpyAsync(dBias, bias, (size_t)Nt * 64, cudaMemcpyHostToDevice, hp.h2d), "copy bias");
        size_t e = 0;
        for (uint32_t r0 = 0; r0 < Mt; r0 += chunk) {
            const uint32_t rows = std::min(chunk, Mt - r0);
            const size_t ao = (size_t)r0 * Kt * tile, co = (size_t)r0 * Nt * tile;
            cuda_check(cudaMemcpyAsync(dA + ao, a + ao, (size_t)rows * Kt * tile * 2, cudaMemcpyHostToDevice,
                                       hp.h2d), "copy A chunk");
            cudaEvent_t in = pipe_event(hp, e++), done = pipe_event(hp, e++);
            cuda_check(cudaEventRecord(in, hp.h2d), "cudaEventRecord");
            cuda_check(cudaStreamWaitEvent(hp.comp, in, 0), "cudaStreamWaitEvent");
            throw_status(foil::gemm::launch(dA + ao, dB, dC + co, rows, Kt, Nt, dBias, relu, err, hp.comp, sms));
            cuda_check(cudaEventRecord(done, hp.comp), "cudaEventRecord");
            cuda_check(cudaStreamWaitEvent(hp.d2h, done, 0), "cudaStreamWaitEvent");
            cuda_check(cudaMemcpyAsync(c + co, dC + co, (size_t)rows * Nt * tile * 2, cudaMemcpyDeviceToHost,
                                       hp.d2h), "copy C chunk");
        }
        pipe_finish(hp, "foil_matmul_tiles_host");
    });
}

extern "C" int foil_conv2d_nhwc_host(int32_t device, const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                                     uint16_t* y, uint32_t N, uint32_t H, uint32_t W, uint32_t Cin, uint32_t Cout,
                                     uint32_t KH, uint32_t KW, uint32_t stride, uint32_t pad, int32_t relu,
                                     uint32_t chunk_images) {
    return guarded([&] {
        if (N == 0 || Cout == 0) return;
        if (!x || !w || !y) throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_nhwc_host: null pointer");
        if (H == 0 || W == 0 || KH == 0 || KW == 0 || stride == 0 || H + 2 * pad < KH || W + 2 * pad < KW)
            throw FoilError(FOIL_ERR_INVALID, "foil_conv2d_nhwc_host: unsupported kernel / stride / padding");
        HostPipe& hp = pipe_for(device);
        DeviceScope scope(device);  // the caller's current device is restored on return
        std::lock_guard<std::mutex> lk(hp.mu);
        pipe_init(hp);
        const uint64_t Ho = (H + 2 * pad - KH) / stride + 1, Wo = (W + 2 * pad - KW) / stride + 1;
        const size_t x_img = (size_t)H * W * Cin, y_img = (size_t)Ho * Wo * Cout;
        uint16_t* dX = static_cast<uint16_t*>(pipe_buffer(hp, 0, (size_t)N * x_img * 2));
        uint16_t* dW = static_cast<uint16_t*>(pipe_buffer(hp, 1, (size_t)Cout * KH * KW * Cin * 2));
        uint16_t* dY = static_cast<uint16_t*>(pipe_buffer(hp, 2, (size_t)N * y_img * 2));
        uint16_t* dBias = bias ? static_cast<uint16_t*>(pipe_buffer(hp, 3, (size_t)Cout * 2)) : nullptr;
        uint32_t chunk = chunk_images ? chunk_images : std::max<uint32_t>(1u, (N + 7u) / 8u);
        cuda_check(cudaMemcpyAsync(dW, w, (size_t)Cout * KH * KW * Cin * 2, cudaMemcpyHostToDevice, hp.h2d),
                   "copy weights");
        if (bias) cuda_check(cudaMemcpyAsync(dBias, bias, (size_t)Cout * 2, cudaMemcpyHostToDevice, hp.h2d), "copy bias");
        size_t e = 0;
        for (uint32_t n0 = 0; n0 < N; n0 += chunk) {
            const uint32_t imgs = std::min(chunk, N - n0);
            cuda_check(cudaMemcpyAsync(dX + n0 * x_img, x + n0 * x_img, imgs * x_img * 2, cudaMemcpyHostToDevice,
                                       hp.h2d), "copy x chunk");
            cudaEvent_t in = pipe_event(hp, e++), done = pipe_event(hp, e++);
            cuda_check(cudaEventRecord(in, hp.h2d), "cudaEventRecord");
            cuda_check(cudaStreamWaitEvent(hp.comp, in, 0), "cudaStreamWaitEvent");
            throw_status(foil_conv2d_nhwc_dev(dX + n0 * x_img, dW, dBias, dY + n0 * y_img, imgs, H, W, Cin, Cout, KH,
                                              KW, stride, pad, relu, hp.comp));
            cuda_check(cudaEventRecord(done, hp.comp), "cudaEventRecord");
            cuda_check(cudaStreamWaitEvent(hp.d2h, done, 0), "cudaStreamWaitEvent");
            cuda_check(cudaMemcpyAsync(y + n0 * y_img, dY + n0 * y_img, imgs * y_img * 2, cudaMemcpyDeviceToHost,
                                       hp.d2h), "copy y chunk");
        }
        pipe_finish(hp, "foil_conv2d_nhwc_host");
    });
}

extern "C" int foil_host_pipeline_release(int32_t device) {
    return guarded([&] {
        HostPipe& hp = pipe_for(device);
        DeviceScope scope(device);  // the caller's current device is restored on return
        std::lock_guard<std::mutex> lk(hp.mu);
        if (hp.h2d) {
            cuda_check(cudaStreamSynchronize(hp.d2h), "cudaStreamSynchronize");
            cuda_check(cudaStreamSynchronize(hp.comp), "cudaStreamSynchronize");
            cuda_check(cudaStreamSynchronize(hp.h2d), "cudaStreamSynchronize");
        }
        for (int i = 0; i < 4; ++i) {
            if (hp.buf[i]) cuda_check(cudaFree(hp.buf[i]), "cudaFree");
            hp.buf[i] = nullptr;
            hp.cap[i] = 0;
        }
    });
}

extern "C" int foil_device_error_dev(void* stream, uint32_t* out) {
    return guarded([&] {
        if (!out) throw FoilError(FOIL_ERR_INVALID, "tt-foil: null output pointer");
        uint32_t* err = error_word_for_current_device();
        cudaStream_t s = (cudaStream_t)stream;
        cuda_check(cudaMemcpyAsync(out, err, 4, cudaMemcpyDeviceToHost, s), "read error word");
        cuda_check(cudaMemsetAsync(err, 0, 4, s), "clear error word");
        cuda_check(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    });
}
