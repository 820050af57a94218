/*
 * foil_c.h — C-ABI of the B200 tt-foil runtime (libfoil.so).
 *
 * Two layers, both plain C (no C++ or torch types in any signature):
 *
 *  1. The runtime boundary.  One C function per entry point of tt-foil's
 *     public C++ API (include/tt_foil/runtime.hpp and src/cb_config.hpp in
 *     the reference).  The C++ header include/tt_foil/runtime.hpp in this
 *     repository is a thin wrapper over these functions, so a program written
 *     against tt-foil links against libtt_foil.so + libfoil.so unchanged.
 *     A "kernel" is a bundle of program-descriptor files (the reference's
 *     per-RISC ELF names); executing it launches the sm_100a CUDA kernel that
 *     implements that program, with the reference's runtime-argument layout.
 *
 *  2. Device-resident kernel entry points (foil_*_dev).  The same CUDA
 *     kernels, called on CUDA device pointers and a caller-supplied CUDA
 *     stream.  They replace the reference's per-example Tensix compute /
 *     reader / writer kernels (examples/<name>/kernels/<role>.cpp) and the host
 *     tile helpers (tests/tile_utils.hpp) when the data already lives in HBM.
 *
 * Error behaviour: every function returns 0 (FOIL_OK) on success or a
 * foil_status code; foil_last_error() returns the message of the most recent
 * failure on the calling thread.  The C++ wrapper turns any non-zero status
 * into std::runtime_error(message), which is the reference's error behaviour
 * (all failures throw std::runtime_error, src/runtime_impl.cpp:53-55 etc.).
 *
 * Data format: bf16 values are uint16_t bit patterns.  "Tile layout" is the
 * reference wire format (tests/tile_utils.hpp:4-12): 32x32 tiles of four
 * 16x16 faces, faces in order (rows 0-15, cols 0-15), (rows 0-15, cols 16-31),
 * (rows 16-31, cols 0-15), (rows 16-31, cols 16-31), row-major inside a face;
 * a matrix of Rt x Ct tiles is stored tile-row-major (tile (i,j) at i*Ct+j).
 */
#ifndef FOIL_C_H
#define FOIL_C_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FOIL_API __attribute__((visibility("default")))
#else
#define FOIL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status codes                                                              */
/* ------------------------------------------------------------------------ */
typedef enum foil_status {
    FOIL_OK = 0,
    FOIL_ERR_INVALID = 1,     /* bad argument or state                     */
    FOIL_ERR_OOM = 2,         /* L1 / DRAM arena exhausted                 */
    FOIL_ERR_NOT_FOUND = 3,   /* a program-descriptor file does not exist  */
    FOIL_ERR_CUDA = 4,        /* CUDA runtime / driver call failed         */
    FOIL_ERR_TIMEOUT = 5,     /* execute deadline passed                   */
    FOIL_ERR_UNSUPPORTED = 6, /* program outside the accelerated path      */
    FOIL_ERR_DEVICE = 7       /* a kernel reported a device-side error     */
} foil_status;

/* Message for the last non-zero status returned on this thread ("" if none). */
FOIL_API const char* foil_last_error(void);

/* Library build identification string (arch, version). */
FOIL_API const char* foil_version(void);

/* ------------------------------------------------------------------------ */
/* Runtime boundary types                                                    */
/* ------------------------------------------------------------------------ */
typedef struct foil_device foil_device; /* opaque; one per open device      */
typedef struct foil_kernel foil_kernel; /* opaque; one per load_kernel       */

/* Logical core coordinate.  Replaces tt::foil::CoreCoord
 * (include/tt_foil/runtime.hpp:27-31). */
typedef struct foil_core {
    uint32_t x;
    uint32_t y;
} foil_core;

/* Buffer locations.  Replaces tt::foil::BufferLocation (runtime.hpp:37-40). */
enum { FOIL_LOC_L1 = 0, FOIL_LOC_DRAM = 1 };

/* Buffer descriptor.  Replaces tt::foil::Buffer (runtime.hpp:44-49):
 * device_addr is the address a kernel receives as a runtime argument — a
 * 32-bit offset inside the owning core's emulated L1 arena, or an offset
 * inside the device's DRAM arena. */
typedef struct foil_buffer {
    int32_t location;      /* FOIL_LOC_L1 or FOIL_LOC_DRAM */
    uint32_t reserved;
    uint64_t device_addr;
    uint64_t size_bytes;
    foil_core core;        /* owning core for L1 buffers */
} foil_buffer;

/* RISC identifiers.  Replaces RiscBinary::RiscId (runtime.hpp:100-106). */
enum {
    FOIL_RISC_BRISC = 0,
    FOIL_RISC_NCRISC = 1,
    FOIL_RISC_TRISC0 = 2,
    FOIL_RISC_TRISC1 = 3,
    FOIL_RISC_TRISC2 = 4
};

/* One program binary.  Replaces tt::foil::RiscBinary (runtime.hpp:99-109). */
typedef struct foil_risc_binary {
    int32_t risc;
    const char* elf_path;  /* path of a program-descriptor file */
} foil_risc_binary;

/* Circular-buffer description.  Replaces tt::foil::CbConfig
 * (src/cb_config.hpp:42-50). */
typedef struct foil_cb_config {
    uint8_t cb_index;
    uint64_t fifo_addr;
    uint32_t fifo_size;
    uint32_t num_pages;
    uint32_t page_size;
} foil_cb_config;

/* ------------------------------------------------------------------------ */
/* Runtime boundary entry points                                             */
/* ------------------------------------------------------------------------ */

/* Open CUDA device `pcie_device_index` and create one emulated L1 arena per
 * requested core.  firmware_dir is accepted and ignored (there is no
 * firmware).  Replaces tt::foil::open_device (runtime.hpp:64-67;
 * src/device.cpp:116-245).  Errors: no cores, bad index, CUDA failure. */
FOIL_API int foil_open_device(int pcie_device_index, const char* firmware_dir,
                     const foil_core* cores, size_t num_cores,
                     foil_device** out_device);

/* Release every arena and the CUDA resources of the device.  Replaces
 * tt::foil::close_device (runtime.hpp:72; src/device.cpp:247-254). */
FOIL_API int foil_close_device(foil_device* device);

/* Bump-allocate `size_bytes` in a core's L1 arena (16-byte alignment) or in
 * the DRAM arena (32-byte alignment).  Replaces tt::foil::allocate_buffer
 * (runtime.hpp:81-85; src/buffer.cpp:11-35).  Errors: size 0, unknown core,
 * arena exhausted. */
FOIL_API int foil_allocate_buffer(foil_device* device, int32_t location,
                         uint64_t size_bytes, foil_core core,
                         foil_buffer* out_buffer);

/* Bump allocator: releasing a buffer reclaims nothing.  Replaces
 * tt::foil::free_buffer (runtime.hpp:88; src/buffer.cpp:37-41). */
FOIL_API int foil_free_buffer(foil_device* device, const foil_buffer* buffer);

/* Blocking host->device / device->host copies (pageable or pinned host
 * memory).  Replace tt::foil::write_buffer / read_buffer (runtime.hpp:91,94;
 * src/runtime_impl.cpp:52-78).  Errors: bytes > size_bytes. */
FOIL_API int foil_write_buffer(foil_device* device, const foil_buffer* buffer,
                      const void* src, uint64_t bytes);
FOIL_API int foil_read_buffer(foil_device* device, const foil_buffer* buffer,
                     void* dst, uint64_t bytes);

/* Read the program-descriptor files named by `binaries` and bind the kernel
 * to `core`.  Replaces tt::foil::load_kernel (runtime.hpp:114-117;
 * src/kernel.cpp:16-62).  Errors: empty list, missing file, core not opened,
 * descriptors of different programs, program outside the path. */
FOIL_API int foil_load_kernel(foil_device* device, const foil_risc_binary* binaries,
                     size_t num_binaries, foil_core core,
                     foil_kernel** out_kernel);

/* Free a kernel handle (the C++ wrapper's shared_ptr deleter). */
FOIL_API int foil_release_kernel(foil_kernel* kernel);

/* Store up to 64 runtime-argument words for one RISC of the kernel.
 * Replaces tt::foil::set_runtime_args (runtime.hpp:120-124;
 * src/kernel.cpp:66-83).  Errors: >64 words, RISC not in the kernel. */
FOIL_API int foil_set_runtime_args(foil_device* device, foil_kernel* kernel,
                          int32_t risc, const uint32_t* args,
                          size_t num_args);

/* Validate and record circular-buffer descriptors (indices < 32, no
 * duplicates, rings inside the core's L1 arena).  The CUDA kernels stage
 * tiles in shared memory, so the rings only need to be valid.  Replaces
 * tt::foil::register_cbs (src/cb_config.hpp:68-71; src/cb_config.cpp:27-112).
 */
FOIL_API int foil_register_cbs(foil_device* device, foil_kernel* kernel,
                      const foil_cb_config* cbs, size_t num_cbs);

/* Launch every kernel, then wait until all have finished or `timeout_ms`
 * (shared budget, <=0 means 5000 ms) has passed.  Kernels of one call that
 * run the same program are fused into one grouped CUDA launch.  Replaces
 * tt::foil::execute (runtime.hpp:132,137; src/dispatch.cpp:218-274).
 * Errors: empty list, bad runtime args, timeout, device-side error. */
FOIL_API int foil_execute(foil_device* device, foil_kernel* const* kernels,
                 size_t num_kernels, int32_t timeout_ms);

/* Pack a 64-bit address of `local_l1_addr` in core `dst`'s L1 arena.
 * Replaces tt::foil::make_noc_unicast_addr (runtime.hpp:151-154;
 * src/noc_addr.cpp:10-22): bits [47:42] = y, [41:36] = x, [35:0] = offset. */
FOIL_API int foil_make_noc_unicast_addr(foil_device* device, foil_core dst,
                               uint64_t local_l1_addr, uint64_t* out_addr);

/* Pack a 64-bit address of `dram_offset` in the DRAM arena.  Replaces
 * tt::foil::make_noc_dram_addr (runtime.hpp:160; runtime_impl.cpp:124-131). */
FOIL_API int foil_make_noc_dram_addr(foil_device* device, uint64_t dram_offset,
                            uint64_t* out_addr);

/* CUDA device pointer behind a buffer (for device-resident callers). */
FOIL_API int foil_buffer_device_ptr(foil_device* device, const foil_buffer* buffer,
                           void** out_ptr);

/* Number of CUDA kernel launches issued by this process so far (all
 * entry points). */
FOIL_API uint64_t foil_launch_count(void);

/* ------------------------------------------------------------------------ */
/* Device-resident kernel entry points.  All pointers are CUDA device        */
/* pointers of the current device; `stream` is a cudaStream_t (NULL = the    */
/* legacy default stream).  Launches are asynchronous.                       */
/* ------------------------------------------------------------------------ */

/* Row-major (rows x cols) bf16 -> tile layout; rows, cols multiples of 32.
 * Replaces row_major_to_tile + tile_matrix (tests/tile_utils.hpp:51-65;
 * tests/test_conv_3x3.cpp:144-158). */
FOIL_API int foil_tilize_dev(const uint16_t* row_major, uint16_t* tiles,
                    uint32_t rows, uint32_t cols, void* stream);

/* Tile layout -> row-major.  Replaces tile_to_row_major + untile_matrix
 * (tests/tile_utils.hpp:68-80; tests/test_conv_3x3.cpp:160-174). */
FOIL_API int foil_untilize_dev(const uint16_t* tiles, uint16_t* row_major,
                      uint32_t rows, uint32_t cols, void* stream);

/* Element-wise stages below: pointers 16-byte aligned; the output may be the
 * same buffer as an input (in place) but must not partially overlap one
 * (FOIL_ERR_INVALID).  A stalled copy sets the device error word.
 *
 * Identity copy of `bytes` (multiple of 16).
 * Replaces examples/tile_copy/kernels/{reader,compute,writer}.cpp. */
FOIL_API int foil_tile_copy_dev(const void* src, void* dst, uint64_t bytes,
                       void* stream);

/* out = bf16(f32(a) + f32(b)) element-wise on n bf16 values (n multiple of
 * 8).  Replaces examples/add_tiles/kernels/compute.cpp:19-43. */
FOIL_API int foil_add_tiles_dev(const uint16_t* a, const uint16_t* b, uint16_t* out,
                       uint64_t n, void* stream);

/* out = max(x, 0) element-wise (bit-exact), n multiple of 8.  Replaces
 * examples/relu/kernels/compute.cpp:19-45. */
FOIL_API int foil_relu_tiles_dev(const uint16_t* in, uint16_t* out, uint64_t n,
                        void* stream);

/* Row-broadcast bias on a tile-layout matrix of rows x cols:
 * out[r][c] = bf16(f32(in[r][c]) + f32(bias[0][c])), where `bias_tiles` is a
 * tile-layout band of 1 x (cols/32) tiles whose row 0 holds the bias (the
 * reference's bias-tile convention, tests/test_bias_add.cpp:53-56); the
 * output must not overlap the bias band.
 * Replaces examples/bias_add/kernels/compute.cpp:19-42. */
FOIL_API int foil_bias_add_tiles_dev(const uint16_t* in, const uint16_t* bias_tiles,
                            uint16_t* out, uint32_t rows, uint32_t cols,
                            void* stream);

/* Tiled bf16 GEMM on tcgen05 tensor cores: C (Mt x Nt tiles) = A (Mt x Kt
 * tiles) . B (Kt x Nt tiles), fp32 accumulation, bf16 output, all in tile
 * layout.  Optional fused epilogue: if `bias` is non-NULL (N = 32*Nt bf16
 * values, one per output column) out = bf16(f32(bf16(acc)) + bias[n]); if
 * `relu` is non-zero the result is clamped at 0.  Replaces the matmul
 * compute kernel (examples/matmul_mnk/kernels/compute.cpp:23-53) and its
 * reader / writer (examples/matmul_mnk/kernels/reader.cpp:28-57,
 * writer.cpp:16-34), followed by bias_add and relu. */
FOIL_API int foil_matmul_tiles_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                          uint32_t Mt, uint32_t Kt, uint32_t Nt,
                          const uint16_t* bias, int32_t relu, void* stream);

/* foil_matmul_tiles_dev whose kernel is also its own all-gather: every
 * output tile is stored to `c` and to each of peer_c[0 .. npeers) (at most
 * 7), other GPUs' buffers opened with foil_peer_open and offset like `c`.
 * With the rows of C split over the GPUs of a node (each rank computing its
 * tile rows into its slice of a full-size C), one launch per rank leaves the
 * whole C on every GPU once all ranks' launches are complete (order a
 * collective, e.g. a one-element all-reduce, after the launch before reading
 * the peers' rows).  Replaces the per-core row split of
 * tests/test_matmul_2core.cpp:43-63 (tests/test_matmul_4x2.cpp:164-180
 * stitches the shards on the host) followed by a separate gather. */
FOIL_API int foil_matmul_tiles_gather_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                          uint16_t* const* peer_c, uint32_t npeers,
                          uint32_t Mt, uint32_t Kt, uint32_t Nt,
                          const uint16_t* bias, int32_t relu, void* stream);

/* foil_matmul_tiles_gather_dev through an NVLink multicast object: `mc_c`
 * is the multicast address, at c's offset, of a buffer bound on every GPU of
 * the node (this one included; e.g. PyTorch symmetric memory's
 * multicast_ptr).  Each output tile is stored once through it and the
 * NVSwitch writes it into every GPU's copy.  The same fence as for
 * foil_matmul_tiles_gather_dev orders the ranks. */
FOIL_API int foil_matmul_tiles_gather_mc_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                          uint16_t* mc_c, uint32_t Mt, uint32_t Kt, uint32_t Nt,
                          const uint16_t* bias, int32_t relu, void* stream);

/* The same result as foil_matmul_tiles_gather_dev, with the transfer on the
 * copy engines instead of the SMs: the GEMM runs as `chunks` launches over
 * row chunks of C (whole 256-row blocks, 1..64 chunks) on `stream`, and as
 * soon as a chunk's launch completes one copy stream per peer copies that
 * chunk into peer_c[d] (cudaMemcpyAsync over NVLink) while the next chunk
 * computes.  `stream` waits for every copy before its later work, so the
 * same fence as for foil_matmul_tiles_gather_dev orders the ranks. */
FOIL_API int foil_matmul_tiles_gather_ce_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                          uint16_t* const* peer_c, uint32_t npeers,
                          uint32_t Mt, uint32_t Kt, uint32_t Nt,
                          const uint16_t* bias, int32_t relu, uint32_t chunks, void* stream);

/* Device buffers shared between the processes of a node (CUDA IPC).
 * foil_peer_alloc allocates `bytes` on CUDA device `device` and writes its
 * 64-byte export handle; another process passes the handle to
 * foil_peer_open to get a pointer to the same memory usable from its own
 * device (peer access over NVLink), and releases it with foil_peer_close.
 * The owner frees with foil_peer_free after every opener has closed it. */
#define FOIL_PEER_HANDLE_BYTES 64
FOIL_API int foil_peer_alloc(int32_t device, uint64_t bytes, void** ptr, uint8_t* handle);
FOIL_API int foil_peer_open(int32_t device, const uint8_t* handle, void** ptr);
FOIL_API int foil_peer_close(int32_t device, void* ptr);
FOIL_API int foil_peer_free(int32_t device, void* ptr);

/* NHWC convolution as an implicit GEMM on tcgen05 tensor cores, with fused
 * bias and relu: y (N, Ho, Wo, Cout) = relu?(bf16(bf16(conv(x, w)) + bias)),
 * x (N, H, W, Cin), w (Cout, KH, KW, Cin), bias (Cout) or NULL, fp32
 * accumulation, Ho = (H + 2 pad - KH) / stride + 1.  Cin and Cout must be
 * multiples of 16.  Replaces the reference's conv path — host im2col
 * (tests/test_conv_3x3.cpp:108-127, test_conv_3x3_s2.cpp:114-133) feeding
 * the tiled matmul (tests/test_conv_3x3.cpp:214-222) — followed by bias_add
 * and relu. */
FOIL_API int foil_conv2d_nhwc_dev(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                                  uint16_t* y, uint32_t N, uint32_t H, uint32_t W, uint32_t Cin,
                                  uint32_t Cout, uint32_t KH, uint32_t KW, uint32_t stride,
                                  uint32_t pad, int32_t relu, void* stream);

/* The same convolution in the reference's own tensor convention: x (N,
 * Cin, H, W) channel-major activations, w (Cout, Cin * KH * KW) -- the
 * reference's reshaped weights, i.e. (Cout, Cin, KH, KW) -- bias (Cout) or
 * NULL, y (N, Cout, Ho, Wo); any Cin and Cout.  The operands are re-laid on
 * the device (batched transposes into a stream-ordered workspace, channels
 * zero-padded to multiples of 16), then the NHWC convolution above runs and
 * its output is transposed back; the caller's host does no im2col or
 * transposition.  Replaces the reference conv tests' host preparation --
 * im2col (tests/test_conv_3x3.cpp:108-127, test_conv_3x3_s2.cpp:114-133) and
 * weight_reshape (tests/test_conv_3x3.cpp:130-141) -- feeding the tiled
 * matmul, for N images at once. */
FOIL_API int foil_conv2d_chw_dev(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* y,
                                 uint32_t N, uint32_t Cin, uint32_t H, uint32_t W, uint32_t Cout,
                                 uint32_t KH, uint32_t KW, uint32_t stride, uint32_t pad, int32_t relu,
                                 void* stream);

/* Allocation-free variant of foil_matmul_tiles_dev, for callers that cannot
 * allocate device memory when they launch (allocator or memory-pool
 * callbacks, processes whose GPU memory another allocator already owns,
 * loops that forbid allocation after start-up).  No counterpart in the
 * reference, which has no allocation-free launch path.  Same kernel and
 * arguments; its 4-byte scratch (the device error word) lives in a 256-byte
 * array compiled into the library, so the call makes no cudaMalloc, cudaFree
 * or other allocating call; scratch needs beyond 256 bytes are rejected.  The
 * first call on each device resolves the array's address (make it before any
 * stream capture).  All calls on a device share the array and each clears it
 * first, so calls that overlap on the GPU race on it.  If `status_out` is
 * non-NULL (host memory; page-locked to stay allocation-free) the call
 * synchronizes `stream` and stores the error word (0 = no bounded wait
 * expired), returning FOIL_ERR_DEVICE when it is set.  With `status_out`
 * NULL the call does not wait and an expired wait is not observable: the
 * word lives only in the library's array (foil_device_error_dev reads the
 * other entry points' word, not this one) and the next call clears it, so
 * a kernel that gave up part-way and left C incomplete then looks like a
 * success.  Pass `status_out` wherever that matters. */
FOIL_API int foil_matmul_tiles_noalloc_dev(const uint16_t* a, const uint16_t* b, uint16_t* c,
                                           uint32_t Mt, uint32_t Kt, uint32_t Nt,
                                           const uint16_t* bias, int32_t relu, void* stream,
                                           uint32_t* status_out);

/* Wall-time limit of every bounded device-side wait (mbarrier, flag and
 * counter waits inside the kernels), in nanoseconds, for the launches that
 * follow; process-wide.  A kernel whose wait runs past it records
 * FOIL_DEVERR_WAIT_TIMEOUT in the device error word, stops its pipeline
 * roles, waits (bounded) for its copies and tensor-core operations in
 * flight, frees its tensor memory and returns, so the context stays usable.
 * 0 restores the default of 2 s.  Returns the previous limit.  The B200
 * counterpart of the reference's dispatch timeout (src/dispatch.cpp:203-208),
 * moved into the kernels. */
FOIL_API uint64_t foil_set_wait_limit_ns(uint64_t ns);

/* Bits of the device error word. */
#define FOIL_DEVERR_WAIT_TIMEOUT 1u /* a bounded wait gave up */
#define FOIL_DEVERR_BAD_SHAPE 2u    /* a kernel saw a shape it cannot handle */
#define FOIL_DEVERR_CONFIG 4u       /* launch parameters inconsistent with the kernel; nothing ran */

/* Read and clear the device-side error word of the current device: 0 if no
 * kernel reported an error (bounded waits that gave up) since the last call.
 * Synchronizes `stream`. */
FOIL_API int foil_device_error_dev(void* stream, uint32_t* out_error);

/* Tiled GEMM on host buffers, pipelined: C (Mt x Nt tiles) = A (Mt x Kt) .
 * B (Kt x Nt), tile streams in host memory, optional bias (Nt * 32 values,
 * one per output column, NULL for none) and relu as in
 * foil_matmul_tiles_dev, on CUDA device `device`.  B is copied first, then A
 * in chunks of `chunk_rows` tile rows (0 = about 32 chunks, at least 8 rows):
 * the copy of chunk i + 1 and the read-back of chunk i - 1 overlap the GEMM
 * of chunk i, and host-to-device and device-to-host copies run at the same
 * time.  Blocking: returns when C is in host memory.  Replaces the
 * reference's blocking sequence write_buffer(A), write_buffer(B), execute,
 * read_buffer(C) (include/tt_foil/runtime.hpp:91, :132, :94;
 * tests/test_matmul_dram.cpp:163-208).  Host buffers should be page-locked
 * for the copies to overlap; pageable buffers work but serialize.  Device
 * buffers are cached per device and grow as needed (one call at a time per
 * device; foil_host_pipeline_release frees them). */
FOIL_API int foil_matmul_tiles_host(int32_t device, const uint16_t* a, const uint16_t* b, uint16_t* c,
                                    uint32_t Mt, uint32_t Kt, uint32_t Nt, const uint16_t* bias,
                                    int32_t relu, uint32_t chunk_rows);

/* NHWC convolution on host buffers, pipelined over chunks of `chunk_images`
 * images (0 = about 8 chunks) as foil_matmul_tiles_host; arguments as
 * foil_conv2d_nhwc_dev.  Replaces the reference conv tests' write_buffer /
 * execute / read_buffer sequence around the host im2col
 * (tests/test_conv_3x3.cpp:236-279). */
FOIL_API int foil_conv2d_nhwc_host(int32_t device, const uint16_t* x, const uint16_t* w,
                                   const uint16_t* bias, uint16_t* y, uint32_t N, uint32_t H,
                                   uint32_t W, uint32_t Cin, uint32_t Cout, uint32_t KH, uint32_t KW,
                                   uint32_t stride, uint32_t pad, int32_t relu,
                                   uint32_t chunk_images);

/* Free the device buffers cached by the host pipelines on `device`. */
FOIL_API int foil_host_pipeline_release(int32_t device);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* FOIL_C_H */
