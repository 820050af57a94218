// ORACLE — test infrastructure only.
//
// CPU restatement of tt-foil's golden path (the reference's own CPU
// reference code in tests/*.cpp and tests/tile_utils.hpp), generalised from
// its compile-time shapes to run-time shapes.  It is the checker for the
// CUDA kernels of tt-foil_b200 and the timed CPU baseline of bench.py; the
// product library never links or calls it.
//
// Pinning: tests/test_oracle.py checks these functions against golden
// fixtures (tests/golden/) produced by the reference's own code, compiled
// from its sources by the recipe oracle/build.py, and — when oracle/_ref is built —
// against that code directly.
//
// Every function states the reference lines it restates.  bf16 values are
// uint16_t bit patterns; matrices are row-major unless a name says "tiles".
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#define ORACLE_API extern "C" __attribute__((visibility("default")))

namespace {

// tests/tile_utils.hpp:33-40 — round to nearest even by adding 0x7fff plus
// the lowest kept bit, then truncating; no NaN special case.
inline uint16_t to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

// tests/tile_utils.hpp:42-47.
inline float from_bf16(uint16_t b) {
    uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Offset of element (r, c) of a 32x32 block inside one tile
// (tests/tile_utils.hpp:51-65: face = (r/16)*2 + c/16, row-major in a face).
inline uint32_t tile_offset(uint32_t r, uint32_t c) {
    return ((r >> 4) * 2u + (c >> 4)) * 256u + (r & 15u) * 16u + (c & 15u);
}

template <class F>
void parallel_rows(uint32_t begin, uint32_t end, int threads, F&& f) {
    if (threads <= 1 || end - begin < 2) {
        f(begin, end);
        return;
    }
    std::vector<std::thread> pool;
    uint32_t n = end - begin;
    uint32_t per = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        uint32_t b = begin + t * per;
        uint32_t e = b + per < end ? b + per : end;
        if (b >= e) break;
        pool.emplace_back([&f, b, e] { f(b, e); });
    }
    for (auto& th : pool) th.join();
}

}  // namespace

ORACLE_API uint16_t oracle_f32_to_bf16(float f) { return to_bf16(f); }
ORACLE_API float oracle_bf16_to_f32(uint16_t b) { return from_bf16(b); }

ORACLE_API void oracle_f32_to_bf16_array(const float* in, uint16_t* out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) out[i] = to_bf16(in[i]);
}

// Row-major (rows x cols) -> tile stream, tile (rt, ct) at rt*Ct + ct.
// tile_matrix (tests/test_conv_3x3.cpp:144-158) built on row_major_to_tile
// (tests/tile_utils.hpp:51-65); tile_A_stream / tile_B_stream
// (tests/test_matmul_mnk.cpp:80-112) are the same map.
ORACLE_API void oracle_tilize(const uint16_t* rm, uint16_t* tiles, uint32_t rows, uint32_t cols) {
    const uint32_t Rt = rows / 32, Ct = cols / 32;
    for (uint32_t rt = 0; rt < Rt; ++rt)
        for (uint32_t ct = 0; ct < Ct; ++ct) {
            uint16_t* t = tiles + (uint64_t(rt) * Ct + ct) * 1024;
            for (uint32_t r = 0; r < 32; ++r)
                for (uint32_t c = 0; c < 32; ++c)
                    t[tile_offset(r, c)] = rm[uint64_t(rt * 32 + r) * cols + ct * 32 + c];
        }
}

// Inverse: untile_matrix (tests/test_conv_3x3.cpp:160-174) on
// tile_to_row_major (tests/tile_utils.hpp:68-80); untile_C_stream
// (tests/test_matmul_mnk.cpp:114-129).
ORACLE_API void oracle_untilize(const uint16_t* tiles, uint16_t* rm, uint32_t rows, uint32_t cols) {
    const uint32_t Rt = rows / 32, Ct = cols / 32;
    for (uint32_t rt = 0; rt < Rt; ++rt)
        for (uint32_t ct = 0; ct < Ct; ++ct) {
            const uint16_t* t = tiles + (uint64_t(rt) * Ct + ct) * 1024;
            for (uint32_t r = 0; r < 32; ++r)
                for (uint32_t c = 0; c < 32; ++c)
                    rm[uint64_t(rt * 32 + r) * cols + ct * 32 + c] = t[tile_offset(r, c)];
        }
}

// C = A . B for output rows [row_begin, row_end): fp32 accumulation in K
// order, one bf16 rounding at the end — matmul_reference
// (tests/test_matmul_mnk.cpp:62-76; test_matmul_kt.cpp, test_matmul_1tile.cpp
// use the same loop).  A is M x K, B is K x N, C is M x N (only the requested
// rows are written).  `threads` > 1 splits the rows over std::threads with
// identical per-element arithmetic.
ORACLE_API void oracle_matmul(const uint16_t* a, const uint16_t* b, uint16_t* c, uint32_t M,
                              uint32_t N, uint32_t K, uint32_t row_begin, uint32_t row_end,
                              int threads) {
    (void)M;
    parallel_rows(row_begin, row_end, threads, [&](uint32_t rb, uint32_t re) {
        for (uint32_t i = rb; i < re; ++i)
            for (uint32_t j = 0; j < N; ++j) {
                float acc = 0.0f;
                for (uint32_t k = 0; k < K; ++k)
                    acc += from_bf16(a[uint64_t(i) * K + k]) * from_bf16(b[uint64_t(k) * N + j]);
                c[uint64_t(i) * N + j] = to_bf16(acc);
            }
    });
}

// Tile-stream GEMM: the reference's device contract (C tiles (mt,nt) =
// sum over kt of A tiles (mt,kt) . B tiles (kt,nt), fp32 accumulate, bf16
// out), evaluated with the golden's sequential K order on untilized data.
ORACLE_API void oracle_matmul_tiles(const uint16_t* a_tiles, const uint16_t* b_tiles,
                                    uint16_t* c_tiles, uint32_t Mt, uint32_t Kt, uint32_t Nt,
                                    int threads) {
    const uint32_t M = Mt * 32, K = Kt * 32, N = Nt * 32;
    std::vector<uint16_t> a(uint64_t(M) * K), b(uint64_t(K) * N), c(uint64_t(M) * N);
    oracle_untilize(a_tiles, a.data(), M, K);
    oracle_untilize(b_tiles, b.data(), K, N);
    oracle_matmul(a.data(), b.data(), c.data(), M, N, K, 0, M, threads);
    oracle_tilize(c.data(), c_tiles, M, N);
}

// Direct convolution on CHW tensors, pad p, stride s, square kernel kh x kw:
// conv3x3_reference (tests/test_conv_3x3.cpp:78-104), conv3x3_s2_reference
// (tests/test_conv_3x3_s2.cpp:86-110) and conv_1x1_reference
// (tests/test_conv_1x1.cpp:80-97, kh = kw = 1, p = 0).  Accumulation order
// per output: ci, then ki, then kj; padded taps are skipped; bf16 once.
// Weights are (Cout, Cin, kh, kw).
ORACLE_API void oracle_conv_chw(const uint16_t* x, const uint16_t* w, uint16_t* y, uint32_t Cin,
                                uint32_t H, uint32_t W, uint32_t Cout, uint32_t kh, uint32_t kw,
                                uint32_t stride, uint32_t pad) {
    const uint32_t Ho = (H + 2 * pad - kh) / stride + 1, Wo = (W + 2 * pad - kw) / stride + 1;
    for (uint32_t co = 0; co < Cout; ++co)
        for (uint32_t ho = 0; ho < Ho; ++ho)
            for (uint32_t wo = 0; wo < Wo; ++wo) {
                float acc = 0.0f;
                for (uint32_t ci = 0; ci < Cin; ++ci)
                    for (uint32_t ki = 0; ki < kh; ++ki)
                        for (uint32_t kj = 0; kj < kw; ++kj) {
                            int ih = int(ho * stride + ki) - int(pad);
                            int iw = int(wo * stride + kj) - int(pad);
                            if (ih < 0 || ih >= int(H) || iw < 0 || iw >= int(W)) continue;
                            acc += from_bf16(x[(uint64_t(ci) * H + ih) * W + iw]) *
                                   from_bf16(w[((uint64_t(co) * Cin + ci) * kh + ki) * kw + kj]);
                        }
                y[(uint64_t(co) * Ho + ho) * Wo + wo] = to_bf16(acc);
            }
}

// Host im2col of a CHW tensor into a (Cin*kh*kw) x (Ho*Wo) row-major matrix,
// row = ci*kh*kw + ki*kw + kj, column = ho*Wo + wo, zeros for padding:
// im2col (tests/test_conv_3x3.cpp:108-127), im2col_s2
// (tests/test_conv_3x3_s2.cpp:114-133); for 1x1 it is the identity
// chw_to_matrix (tests/test_conv_1x1.cpp:102-107).
ORACLE_API void oracle_im2col_chw(const uint16_t* x, uint16_t* a, uint32_t Cin, uint32_t H,
                                  uint32_t W, uint32_t kh, uint32_t kw, uint32_t stride,
                                  uint32_t pad) {
    const uint32_t Ho = (H + 2 * pad - kh) / stride + 1, Wo = (W + 2 * pad - kw) / stride + 1;
    const uint64_t ncol = uint64_t(Ho) * Wo;
    std::memset(a, 0, uint64_t(Cin) * kh * kw * ncol * 2);
    for (uint32_t ci = 0; ci < Cin; ++ci)
        for (uint32_t ki = 0; ki < kh; ++ki)
            for (uint32_t kj = 0; kj < kw; ++kj) {
                uint64_t row = uint64_t(ci) * kh * kw + ki * kw + kj;
                for (uint32_t ho = 0; ho < Ho; ++ho) {
                    int ih = int(ho * stride + ki) - int(pad);
                    if (ih < 0 || ih >= int(H)) continue;
                    for (uint32_t wo = 0; wo < Wo; ++wo) {
                        int iw = int(wo * stride + kj) - int(pad);
                        if (iw < 0 || iw >= int(W)) continue;
                        a[row * ncol + uint64_t(ho) * Wo + wo] = x[(uint64_t(ci) * H + ih) * W + iw];
                    }
                }
            }
}

// Weight reshape (Cout, Cin, kh, kw) -> (Cout, Cin*kh*kw) is the identity on
// row-major memory (tests/test_conv_3x3.cpp:130-141); provided for symmetry.
ORACLE_API void oracle_weight_reshape(const uint16_t* w, uint16_t* wm, uint32_t Cout, uint32_t Cin,
                                      uint32_t kh, uint32_t kw) {
    std::memcpy(wm, w, uint64_t(Cout) * Cin * kh * kw * 2);
}

// NHWC convolution with fused bias and relu, the layout of the B200
// implicit-GEMM conv.  Same sums as oracle_conv_chw, same per-output
// accumulation order (ci, ki, kj).  x is (N, H, W, Cin); w is
// (Cout, kh, kw, Cin); y is (N, Ho, Wo, Cout).  Epilogue = composition of the
// reference goldens: y = relu(bf16(bf16(acc) + bias[co]))
// (tests/test_bias_add.cpp:61-68, tests/test_relu.cpp:54-59).  `bias` may be
// null; relu != 0 enables the clamp.  Images [n_begin, n_end) are computed.
ORACLE_API void oracle_conv_nhwc(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                                 uint16_t* y, uint32_t N, uint32_t H, uint32_t W, uint32_t Cin,
                                 uint32_t Cout, uint32_t kh, uint32_t kw, uint32_t stride,
                                 uint32_t pad, int relu, uint32_t n_begin, uint32_t n_end,
                                 int threads) {
    (void)N;
    const uint32_t Ho = (H + 2 * pad - kh) / stride + 1, Wo = (W + 2 * pad - kw) / stride + 1;
    // Parallelise over output rows (n, ho) with identical arithmetic.
    const uint32_t rb0 = n_begin * Ho, re0 = n_end * Ho;
    parallel_rows(rb0, re0, threads, [&](uint32_t rb, uint32_t re) {
        for (uint32_t row = rb; row < re; ++row) {
            const uint32_t n = row / Ho, ho = row % Ho;
            for (uint32_t wo = 0; wo < Wo; ++wo)
                for (uint32_t co = 0; co < Cout; ++co) {
                    float acc = 0.0f;
                    for (uint32_t ci = 0; ci < Cin; ++ci)
                        for (uint32_t ki = 0; ki < kh; ++ki)
                            for (uint32_t kj = 0; kj < kw; ++kj) {
                                int ih = int(ho * stride + ki) - int(pad);
                                int iw = int(wo * stride + kj) - int(pad);
                                if (ih < 0 || ih >= int(H) || iw < 0 || iw >= int(W)) continue;
                                acc += from_bf16(x[((uint64_t(n) * H + ih) * W + iw) * Cin + ci]) *
                                       from_bf16(w[((uint64_t(co) * kh + ki) * kw + kj) * Cin + ci]);
                            }
                    uint16_t o = to_bf16(acc);
                    if (bias) o = to_bf16(from_bf16(o) + from_bf16(bias[co]));
                    if (relu) o = to_bf16(from_bf16(o) < 0.0f ? 0.0f : from_bf16(o));
                    y[((uint64_t(n) * Ho + ho) * Wo + wo) * Cout + co] = o;
                }
        }
    });
}

// Row-broadcast bias: out[r][c] = bf16(in[r][c] + bias[c])
// (tests/test_bias_add.cpp:61-68), row-major.
ORACLE_API void oracle_bias_add(const uint16_t* in, const uint16_t* bias, uint16_t* out,
                                uint32_t rows, uint32_t cols) {
    for (uint64_t r = 0; r < rows; ++r)
        for (uint32_t c = 0; c < cols; ++c)
            out[r * cols + c] = to_bf16(from_bf16(in[r * cols + c]) + from_bf16(bias[c]));
}

// relu: bf16(v < 0 ? 0 : v) (tests/test_relu.cpp:54-59).
ORACLE_API void oracle_relu(const uint16_t* in, uint16_t* out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        float v = from_bf16(in[i]);
        out[i] = to_bf16(v < 0.0f ? 0.0f : v);
    }
}

// add: bf16(fp32(a) + fp32(b)) (tests/test_add_tiles.cpp:57-61).
ORACLE_API void oracle_add(const uint16_t* a, const uint16_t* b, uint16_t* out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) out[i] = to_bf16(from_bf16(a[i]) + from_bf16(b[i]));
}

// Reference test inputs (closed-form, no RNG):
// matmul family A[r][k] = bf16(0.005 * ((r+1) + k%7)), B[k][c] = bf16(0.005 *
// ((c+1) + k%5)) (tests/test_matmul_mnk.cpp:146-155).
ORACLE_API void oracle_gen_matmul_inputs(uint16_t* a, uint16_t* b, uint32_t M, uint32_t K,
                                         uint32_t N) {
    for (uint32_t r = 0; r < M; ++r)
        for (uint32_t k = 0; k < K; ++k)
            a[uint64_t(r) * K + k] = to_bf16(0.005f * static_cast<float>((r + 1) + (k % 7)));
    for (uint32_t k = 0; k < K; ++k)
        for (uint32_t c = 0; c < N; ++c)
            b[uint64_t(k) * N + c] = to_bf16(0.005f * static_cast<float>((c + 1) + (k % 5)));
}

// conv inputs: x[ci][h][w] = bf16(0.005 * ((ci+1) + (h*W+w)%7)),
// w[co][ci][ki][kj] = bf16(0.005 * ((co+1) + ci%5 + ki*3+kj))
// (tests/test_conv_3x3.cpp:190-202; 1x1: tests/test_conv_1x1.cpp:168-182
// with ki = kj = 0).
ORACLE_API void oracle_gen_conv_inputs(uint16_t* x, uint16_t* w, uint32_t Cin, uint32_t H,
                                       uint32_t W, uint32_t Cout, uint32_t kh, uint32_t kw) {
    for (uint32_t ci = 0; ci < Cin; ++ci)
        for (uint32_t h = 0; h < H; ++h)
            for (uint32_t x_ = 0; x_ < W; ++x_)
                x[(uint64_t(ci) * H + h) * W + x_] =
                    to_bf16(0.005f * static_cast<float>((ci + 1) + ((h * W + x_) % 7)));
    for (uint32_t co = 0; co < Cout; ++co)
        for (uint32_t ci = 0; ci < Cin; ++ci)
            for (uint32_t ki = 0; ki < kh; ++ki)
                for (uint32_t kj = 0; kj < kw; ++kj)
                    w[((uint64_t(co) * Cin + ci) * kh + ki) * kw + kj] =
                        to_bf16(0.005f * static_cast<float>((co + 1) + (ci % 5) + (ki * 3 + kj)));
}

// Comparator of the reference tests (tests/test_matmul_mnk.cpp:217-239):
// element i fails when |got - exp| > max(abs_tol, rel_tol * |exp|).  Returns
// the number of failures; writes the worst abs and rel errors.
ORACLE_API uint64_t oracle_compare(const uint16_t* got, const uint16_t* exp, uint64_t n,
                                   float abs_tol, float rel_tol, float* worst_abs,
                                   float* worst_rel) {
    uint64_t bad = 0;
    float wa = 0.0f, wr = 0.0f;
    for (uint64_t i = 0; i < n; ++i) {
        float g = from_bf16(got[i]), e = from_bf16(exp[i]);
        float d = std::fabs(g - e), ref = std::fabs(e);
        float tol = abs_tol > rel_tol * ref ? abs_tol : rel_tol * ref;
        if (d > wa) wa = d;
        if (ref > 0.0f && d / ref > wr) wr = d / ref;
        if (d > tol || d != d) ++bad;
    }
    if (worst_abs) *worst_abs = wa;
    if (worst_rel) *worst_rel = wr;
    return bad;
}
