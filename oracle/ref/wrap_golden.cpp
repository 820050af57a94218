// ORACLE — test infrastructure only.
//
// Exposes the reference's own golden functions, compiled from its sources
// where they lie (the test file is included from the reference tree by the
// recipe oracle/build.py), through extern "C" entry points.  The
// reference keeps its goldens in anonymous namespaces of test files whose
// main() drives the device, so this translation unit includes the whole test
// file with main renamed and adds wrappers in the same unit.  Shapes are the
// test's compile-time MM_* values, passed by oracle/build.py.
//
// Built once per (test file, shape): REF_TEST names the file, REF_TAG the
// symbol suffix, REF_KIND selects the wrapper set.
#include <algorithm>
#include <cstdint>
#include <vector>

#define REF_CAT2(a, b) a##b
#define REF_CAT(a, b) REF_CAT2(a, b)
#define REF_STR2(x) #x
#define REF_STR(x) REF_STR2(x)

#define main REF_CAT(reference_test_main_, REF_TAG)
#include REF_STR(REF_TEST)
#undef main

#define REF_EXPORT extern "C" __attribute__((visibility("default")))

namespace {
template <class T>
std::vector<T> vec(const T* p, size_t n) {
    return std::vector<T>(p, p + n);
}
template <class T>
void out(const std::vector<T>& v, T* p) {
    std::copy(v.begin(), v.end(), p);
}
}  // namespace

#if REF_KIND == 1  // matmul tests: matmul_reference + tile streams
REF_EXPORT void REF_CAT(ref_dims_, REF_TAG)(uint32_t* d) {
    d[0] = kMt; d[1] = kKt; d[2] = kNt;
}
REF_EXPORT void REF_CAT(ref_matmul_, REF_TAG)(const uint16_t* a, const uint16_t* b, uint16_t* c) {
    std::vector<uint16_t> cv;
    matmul_reference(vec(a, size_t(kM) * kK), vec(b, size_t(kK) * kN), cv);
    out(cv, c);
}
REF_EXPORT void REF_CAT(ref_tile_a_, REF_TAG)(const uint16_t* a, uint16_t* t) {
    std::vector<uint16_t> o;
    tile_A_stream(vec(a, size_t(kM) * kK), o);
    out(o, t);
}
REF_EXPORT void REF_CAT(ref_tile_b_, REF_TAG)(const uint16_t* b, uint16_t* t) {
    std::vector<uint16_t> o;
    tile_B_stream(vec(b, size_t(kK) * kN), o);
    out(o, t);
}
REF_EXPORT void REF_CAT(ref_untile_c_, REF_TAG)(const uint16_t* t, uint16_t* c) {
    std::vector<uint16_t> o;
    untile_C_stream(vec(t, size_t(kM) * kN), o);
    out(o, c);
}
#elif REF_KIND == 2  // conv_3x3 (stride 1)
REF_EXPORT void REF_CAT(ref_dims_, REF_TAG)(uint32_t* d) {
    d[0] = kCin; d[1] = kH; d[2] = kW; d[3] = kCout;
}
REF_EXPORT void REF_CAT(ref_conv_, REF_TAG)(const uint16_t* x, const uint16_t* w, uint16_t* y) {
    std::vector<uint16_t> yv;
    conv3x3_reference(vec(x, size_t(kCin) * kH * kW), vec(w, size_t(kCout) * kCin * 9), yv);
    out(yv, y);
}
REF_EXPORT void REF_CAT(ref_im2col_, REF_TAG)(const uint16_t* x, uint16_t* a) {
    std::vector<uint16_t> av;
    im2col(vec(x, size_t(kCin) * kH * kW), av);
    out(av, a);
}
#elif REF_KIND == 3  // conv_3x3 stride 2
REF_EXPORT void REF_CAT(ref_dims_, REF_TAG)(uint32_t* d) {
    d[0] = kCin; d[1] = kHin; d[2] = kWin; d[3] = kCout;
}
REF_EXPORT void REF_CAT(ref_conv_, REF_TAG)(const uint16_t* x, const uint16_t* w, uint16_t* y) {
    std::vector<uint16_t> yv;
    conv3x3_s2_reference(vec(x, size_t(kCin) * kHin * kWin), vec(w, size_t(kCout) * kCin * 9), yv);
    out(yv, y);
}
REF_EXPORT void REF_CAT(ref_im2col_, REF_TAG)(const uint16_t* x, uint16_t* a) {
    std::vector<uint16_t> av;
    im2col_s2(vec(x, size_t(kCin) * kHin * kWin), av);
    out(av, a);
}
#elif REF_KIND == 4  // conv_1x1
REF_EXPORT void REF_CAT(ref_dims_, REF_TAG)(uint32_t* d) {
    d[0] = kCin; d[1] = kH; d[2] = kW; d[3] = kCout;
}
REF_EXPORT void REF_CAT(ref_conv_, REF_TAG)(const uint16_t* x, const uint16_t* w, uint16_t* y) {
    std::vector<uint16_t> yv;
    conv_1x1_reference(vec(x, size_t(kCin) * kH * kW), vec(w, size_t(kCout) * kCin), yv);
    out(yv, y);
}
#else
#error "REF_KIND must be 1..4"
#endif
