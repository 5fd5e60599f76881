// Test infrastructure (oracle/_ref only): a C-ABI shim over the reference's
// own CPU trainer (cpu/codebook.cpp, cpu/jl_transform.cpp, compiled from the
// reference tree by oracle/Makefile). Tests and golden-vector generation call
// these through ctypes to pin the oracle and the product's training against
// the reference implementation. Nothing in the product links this.
#include "cpu/codebook.h"
#include "cpu/jl_transform.h"
#include <cstring>
#include <exception>
#include <vector>

extern "C" {

// JLTransform ctor + pi_data(): cpu/jl_transform.cpp:21-56
int ref_rotation(int d, int seed, float* pi_out) {
    try {
        JLTransform jl(d, seed);
        std::memcpy(pi_out, jl.pi_data(), sizeof(float) * (size_t)d * d);
        return 0;
    } catch (const std::exception&) { return 1; }
}

// JLTransform::apply: cpu/jl_transform.cpp:58-70 (cblas_sgemm)
int ref_apply(int d, int seed, const float* x, int n, float* y) {
    try { JLTransform jl(d, seed); jl.apply(x, y, n); return 0; }
    catch (const std::exception&) { return 1; }
}

// JLTransform::estimate_sigma: cpu/jl_transform.cpp:73-83
float ref_sigma(const float* x, int n, int d) {
    JLTransform jl(1, 42);  // rotation of a 1x1 matrix is irrelevant here
    // estimate_sigma reads d_ from the object; build one with the right d.
    JLTransform jd(d, 42);
    jd.estimate_sigma(x, n);
    (void)jl;
    return jd.sigma();
}

// LloydMaxCodebook ctor: cpu/codebook.cpp:60-80
int ref_c1d(int d, int M, int B, float sigma, float* out) {
    try {
        LloydMaxCodebook cb(d, M, B, sigma);
        std::memcpy(out, cb.c1d().data(), sizeof(float) * cb.K1D());
        return cb.K1D();
    } catch (const std::exception&) { return -1; }
}

// LloydMaxCodebook::encode: cpu/codebook.cpp:96-110
int ref_encode(int d, int M, int B, float sigma, const float* y, int n, unsigned char* codes) {
    try { LloydMaxCodebook cb(d, M, B, sigma); cb.encode(y, codes, n); return 0; }
    catch (const std::exception&) { return 1; }
}

// LloydMaxCodebook::build_flat_lut: cpu/codebook.cpp:112-129
int ref_flat_lut(int d, int M, int B, float sigma, const float* q_rot, float* out) {
    try { LloydMaxCodebook cb(d, M, B, sigma); cb.build_flat_lut(q_rot, out); return 0; }
    catch (const std::exception&) { return 1; }
}

// LloydMaxCodebook::build_lut + adc_distance: cpu/codebook.cpp:131-159
int ref_adc(int d, int M, int B, float sigma, const float* q_rot,
            const unsigned char* codes, int n, float* out) {
    try {
        LloydMaxCodebook cb(d, M, B, sigma);
        std::vector<float> lut((size_t)M * cb.Ds() * cb.K1D());
        cb.build_lut(q_rot, lut.data());
        for (int i = 0; i < n; ++i) out[i] = cb.adc_distance(codes + (size_t)i * M, lut.data());
        return 0;
    } catch (const std::exception&) { return 1; }
}

// LloydMaxCodebook::reconstruct: cpu/codebook.cpp:161-171
int ref_reconstruct(int d, int M, int B, float sigma, const unsigned char* codes, int n, float* out) {
    try {
        LloydMaxCodebook cb(d, M, B, sigma);
        for (int i = 0; i < n; ++i) cb.reconstruct(codes + (size_t)i * M, out + (size_t)i * d);
        return 0;
    } catch (const std::exception&) { return 1; }
}

// train_1d_kmeans: cpu/codebook.cpp:8-58
int ref_kmeans1d(const float* vals, int n, int Kr, int max_iter, float* out) {
    std::vector<float> c = train_1d_kmeans(vals, n, Kr, max_iter);
    std::memcpy(out, c.data(), sizeof(float) * c.size());
    return (int)c.size();
}

}  // extern "C"
