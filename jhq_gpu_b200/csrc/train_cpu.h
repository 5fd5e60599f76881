// train_cpu.h — host-side training steps of JHQ.
//
// These restate the reference's CPU trainer (cpu/jl_transform.cpp,
// cpu/codebook.cpp, cpu/erfinv.h) step for step; sigma, the Lloyd-Max
// codewords, the 1-D k-means and reconstruct reproduce the reference
// bit for bit. The QR rotation follows the same Householder convention as
// LAPACK sgeqrf/sorgqr (R diagonal = -sign(alpha)*norm) evaluated in double,
// so Pi equals the reference's to rounding, not bit for bit; import the
// reference's Pi through jhq_set_trained when identical training is needed.
#pragma once
#include <cstdint>
#include <vector>

namespace jhq::train {

// cpu/jl_transform.cpp:73-83
float estimate_sigma(const float* x, int64_t n, int d);
// cpu/erfinv.h:7-27
float erfinv_f(float x);
// cpu/codebook.cpp:60-80 — K1D analytical codewords, ascending.
std::vector<float> lloyd_max_c1d(float sigma, int K1D);
// cpu/codebook.cpp:8-58
std::vector<float> kmeans_1d(const float* vals, int64_t n, int Kr, int max_iter = 25);
// cpu/jl_transform.cpp:25-56 — d*d column-major orthogonal matrix.
std::vector<float> build_rotation(int d, int seed);
// cpu/codebook.cpp:161-171 — rows of codes -> yhat.
void reconstruct(const uint8_t* codes, int64_t n, int d, int M, int B,
                 const float* c1d, float* out);

}  // namespace jhq::train
