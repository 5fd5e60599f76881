// train_cpu.cpp — host-side training steps (see train_cpu.h).
// Compiled with -ffp-contract=off: no multiply-add is fused behind our back,
// which keeps sigma / c1d / 1-D k-means identical to the reference's cpu/.
#include "train_cpu.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <random>
#include <thread>

namespace jhq::train {

float estimate_sigma(const float* x, int64_t n, int d) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const float* xi = x + i * d;
        for (int j = 0; j < d; ++j) s += (double)xi[j] * xi[j];
    }
    return (float)std::sqrt(s / ((double)n * d));
}

float erfinv_f(float x) {
    // Winitzki (2008), a = 0.147, then one Newton step on erf(z) - x.
    if (x >= 1.0f) return std::numeric_limits<float>::infinity();
    if (x <= -1.0f) return -std::numeric_limits<float>::infinity();
    if (x == 0.0f) return 0.0f;
    const float sign = (x > 0.0f) ? 1.0f : -1.0f;
    const float a = std::fabs(x);
    const float kC = 0.147f;
    const float k2Pi = 2.0f / 3.14159265358979f;
    const float ln1 = std::log(1.0f - a * a);
    const float t = k2Pi / kC + 0.5f * ln1;
    float z = sign * std::sqrt(std::sqrt(t * t - ln1 / kC) - t);
    const float err = std::erf(z) - x;
    const float der = (2.0f / std::sqrt(float(M_PI))) * std::exp(-z * z);
    z -= err / der;
    return z;
}

std::vector<float> lloyd_max_c1d(float sigma, int K1D) {
    std::vector<float> c(K1D);
    for (int i = 0; i < K1D; ++i) {
        float q = (i + 0.5f) / (float)K1D;
        c[i] = sigma * float(M_SQRT2) * erfinv_f(2.0f * q - 1.0f);
    }
    return c;
}

static inline int nearest_sorted(const float* c, int n, float v) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = (lo + hi) / 2;
        if (v < 0.5f * (c[mid] + c[mid + 1])) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

std::vector<float> kmeans_1d(const float* vals, int64_t n64, int Kr, int max_iter) {
    // Same result as a sequential run of cpu/codebook.cpp:8-58, faster:
    //  - the quantile seeds are order statistics, found with nth_element instead
    //    of a full sort (the values are identical);
    //  - the assignment (pure function of the value) runs on all host threads;
    //  - the double sums are still accumulated in index order, one pass, so every
    //    rounding step is the reference's.
    int n = (int)n64;
    if (n <= 0 || Kr <= 0) return {};
    if (n < Kr) Kr = n;
    std::vector<int> qpos(Kr);
    for (int i = 0; i < Kr; ++i) qpos[i] = std::min((int)((i + 0.5f) / Kr * n), n - 1);
    std::vector<float> quant(Kr);
    {
        std::vector<float> work(vals, vals + n);
        std::vector<int> order(Kr);
        for (int i = 0; i < Kr; ++i) order[i] = i;
        std::sort(order.begin(), order.end(), [&](int a, int b) { return qpos[a] < qpos[b]; });
        int lo = 0;
        for (int oi : order) {
            int p = qpos[oi];
            if (p >= lo) {
                std::nth_element(work.begin() + lo, work.begin() + p, work.end());
                lo = p + 1;
                quant[oi] = work[p];
            } else {
                quant[oi] = work[p];       // repeated position: already in place
            }
        }
    }
    std::vector<float> c(quant);
    std::vector<double> sum(Kr);
    std::vector<int> cnt(Kr);
    std::vector<uint8_t> lab((size_t)n);
    unsigned nth = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
    for (int iter = 0; iter < max_iter; ++iter) {
        std::vector<std::thread> pool;
        const int64_t chunk = ((int64_t)n + nth - 1) / nth;
        for (unsigned t = 0; t < nth; ++t) {
            pool.emplace_back([&, t] {
                int64_t a = t * chunk, b = std::min<int64_t>(n, a + chunk);
                for (int64_t i = a; i < b; ++i) lab[i] = (uint8_t)nearest_sorted(c.data(), Kr, vals[i]);
            });
        }
        for (auto& th : pool) th.join();
        std::fill(sum.begin(), sum.end(), 0.0);
        std::fill(cnt.begin(), cnt.end(), 0);
        for (int i = 0; i < n; ++i) {
            sum[lab[i]] += vals[i];
            cnt[lab[i]]++;
        }
        bool changed = false;
        for (int i = 0; i < Kr; ++i) {
            float nc = cnt[i] == 0 ? quant[i] : (float)(sum[i] / cnt[i]);
            if (nc != c[i]) { c[i] = nc; changed = true; }
        }
        std::sort(c.begin(), c.end());
        if (!changed) break;
    }
    return c;
}

std::vector<float> build_rotation(int d, int seed) {
    // Gaussian matrix filled in column-major memory order, exactly as the
    // reference fills Pi_ (cpu/jl_transform.cpp:27-29).
    std::mt19937 rng(seed);
    std::normal_distribution<float> norm(0.0f, 1.0f);
    std::vector<float> g((size_t)d * d);
    for (float& v : g) v = norm(rng);

    // Householder QR in double: A = Q R with H_j = I - tau v v^T, v_0 = 1,
    // beta = -sign(alpha) * |x| (the LAPACK xLARFG convention).
    std::vector<double> A((size_t)d * d);           // column-major
    for (size_t i = 0; i < A.size(); ++i) A[i] = g[i];
    std::vector<double> tau(d, 0.0);
    auto at = [&](int r, int c) -> double& { return A[(size_t)c * d + r]; };
    for (int j = 0; j < d; ++j) {
        double alpha = at(j, j), xn2 = 0.0;
        for (int r = j + 1; r < d; ++r) xn2 += at(r, j) * at(r, j);
        if (xn2 == 0.0) { tau[j] = 0.0; continue; }
        double beta = -std::copysign(std::sqrt(alpha * alpha + xn2), alpha);
        tau[j] = (beta - alpha) / beta;
        double scale = 1.0 / (alpha - beta);
        for (int r = j + 1; r < d; ++r) at(r, j) *= scale;
        at(j, j) = beta;
        for (int c = j + 1; c < d; ++c) {             // apply H_j to A[j:, c]
            double w = at(j, c);
            for (int r = j + 1; r < d; ++r) w += at(r, j) * at(r, c);
            w *= tau[j];
            at(j, c) -= w;
            for (int r = j + 1; r < d; ++r) at(r, c) -= w * at(r, j);
        }
    }
    // Q = H_0 H_1 ... H_{d-1}, accumulated backwards on the identity.
    std::vector<double> Q((size_t)d * d, 0.0);
    auto q = [&](int r, int c) -> double& { return Q[(size_t)c * d + r]; };
    for (int i = 0; i < d; ++i) q(i, i) = 1.0;
    for (int j = d - 1; j >= 0; --j) {
        if (tau[j] == 0.0) continue;
        for (int c = j; c < d; ++c) {
            double w = q(j, c);
            for (int r = j + 1; r < d; ++r) w += at(r, j) * q(r, c);
            w *= tau[j];
            q(j, c) -= w;
            for (int r = j + 1; r < d; ++r) q(r, c) -= w * at(r, j);
        }
    }
    std::vector<float> P((size_t)d * d);
    for (size_t i = 0; i < P.size(); ++i) P[i] = (float)Q[i];
    return P;
}

void reconstruct(const uint8_t* codes, int64_t n, int d, int M, int B,
                 const float* c1d, float* out) {
    const int Ds = d / M, bpd = B / Ds, mask = (1 << bpd) - 1;
    for (int64_t i = 0; i < n; ++i)
        for (int m = 0; m < M; ++m) {
            uint8_t cm = codes[i * M + m];
            for (int k = 0; k < Ds; ++k)
                out[i * d + m * Ds + k] = c1d[(cm >> (k * bpd)) & mask];
        }
}

}  // namespace jhq::train
