// train_gpu.cu — the training steps of train() on the device, bit-identical to
// their host restatements (train_cpu.cpp, which follows the reference's cpu/
// and jhq_gpu_index.cu):
//
//  * the residual codebook: 1-D k-means of the n*d residuals y - yhat
//    (cpu/codebook.cpp:8-58 via jhq_gpu_index.cu:302-330);
//  * the IVF Lloyd mean update (jhq_gpu_index.cu:259-297).
//
// Both accumulate per-cluster sums in double IN INDEX ORDER, and double
// addition is not associative, so a parallel reduction would change the
// rounding. Here the members of each cluster are first put in index order by a
// stable radix sort on the cluster label (CUB), then every sum is one thread's
// sequential fold over its members — the same chain of roundings as the
// reference's loop, run for all clusters (1-D) or all (cluster, dim) pairs
// (Lloyd) in parallel. The quantile seeds of the 1-D k-means are order
// statistics of the values, taken from a device radix sort (the same values
// std::sort gives, except that the sort puts -0.0 before +0.0 where the
// reference's order between the two is unspecified).
#include <cub/cub.cuh>

#include <algorithm>
#include <vector>

#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {
namespace {

__device__ __forceinline__ int nearest_sorted_dev(const float* c, int n, float v) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (v < 0.5f * (c[mid] + c[mid + 1])) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

// r = y - c1d[bits of the primary code] for every element (in place).
__global__ void residuals_kernel(float* __restrict__ y, const uint8_t* __restrict__ codes,
                                 int64_t n, int d, int M, int B, const float* __restrict__ c1d) {
    const int Ds = d / M, bpd = B / Ds, kmask = (1 << bpd) - 1;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * d) return;
    const int64_t i = t / d;
    const int j = (int)(t % d), m = j / Ds, k = j % Ds;
    const int idx = (codes[i * M + m] >> (k * bpd)) & kmask;
    y[t] = __fsub_rn(y[t], c1d[idx]);
}

__global__ void label_kernel(const float* __restrict__ v, int64_t n, const float* __restrict__ c_g,
                             int K, uint8_t* __restrict__ lab, unsigned long long* __restrict__ cnt) {
    __shared__ float c[256];
    __shared__ unsigned int h[256];
    for (int i = threadIdx.x; i < K; i += blockDim.x) { c[i] = c_g[i]; h[i] = 0; }
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int l = nearest_sorted_dev(c, K, v[i]);
        lab[i] = (uint8_t)l;
        atomicAdd(&h[l], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < K; i += blockDim.x)
        if (h[i]) atomicAdd(&cnt[i], (unsigned long long)h[i]);
}

// one warp per cluster: the index-order double fold of its members. The warp
// stages 256 values at a time in shared memory (coalesced loads, the next chunk
// in flight) and lane 0 adds them in order: the fold is bounded by the latency
// of the dependent double adds, not by memory.
constexpr int FOLD_CHUNK = 256;
__global__ void fold1d_kernel(const float* __restrict__ sorted, const int64_t* __restrict__ off,
                              int K, double* __restrict__ sum) {
    __shared__ float stage[8][2][FOLD_CHUNK];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int c = blockIdx.x * 8 + w;
    if (c >= K) return;
    const int64_t b = off[c], e = off[c + 1];
    double acc = 0.0;
    float v[FOLD_CHUNK / 32];
    auto load = [&](int64_t at) {
#pragma unroll
        for (int u = 0; u < FOLD_CHUNK / 32; ++u) {
            const int64_t i = at + u * 32 + lane;
            v[u] = i < e ? __ldg(sorted + i) : 0.0f;
        }
    };
    int buf = 0;
    if (b < e) load(b);
    for (int64_t at = b; at < e; at += FOLD_CHUNK) {
#pragma unroll
        for (int u = 0; u < FOLD_CHUNK / 32; ++u) stage[w][buf][u * 32 + lane] = v[u];
        __syncwarp();
        if (at + FOLD_CHUNK < e) load(at + FOLD_CHUNK);
        if (lane == 0) {
            const int cnt = (int)((e - at) < FOLD_CHUNK ? (e - at) : FOLD_CHUNK);
            for (int i = 0; i < cnt; ++i) acc = __dadd_rn(acc, (double)stage[w][buf][i]);
        }
        buf ^= 1;
        __syncwarp();
    }
    if (lane == 0) sum[c] = acc;
}

// thread per (cluster, dim): index-order double fold over the cluster's rows
// (member row ids sorted by cluster, stable), then the mean as the reference
// forms it: (float)(sum * (1.0 / count)); empty clusters are reseeded on the
// host (LCG rule) after the copy back.
__global__ void lloyd_fold_kernel(const float* __restrict__ y, int d,
                                  const int32_t* __restrict__ rows, const int64_t* __restrict__ off,
                                  int nl, float* __restrict__ cents) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)nl * d) return;
    const int c = (int)(t / d), j = (int)(t % d);
    const int64_t b = off[c], e = off[c + 1];
    if (e == b) return;
    double acc = 0.0;
    int64_t i = b;
    for (; i + 4 <= e; i += 4) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = __ldg(y + (int64_t)__ldg(rows + i + u) * d + j);
#pragma unroll
        for (int u = 0; u < 4; ++u) acc = __dadd_rn(acc, (double)v[u]);
    }
    for (; i < e; ++i) acc = __dadd_rn(acc, (double)__ldg(y + (int64_t)__ldg(rows + i) * d + j));
    const double inv = __ddiv_rn(1.0, (double)(e - b));
    cents[t] = (float)__dmul_rn(acc, inv);
}

__global__ void iota_kernel(int32_t* __restrict__ v, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = (int32_t)i;
}

int bits_for(int K) {
    int b = 1;
    while ((1 << b) < K) ++b;
    return b;
}

}  // namespace

void residuals_device(float* d_y, const uint8_t* d_codes, int64_t n, int d, int M, int B,
                      const float* d_c1d, cudaStream_t s) {
    const int64_t total = n * d;
    if (total <= 0) return;
    residuals_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(d_y, d_codes, n, d, M, B, d_c1d);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

std::vector<float> kmeans_1d_device(const float* d_vals, int64_t n64, int Kr, int max_iter,
                                    cudaStream_t s) {
    if (n64 <= 0 || Kr <= 0) return {};
    if (n64 > INT32_MAX) fail(JHQ_EINVAL, "kmeans_1d: more than 2^31-1 values");
    const int n = (int)n64;
    if (n < Kr) Kr = n;
    if (Kr > 256) fail(JHQ_EINVAL, "kmeans_1d: at most 256 centroids");
    // quantile seeds (cpu/codebook.cpp:13-20): order statistics of the values
    std::vector<float> quant(Kr);
    {
        DevBuf<float> sorted((size_t)n);
        size_t tmp = 0;
        JHQ_CUDA(cub::DeviceRadixSort::SortKeys(nullptr, tmp, d_vals, sorted.get(), n, 0, 32, s));
        DevBuf<unsigned char> work(std::max<size_t>(tmp, 1));
        JHQ_CUDA(cub::DeviceRadixSort::SortKeys(work.get(), tmp, d_vals, sorted.get(), n, 0, 32, s));
        count_launch();
        for (int i = 0; i < Kr; ++i) {
            const int idx = std::min((int)((i + 0.5f) / Kr * n), n - 1);
            JHQ_CUDA(cudaMemcpyAsync(&quant[i], sorted.get() + idx, 4, cudaMemcpyDeviceToHost, s));
        }
        JHQ_CUDA(cudaStreamSynchronize(s));
    }
    std::vector<float> c(quant);
    DevBuf<float> dc(256), vals_sorted((size_t)n);
    DevBuf<uint8_t> lab((size_t)n), lab_sorted((size_t)n);
    DevBuf<unsigned long long> dcnt((size_t)Kr);
    DevBuf<int64_t> doff((size_t)Kr + 1);
    DevBuf<double> dsum((size_t)Kr);
    const int bits = bits_for(Kr);
    size_t tmp = 0;
    JHQ_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, lab.get(), lab_sorted.get(), d_vals,
                                             vals_sorted.get(), n, 0, bits, s));
    DevBuf<unsigned char> work(std::max<size_t>(tmp, 1));
    std::vector<unsigned long long> cnt(Kr);
    std::vector<int64_t> off(Kr + 1);
    std::vector<double> sum(Kr);
    int dev = 0, sms = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    for (int iter = 0; iter < max_iter; ++iter) {
        JHQ_CUDA(cudaMemcpyAsync(dc.get(), c.data(), (size_t)Kr * 4, cudaMemcpyHostToDevice, s));
        JHQ_CUDA(cudaMemsetAsync(dcnt.get(), 0, (size_t)Kr * 8, s));
        label_kernel<<<sms * 8, 256, 0, s>>>(d_vals, n, dc.get(), Kr, lab.get(), dcnt.get());
        JHQ_LAUNCH_CHECK();
        count_launch();
        JHQ_CUDA(cub::DeviceRadixSort::SortPairs(work.get(), tmp, lab.get(), lab_sorted.get(),
                                                 d_vals, vals_sorted.get(), n, 0, bits, s));
        count_launch();
        JHQ_CUDA(cudaMemcpyAsync(cnt.data(), dcnt.get(), (size_t)Kr * 8, cudaMemcpyDeviceToHost, s));
        JHQ_CUDA(cudaStreamSynchronize(s));
        off[0] = 0;
        for (int i = 0; i < Kr; ++i) off[i + 1] = off[i] + (int64_t)cnt[i];
        JHQ_CUDA(cudaMemcpyAsync(doff.get(), off.data(), (size_t)(Kr + 1) * 8, cudaMemcpyHostToDevice, s));
        fold1d_kernel<<<(unsigned)ceil_div(Kr, 8), 256, 0, s>>>(vals_sorted.get(), doff.get(), Kr,
                                                                dsum.get());
        JHQ_LAUNCH_CHECK();
        count_launch();
        JHQ_CUDA(cudaMemcpyAsync(sum.data(), dsum.get(), (size_t)Kr * 8, cudaMemcpyDeviceToHost, s));
        JHQ_CUDA(cudaStreamSynchronize(s));
        // update (cpu/codebook.cpp:39-54)
        bool changed = false;
        for (int i = 0; i < Kr; ++i) {
            const float nc = cnt[i] == 0 ? quant[i] : (float)(sum[i] / (double)(int)cnt[i]);
            if (nc != c[i]) { c[i] = nc; changed = true; }
        }
        std::sort(c.begin(), c.end());
        if (!changed) break;
    }
    return c;
}

void lloyd_update_device(const float* d_y, int64_t n, int d, int nl, const int32_t* d_assign,
                         float* d_cents, std::vector<int64_t>& counts, cudaStream_t s) {
    if (n > INT32_MAX) fail(JHQ_EINVAL, "lloyd: more than 2^31-1 rows");
    const int ni = (int)n;
    DevBuf<int32_t> rows((size_t)n), rows_sorted((size_t)n), keys_sorted((size_t)n);
    iota_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(rows.get(), n);
    JHQ_LAUNCH_CHECK();
    count_launch();
    const int bits = bits_for(std::max(nl, 2));
    size_t tmp = 0;
    JHQ_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, d_assign, keys_sorted.get(), rows.get(),
                                             rows_sorted.get(), ni, 0, bits, s));
    DevBuf<unsigned char> work(std::max<size_t>(tmp, 1));
    JHQ_CUDA(cub::DeviceRadixSort::SortPairs(work.get(), tmp, d_assign, keys_sorted.get(), rows.get(),
                                             rows_sorted.get(), ni, 0, bits, s));
    count_launch();
    // counts / offsets from the sorted keys on the host (nl + 1 values)
    std::vector<int32_t> ks((size_t)n);
    JHQ_CUDA(cudaMemcpyAsync(ks.data(), keys_sorted.get(), (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    JHQ_CUDA(cudaStreamSynchronize(s));
    counts.assign(nl, 0);
    for (int32_t k : ks) {
        if (k < 0 || k >= nl) fail(JHQ_EDEVICE, "lloyd: invalid assignment");
        counts[k]++;
    }
    std::vector<int64_t> off(nl + 1, 0);
    for (int c = 0; c < nl; ++c) off[c + 1] = off[c] + counts[c];
    DevBuf<int64_t> doff((size_t)nl + 1);
    JHQ_CUDA(cudaMemcpyAsync(doff.get(), off.data(), (size_t)(nl + 1) * 8, cudaMemcpyHostToDevice, s));
    const int64_t total = (int64_t)nl * d;
    lloyd_fold_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(d_y, d, rows_sorted.get(),
                                                                      doff.get(), nl, d_cents);
    JHQ_LAUNCH_CHECK();
    count_launch();
    JHQ_CUDA(cudaStreamSynchronize(s));
}

}  // namespace jhq
