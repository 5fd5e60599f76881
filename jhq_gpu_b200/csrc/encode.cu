// encode.cu — database-side kernels of add(): primary + residual encode
// and the scatter of primary codes into the page layout.
//
// encode_kernel restates primary_encode_kernel + residual_encode_kernel
// (jhq_v14_streaming_add/encode.cu:20-86) as one pass over each rotated row:
//   code_m  = OR_k nearest(c1d, y[m*Ds+k]) << (k*bpd)        (midpoint search,
//             ties to the upper codeword, encode.cu:6-18)
//   r_j     = y_j - c1d[bits of code], ri = nearest(res_c1d, r_j)
//   Br = 4 -> dim j in the low nibble of byte j/2 when j is even (encode.cu:74-78)
//   corr    = 2 * (in-order fma chain of yhat_j * rhat_j)     (encode.cu:85)
// With per-subspace residual codebooks, dim j is coded against codebook j / Ds.
// One thread per row, rows stream from L2; this runs at add() time only.
#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {
namespace {

__device__ __forceinline__ int nearest_sorted(const float* c, int n, float v) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (v < 0.5f * (c[mid] + c[mid + 1])) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

__global__ void encode_kernel(const float* __restrict__ y, int64_t n, int d, int M, int B, int Br,
                              const float* __restrict__ c1d_g, const float* __restrict__ res_g,
                              int res_per_sub, uint8_t* __restrict__ pcodes,
                              uint8_t* __restrict__ rcodes, int bpv_pad, float* __restrict__ corr) {
    __shared__ float c1d[256];
    __shared__ float rc1d[256];
    const int Ds = d / M, bpd = B / Ds, K1D = 1 << bpd, kmask = K1D - 1, Kr = 1 << Br;
    for (int i = threadIdx.x; i < K1D; i += blockDim.x) c1d[i] = c1d_g[i];
    if (res_g && !res_per_sub)
        for (int i = threadIdx.x; i < Kr; i += blockDim.x) rc1d[i] = res_g[i];
    __syncthreads();
    const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n) return;
    const float* yv = y + v * d;
    uint8_t* rc = rcodes + v * bpv_pad;
    float dot = 0.0f;
    unsigned cur = 0;
    for (int m = 0; m < M; ++m) {
        unsigned code = 0;
        for (int k = 0; k < Ds; ++k)
            code |= (unsigned)nearest_sorted(c1d, K1D, yv[m * Ds + k]) << (k * bpd);
        pcodes[v * M + m] = (uint8_t)code;
        if (rcodes == nullptr) continue;                 // primary codes only (train)
        // the subspace's own residual codebook (per-subspace mode, read through
        // L1) or the global one in shared memory
        const float* rcb = res_per_sub ? res_g + (size_t)m * Kr : rc1d;
        for (int k = 0; k < Ds; ++k) {
            const int j = m * Ds + k;
            const float yh = c1d[(code >> (k * bpd)) & kmask];
            const float r = yv[j] - yh;
            const int ri = nearest_sorted(rcb, Kr, r);
            if (Br == 4) {
                if ((j & 1) == 0) cur = (unsigned)ri;
                else { rc[j >> 1] = (uint8_t)(cur | ((unsigned)ri << 4)); cur = 0; }
            } else {
                rc[j] = (uint8_t)ri;
            }
            dot = __fmaf_rn(yh, rcb[ri], dot);
        }
    }
    if (rcodes == nullptr) return;
    int written = (Br == 4) ? d / 2 : d;
    if (Br == 4 && (d & 1)) rc[written++] = (uint8_t)cur;
    for (int b = written; b < bpv_pad; ++b) rc[b] = 0;
    corr[v] = 2.0f * dot;
}

// Thread per (slot, 16-byte group): pages[p][g][lane][0..15].
__global__ void scatter_pages_kernel(const int32_t* __restrict__ slot_ids, int64_t nslots,
                                     const uint8_t* __restrict__ pcodes, int M, int Mp,
                                     uint8_t* __restrict__ pages) {
    const int G = Mp / 16;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nslots * G) return;
    const int64_t slot = t / G;
    const int g = (int)(t % G);
    const int32_t v = slot_ids[slot];
    uint32_t w[4] = {0, 0, 0, 0};
    if (v >= 0) {
        const uint8_t* src = pcodes + (int64_t)v * M;
#pragma unroll
        for (int b = 0; b < 16; ++b) {
            int m = g * 16 + b;
            uint32_t byte = (m < M) ? src[m] : 0u;
            w[b >> 2] |= byte << ((b & 3) * 8);
        }
    }
    const int64_t page = slot / 32;
    const int lane = (int)(slot % 32);
    uint4* dst = reinterpret_cast<uint4*>(pages + ((page * G + g) * 32 + lane) * 16);
    *dst = make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void set_int_kernel(int* dst, int value) { *dst = value; }

__global__ void popcount_kernel(const uint8_t* __restrict__ codes, int64_t n, int M,
                                int32_t* __restrict__ pop) {
    const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= n) return;
    int c = 0;
    for (int m = 0; m < M; ++m) c += __popc((unsigned)codes[v * M + m]);
    pop[v] = c;
}

__global__ void scale_kernel(float* __restrict__ v, int64_t n, float f) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = __fmul_rn(v[i], f);
}

}  // namespace

void set_int(int* dst, int value, cudaStream_t s) {
    set_int_kernel<<<1, 1, 0, s>>>(dst, value);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void popcount_rows(const uint8_t* codes, int64_t n, int M, int32_t* pop, cudaStream_t s) {
    if (n <= 0) return;
    popcount_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(codes, n, M, pop);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void scale_floats(float* v, int64_t n, float f, cudaStream_t s) {
    if (n <= 0) return;
    scale_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(v, n, f);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void encode_rows(const float* y, int64_t n, int d, int M, int B, int Br,
                 const float* c1d, const float* res_c1d, bool res_per_sub, uint8_t* pcodes,
                 uint8_t* rcodes, int bpv_pad, float* corr, cudaStream_t s) {
    if (n <= 0) return;
    encode_kernel<<<(unsigned)ceil_div(n, 128), 128, 0, s>>>(y, n, d, M, B, Br, c1d, res_c1d,
                                                             res_per_sub ? 1 : 0, pcodes, rcodes,
                                                             bpv_pad, corr);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void scatter_pages(const int32_t* slot_ids, int64_t nslots, const uint8_t* pcodes,
                   int M, int Mp, uint8_t* pages, cudaStream_t s) {
    if (nslots <= 0) return;
    int64_t total = nslots * (Mp / 16);
    scatter_pages_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(slot_ids, nslots, pcodes,
                                                                        M, Mp, pages);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq
