// gemm.cu — fp32 row products for the JL rotation (y = Pi x, reference
// cuBLAS SGEMM at jhq_gpu_index.cu:209-225/:444-448 and search.cu:338-339)
// and the IVF coarse scores s = |c|^2 - 2 <q, c> (search.cu:341-342 + :32,
// jhq_gpu_index.cu:378-387 + :23-39).
//
// Every output is one in-order fused multiply-add chain over k starting at 0,
// so results are deterministic and equal bit for bit to the oracle's
// (oracle/jhq_oracle.c: oracle_rotate / dot_chain). Two tilings:
//  - gemm_tiled_kernel : 128x128 CTA tile, 8x8 outputs per thread, for tall
//                        operands (add-time rotation, k-means assignment);
//  - gemm_skinny_kernel: 8 rows x 128 columns per CTA, rows staged in shared
//                        memory, B streamed coalesced — for query batches,
//                        where a 128-row tile would leave most SMs idle.
// The product is tiny next to the ADC scan at the flat and IVF configs
// (C1: 64x1024x1024 per batch); it is not on tensor cores because the
// codes must stay bit-exact with the fp32 fma-chain rotation.
#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {

std::atomic<int64_t> g_kernel_launches{0};

namespace {

constexpr int TBM = 128, TBN = 128, TBK = 8;

template <int EPI>
__device__ __forceinline__ float epilogue(float acc, const float* norms, int n) {
    if (EPI == EPI_COARSE) return norms[n] - 2.0f * acc;
    return acc;
}

template <int EPI>
__global__ void __launch_bounds__(256)
gemm_tiled_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                  int64_t R, int K, int N, const float* __restrict__ norms) {
    __shared__ float As[TBK][TBM + 4];
    __shared__ float Bs[TBK][TBN + 4];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int64_t r0 = (int64_t)blockIdx.y * TBM;
    const int n0 = blockIdx.x * TBN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    for (int k0 = 0; k0 < K; k0 += TBK) {
        // A tile: 128 rows x 8 k (4 per thread)
        {
            int r = tid / 2, kq = (tid % 2) * 4;
            int64_t gr = r0 + r;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                int gk = k0 + kq + t;
                As[kq + t][r] = (gr < R && gk < K) ? A[gr * K + gk] : 0.0f;
            }
        }
        // B tile: 8 k x 128 n (4 per thread)
        {
            int kr = tid / 32, nq = (tid % 32) * 4;
            int gk = k0 + kr;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                int gn = n0 + nq + t;
                Bs[kr][nq + t] = (gk < K && gn < N) ? B[(int64_t)gk * N + gn] : 0.0f;
            }
        }
        __syncthreads();
        const int kmax = min(TBK, K - k0);
        if (kmax == TBK) {
#pragma unroll
            for (int kk = 0; kk < TBK; ++kk) {
                float a[8], b[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) a[i] = As[kk][ty * 8 + i];
#pragma unroll
                for (int j = 0; j < 8; ++j) b[j] = Bs[kk][tx * 8 + j];
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
            }
        } else {
            for (int kk = 0; kk < kmax; ++kk) {
                float a[8], b[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) a[i] = As[kk][ty * 8 + i];
#pragma unroll
                for (int j = 0; j < 8; ++j) b[j] = Bs[kk][tx * 8 + j];
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int64_t gr = r0 + ty * 8 + i;
        if (gr >= R) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            int gn = n0 + tx * 8 + j;
            if (gn < N) C[gr * N + gn] = epilogue<EPI>(acc[i][j], norms, gn);
        }
    }
}

constexpr int SK_ROWS = 8, SK_COLS = 128, SK_KC = 512;

template <int EPI>
__global__ void __launch_bounds__(SK_COLS)
gemm_skinny_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                   int64_t R, int K, int N, const float* __restrict__ norms) {
    __shared__ float As[SK_ROWS][SK_KC];
    const int64_t r0 = (int64_t)blockIdx.y * SK_ROWS;
    const int n = blockIdx.x * SK_COLS + threadIdx.x;
    float acc[SK_ROWS];
#pragma unroll
    for (int r = 0; r < SK_ROWS; ++r) acc[r] = 0.0f;
    for (int kc = 0; kc < K; kc += SK_KC) {
        const int kl = min(SK_KC, K - kc);
        for (int i = threadIdx.x; i < SK_ROWS * SK_KC; i += SK_COLS) {
            int r = i / SK_KC, k = i % SK_KC;
            int64_t gr = r0 + r;
            As[r][k] = (gr < R && k < kl) ? A[gr * K + kc + k] : 0.0f;
        }
        __syncthreads();
        if (n < N) {
            const float* bp = B + (int64_t)kc * N + n;
            int k = 0;
            for (; k + 4 <= kl; k += 4) {
                float b0 = __ldg(bp + (int64_t)(k + 0) * N);
                float b1 = __ldg(bp + (int64_t)(k + 1) * N);
                float b2 = __ldg(bp + (int64_t)(k + 2) * N);
                float b3 = __ldg(bp + (int64_t)(k + 3) * N);
#pragma unroll
                for (int r = 0; r < SK_ROWS; ++r) {
                    float4 a = *reinterpret_cast<const float4*>(&As[r][k]);
                    acc[r] = __fmaf_rn(a.x, b0, acc[r]);
                    acc[r] = __fmaf_rn(a.y, b1, acc[r]);
                    acc[r] = __fmaf_rn(a.z, b2, acc[r]);
                    acc[r] = __fmaf_rn(a.w, b3, acc[r]);
                }
            }
            for (; k < kl; ++k) {
                float b = __ldg(bp + (int64_t)k * N);
#pragma unroll
                for (int r = 0; r < SK_ROWS; ++r) acc[r] = __fmaf_rn(As[r][k], b, acc[r]);
            }
        }
        __syncthreads();
    }
    if (n < N) {
#pragma unroll
        for (int r = 0; r < SK_ROWS; ++r) {
            int64_t gr = r0 + r;
            if (gr < R) C[gr * N + n] = epilogue<EPI>(acc[r], norms, n);
        }
    }
}

}  // namespace

void gemm_rows(const float* A, const float* B, float* C, int64_t R, int K, int N,
               GemmEpi epi, const float* norms, cudaStream_t s) {
    if (R <= 0 || N <= 0) return;
    if (R <= 1024) {
        dim3 grid((unsigned)ceil_div(N, SK_COLS), (unsigned)ceil_div(R, SK_ROWS));
        if (epi == EPI_COARSE)
            gemm_skinny_kernel<EPI_COARSE><<<grid, SK_COLS, 0, s>>>(A, B, C, R, K, N, norms);
        else
            gemm_skinny_kernel<EPI_STORE><<<grid, SK_COLS, 0, s>>>(A, B, C, R, K, N, norms);
    } else {
        dim3 grid((unsigned)ceil_div(N, TBN), (unsigned)ceil_div(R, TBM));
        if (grid.y > 65535) fail(JHQ_EINVAL, "gemm_rows: too many rows in one call");
        if (epi == EPI_COARSE)
            gemm_tiled_kernel<EPI_COARSE><<<grid, 256, 0, s>>>(A, B, C, R, K, N, norms);
        else
            gemm_tiled_kernel<EPI_STORE><<<grid, 256, 0, s>>>(A, B, C, R, K, N, norms);
    }
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq
