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
//  - gemm_skinny_kernel: 16 rows x 64 columns per CTA, both operands staged
//                        through shared memory by double-buffered cp.async —
//                        for query batches, where a 128-row tile would leave
//                        most SMs idle.
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

// Fused assignment: argmin_n (norms[n] - 2 <A_r, B[:, n]>) over all N columns
// without materialising the scores (assign_from_dots_kernel semantics,
// jhq_gpu_index.cu:23-39: strict <, lowest column wins ties). CTA = 128 rows;
// it sweeps the columns in 128-wide tiles with the same 8x8-per-thread fma
// chains as gemm_tiled_kernel, keeps a running (best, index) per thread-row,
// then reduces the 16 threads that share a row.
__global__ void __launch_bounds__(256)
gemm_argmin_kernel(const float* __restrict__ A, const float* __restrict__ B,
                   const float* __restrict__ norms, int64_t R, int K, int N,
                   int32_t* __restrict__ out) {
    __shared__ float As[TBK][TBM + 4];
    __shared__ float Bs[TBK][TBN + 4];
    __shared__ float red_v[TBM][17];
    __shared__ int red_i[TBM][17];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int64_t r0 = (int64_t)blockIdx.x * TBM;
    float best[8];
    int bidx[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { best[i] = __int_as_float(0x7f800000); bidx[i] = 0x7fffffff; }
    for (int n0 = 0; n0 < N; n0 += TBN) {
        float acc[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
        for (int k0 = 0; k0 < K; k0 += TBK) {
            {
                int r = tid / 2, kq = (tid % 2) * 4;
                int64_t gr = r0 + r;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    int gk = k0 + kq + t;
                    As[kq + t][r] = (gr < R && gk < K) ? A[gr * K + gk] : 0.0f;
                }
            }
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
            __syncthreads();
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {            // columns ascending within the thread
            const int gn = n0 + tx * 8 + j;
            if (gn >= N) break;
            const float nb = norms[gn];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float sc = nb - 2.0f * acc[i][j];
                if (sc < best[i]) { best[i] = sc; bidx[i] = gn; }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) { red_v[ty * 8 + i][tx] = best[i]; red_i[ty * 8 + i][tx] = bidx[i]; }
    __syncthreads();
    if (tid < TBM) {
        const int64_t gr = r0 + tid;
        float bv = red_v[tid][0];
        int bi = red_i[tid][0];
        for (int t = 1; t < 16; ++t) {
            const float v = red_v[tid][t];
            const int ix = red_i[tid][t];
            if (v < bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
        }
        if (gr < R) out[gr] = bi == 0x7fffffff ? 0 : bi;
    }
}

// Skinny path: CTA = SK_ROWS rows x SK_BN columns, 256 threads; thread
// (column c, row group r) owns rows r*SK_TR .. r*SK_TR+SK_TR-1 of column c:
// SK_TR (1 or 4) independent chains. Chunks of SK_KC rows of B (and the matching
// SK_ROWS x SK_KC slice of A) are staged in shared memory by cp.async in a
// ring of SK_STAGES buffers: a chunk computes in less time than an L2 round
// trip, so SK_STAGES - 1 chunks are kept in flight. 16 rows per CTA keep the L2 re-reads of B (the d x d
// rotation) at a quarter of a 4-row tiling.
constexpr int SK_RG = 4, SK_BN = 64, SK_KC = 64, SK_STAGES = 6;
constexpr int SK_THREADS = SK_BN * SK_RG;
template <int SK_TR>
constexpr int sk_smem_bytes() { return SK_STAGES * (SK_KC * SK_BN + SK_TR * SK_RG * SK_KC) * 4; }

__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool ok) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    const int n = ok ? 4 : 0;                        // 0 -> zero fill, no read
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" :: "r"(d), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async16(float* dst, const float* src, int bytes) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" :: "r"(d), "l"(src), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" :: "n"(N)); }

template <int EPI, int SK_TR>
__global__ void __launch_bounds__(SK_THREADS)
gemm_skinny_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                   int64_t R, int K, int N, const float* __restrict__ norms, int vec16) {
    constexpr int SK_ROWS = SK_TR * SK_RG;
    extern __shared__ __align__(16) float sk_smem[];
    auto Bs = reinterpret_cast<float (*)[SK_KC][SK_BN]>(sk_smem);
    auto As = reinterpret_cast<float (*)[SK_ROWS][SK_KC]>(sk_smem + SK_STAGES * SK_KC * SK_BN);
    const int tid = threadIdx.x, col = tid % SK_BN, rg = tid / SK_BN;
    const int n0 = blockIdx.x * SK_BN;
    const int64_t r0 = (int64_t)blockIdx.y * SK_ROWS;
    const int n = n0 + col;

    auto stage = [&](int buf, int k0) {
        if (vec16) {
            for (int i = tid; i < SK_KC * (SK_BN / 4); i += SK_THREADS) {
                const int kr = i / (SK_BN / 4), c4 = (i % (SK_BN / 4)) * 4;
                const int gk = k0 + kr, gn = n0 + c4;
                int bytes = 0;
                if (gk < K && gn < N) bytes = min(4, N - gn) * 4;
                cp_async16(&Bs[buf][kr][c4], bytes ? B + (int64_t)gk * N + gn : B, bytes);
            }
            for (int i = tid; i < SK_ROWS * (SK_KC / 4); i += SK_THREADS) {
                const int r = i / (SK_KC / 4), c4 = (i % (SK_KC / 4)) * 4;
                const int64_t gr = r0 + r;
                const int gk = k0 + c4;
                int bytes = 0;
                if (gr < R && gk < K) bytes = min(4, K - gk) * 4;
                cp_async16(&As[buf][r][c4], bytes ? A + gr * K + gk : A, bytes);
            }
        } else {
            for (int i = tid; i < SK_KC * SK_BN; i += SK_THREADS) {
                const int kr = i / SK_BN, c = i % SK_BN;
                const int gk = k0 + kr, gn = n0 + c;
                const bool ok = gk < K && gn < N;
                cp_async4(&Bs[buf][kr][c], ok ? B + (int64_t)gk * N + gn : B, ok);
            }
            for (int i = tid; i < SK_ROWS * SK_KC; i += SK_THREADS) {
                const int r = i / SK_KC, c = i % SK_KC;
                const int64_t gr = r0 + r;
                const int gk = k0 + c;
                const bool ok = gr < R && gk < K;
                cp_async4(&As[buf][r][c], ok ? A + gr * K + gk : A, ok);
            }
        }
        cp_async_commit();
    };

    float acc[SK_TR];
#pragma unroll
    for (int r = 0; r < SK_TR; ++r) acc[r] = 0.0f;
    const int nchunks = (K + SK_KC - 1) / SK_KC;
    for (int p = 0; p < SK_STAGES - 1; ++p) {
        if (p < nchunks) stage(p, p * SK_KC);
        else cp_async_commit();                      // empty group: uniform group counts
    }
    for (int ch = 0; ch < nchunks; ++ch) {
        const int buf = ch % SK_STAGES;
        cp_async_wait<SK_STAGES - 2>();              // chunk ch has landed
        __syncthreads();                             // ... for every thread; chunk ch - 1 is consumed
        const int nx = ch + SK_STAGES - 1;
        if (nx < nchunks) stage(nx % SK_STAGES, nx * SK_KC);
        else cp_async_commit();
        const int kl = min(SK_KC, K - ch * SK_KC);
        if (kl == SK_KC) {
#pragma unroll
            for (int k = 0; k < SK_KC; k += 4) {
                const float b0 = Bs[buf][k][col], b1 = Bs[buf][k + 1][col];
                const float b2 = Bs[buf][k + 2][col], b3 = Bs[buf][k + 3][col];
#pragma unroll
                for (int r = 0; r < SK_TR; ++r) {
                    const float4 a = *reinterpret_cast<const float4*>(&As[buf][rg * SK_TR + r][k]);
                    acc[r] = __fmaf_rn(a.x, b0, acc[r]);
                    acc[r] = __fmaf_rn(a.y, b1, acc[r]);
                    acc[r] = __fmaf_rn(a.z, b2, acc[r]);
                    acc[r] = __fmaf_rn(a.w, b3, acc[r]);
                }
            }
        } else {
            for (int k = 0; k < kl; ++k) {
                const float b = Bs[buf][k][col];
#pragma unroll
                for (int r = 0; r < SK_TR; ++r)
                    acc[r] = __fmaf_rn(As[buf][rg * SK_TR + r][k], b, acc[r]);
            }
        }
    }
    if (n < N) {
#pragma unroll
        for (int r = 0; r < SK_TR; ++r) {
            const int64_t gr = r0 + rg * SK_TR + r;
            if (gr < R) C[gr * N + n] = epilogue<EPI>(acc[r], norms, n);
        }
    }
}

}  // namespace

void gemm_argmin(const float* A, const float* B, const float* norms, int64_t R, int K, int N,
                 int32_t* out, cudaStream_t s) {
    if (R <= 0 || N <= 0) return;
    gemm_argmin_kernel<<<(unsigned)ceil_div(R, TBM), 256, 0, s>>>(A, B, norms, R, K, N, out);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void gemm_rows(const float* A, const float* B, float* C, int64_t R, int K, int N,
               GemmEpi epi, const float* norms, cudaStream_t s) {
    if (R <= 0 || N <= 0) return;
    if (R <= 1024) {
        // 1 row per thread for small batches (4x the CTAs), 4 otherwise (a
        // quarter of the L2 re-reads of B)
        const int tr = R <= 256 ? 1 : 4;
        dim3 grid((unsigned)ceil_div(N, SK_BN), (unsigned)ceil_div(R, tr * SK_RG));
        const int vec16 = (N % 4 == 0) && (K % 4 == 0) && (((uintptr_t)A | (uintptr_t)B) % 16 == 0);
        if (grid.y > 65535) fail(JHQ_EINVAL, "gemm_rows: too many rows in one call");
        auto launch = [&](auto kern, int smem) {      // ring above the 48 KB static limit
            JHQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            kern<<<grid, SK_THREADS, smem, s>>>(A, B, C, R, K, N, norms, vec16);
        };
        if (tr == 1) {
            if (epi == EPI_COARSE) launch(gemm_skinny_kernel<EPI_COARSE, 1>, sk_smem_bytes<1>());
            else launch(gemm_skinny_kernel<EPI_STORE, 1>, sk_smem_bytes<1>());
        } else {
            if (epi == EPI_COARSE) launch(gemm_skinny_kernel<EPI_COARSE, 4>, sk_smem_bytes<4>());
            else launch(gemm_skinny_kernel<EPI_STORE, 4>, sk_smem_bytes<4>());
        }
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
