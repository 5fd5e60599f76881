// coarse_tc.cu — approximate IVF coarse scores on the 5th-generation tensor
// cores (tcgen05.mma kind::tf32, accumulator in TMEM, operands staged by TMA).
//
//   s~[q][c] = |c|^2 - 2 * (q3[q] . c3[c])      (tf32 inputs, fp32 sums)
//
// with the 3-term tf32 split of each fp32 value x = hi + lo (hi = x with its 13
// low mantissa bits cleared, lo = x - hi, exact): the rows are laid out as
//   q3 = [q_hi | q_hi | q_lo],  c3 = [c_hi | c_lo | c_hi]   (K = 3d),
// so one GEMM over K = 3d sums q_hi.c_hi + q_hi.c_lo + q_lo.c_hi, which misses
// only q_lo.c_lo (< 2^-20 |q_i c_i|). The scores are approximate within a
// bound that select_probes_margin (ivf.cu) states and turns into the EXACT
// top-nprobe lists of the
// fp32 fma-chain scores (the order the reference's coarse GEMM + selection
// define, jhq_v14_streaming_add/search.cu:13-62), so the probe lists stay
// bit-identical to the fp32 path while the contraction runs on tensor cores.
//
// Tiling: one CTA per 128-query x 256-centroid tile, 128 threads, K in chunks of 32.
//   warp 0 lane 0   TMA producer: K chunks of 32 fp32 (one 128-byte swizzle
//                   row) of the query tile [128][32] and centroid tile
//                   [256][32], double-buffered in shared memory (2 x 48 KB);
//   warp 1 lane 0   MMA issuer: 4 x tcgen05.mma (M=128, N=256, K=8) per chunk
//                   into a 256-column fp32 accumulator in TMEM; tcgen05.commit
//                   frees the stage, a last commit signals the epilogue;
//   warps 0-3       epilogue: tcgen05.ld 32x32b (warp w owns TMEM lanes
//                   32w..32w+31 = tile rows), transposed through shared memory
//                   so each warp stores 128-byte row segments of s~; each row's
//                   minimum over the tile goes to tile_min [nq][ntiles] (the
//                   selection's threshold bound).
// Two CTAs fit per SM (2 x 97 KB shared, 2 x 256 TMEM columns), so one CTA's
// epilogue overlaps the other's loads and MMAs.
//
// Every mbarrier wait is bounded (about a second of clock cycles); a wait that
// gives up sets g_tc_error, the CTA stops issuing work, waits (bounded) for
// the copies and MMAs it already issued, frees its TMEM and returns.
// No TMA load here uses cluster multicast; the operands are this GPU's own memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {

__device__ int g_tc_error;

namespace {

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 32;
constexpr int TC_STAGES = 2;
constexpr int TC_THREADS = 128;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 4;              // 16 KB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 4;              // 32 KB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_SMEM = TC_STAGES * TC_STAGE_BYTES + 1024 + 128;
constexpr uint32_t TC_TMEM_COLS = 256;
// Instruction descriptor: fp32 accumulate (bit 4), A and B tf32 (bits 7-9,
// 10-12 = 2), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t TC_IDESC = (1u << 4) | (2u << 7) | (2u << 10) |
                              ((uint32_t)(TC_BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
constexpr long long TC_WAIT_CYCLES = 1ll << 31;

__device__ __forceinline__ float tf32_hi(float v) {
    return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait for the phase of parity `parity` to complete.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (clock64() - t0 > TC_WAIT_CYCLES) {
            atomicExch(&g_tc_error, 1);
            return false;
        }
    }
    return true;
}

// 128-byte-swizzled K-major operand: rows of 128 bytes, 8-row groups 1024
// bytes apart (stride byte offset), leading byte offset unused (16 B),
// descriptor version 1, layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        :: "r"(dst), "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar) : "memory");
}

__global__ void __launch_bounds__(TC_THREADS, 2)
coarse_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_c,
                 const float* __restrict__ norms, float* __restrict__ scores,
                 float* __restrict__ tile_min, int nq, int nlist, int K) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ float nrm_s[TC_BN];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + TC_STAGES * TC_STAGE_BYTES);   // full[S] empty[S] done
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * TC_STAGES + 1);
    int* flags = (int*)(tmem_slot + 1);                                 // abort, issued
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * TC_BN, m0 = blockIdx.y * TC_BM;
    const int nk = (K + TC_BK - 1) / TC_BK;
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + TC_STAGES),
                   done = smem_u32(bars + 2 * TC_STAGES);

    if (tid == 0) {
        for (int s = 0; s < 2 * TC_STAGES + 1; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(bars + s)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        flags[0] = 0;
        flags[1] = 0;
    }
    for (int i = tid; i < TC_BN; i += TC_THREADS)
        nrm_s[i] = n0 + i < nlist ? norms[n0 + i] : __int_as_float(0x7f800000);   // +inf
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {                       // TMA producer
        for (int kc = 0; kc < nk; ++kc) {
            const int s = kc % TC_STAGES;
            if (kc >= TC_STAGES && !mbar_wait(empty0 + 8 * s, ((kc / TC_STAGES) - 1) & 1)) {
                flags[0] = 1;
                break;
            }
            if (*(volatile int*)&flags[0]) break;
            const uint32_t fb = full0 + 8 * s;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                         :: "r"(fb), "r"((uint32_t)TC_STAGE_BYTES) : "memory");
            const uint32_t a_s = smem_u32(smem + s * TC_STAGE_BYTES);
            tma_load_2d(a_s, &map_q, kc * TC_BK, m0, fb);
            tma_load_2d(a_s + TC_A_BYTES, &map_c, kc * TC_BK, n0, fb);
            flags[1] = kc + 1;
        }
    } else if (warp == 1 && lane == 0) {                // MMA issuer
        for (int kc = 0; kc < nk; ++kc) {
            const int s = kc % TC_STAGES;
            if (!mbar_wait(full0 + 8 * s, (kc / TC_STAGES) & 1)) {
                *(volatile int*)&flags[0] = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_s = smem_u32(smem + s * TC_STAGE_BYTES);
            const uint64_t da = sw128_desc(a_s), db = sw128_desc(a_s + TC_A_BYTES);
#pragma unroll
            for (int k = 0; k < TC_BK / 8; ++k) {
                // +32 bytes per K=8 step inside the swizzle row (start address in 16-byte units)
                const uint32_t acc = (kc | k) != 0;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                    :: "r"(tmem), "l"(da + 2 * k), "l"(db + 2 * k), "r"(TC_IDESC), "r"(acc));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(empty0 + 8 * s) : "memory");
        }
        // Always signal: the epilogue's wait then covers every MMA issued.
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     :: "r"(done) : "memory");
    }
    __syncwarp();

    // ---- epilogue ----
    const bool ok = mbar_wait(done, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    __syncthreads();
    const bool run = ok && !*(volatile int*)&flags[0];
    if (run) {
        float* tile = (float*)smem + warp * (32 * 33);
        const int row0 = m0 + warp * 32;
        float rmin = __int_as_float(0x7f800000);       // this thread's row over the tile
        for (int cb = 0; cb < TC_BN && n0 + cb < nlist; cb += 32) {
            uint32_t r[32];
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)cb;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                  "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                  "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
                  "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                  "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                  "=r"(r[30]), "=r"(r[31])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float sv = nrm_s[cb + j] - 2.0f * __uint_as_float(r[j]);   // +inf past nlist
                tile[lane * 33 + j] = sv;
                rmin = fminf(rmin, sv);
            }
            __syncwarp();
            const int col = n0 + cb + lane;
            for (int rr = 0; rr < 32; ++rr) {
                const int row = row0 + rr;
                if (row < nq && col < nlist) scores[(int64_t)row * nlist + col] = tile[rr * 33 + lane];
            }
            __syncwarp();
        }
        if (row0 + lane < nq) tile_min[(int64_t)(row0 + lane) * gridDim.x + blockIdx.x] = rmin;
    }
    if (tid == 0 && !run) {
        // Copies still in flight land before the shared memory is released.
        const int issued = flags[1];
        for (int kc = (issued > TC_STAGES ? issued - TC_STAGES : 0); kc < issued; ++kc)
            mbar_wait(full0 + 8 * (kc % TC_STAGES), (kc / TC_STAGES) & 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(TC_TMEM_COLS));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) ==
                cudaSuccess && qr == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    if (!fn) fail(JHQ_EDEVICE, "coarse_scores_tc: cuTensorMapEncodeTiled unavailable");
    return fn;
}

// Rows of x -> [hi | hi | lo] rows of out (n x 3d).
__global__ void split3_kernel(const float* __restrict__ x, int64_t n, int d, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * d) return;
    const int64_t r = i / d;
    const int j = (int)(i - r * d);
    const float v = x[i];
    const float hi = tf32_hi(v);
    float* o = out + r * 3 * d;
    o[j] = hi;
    o[d + j] = hi;
    o[2 * d + j] = v - hi;
}

// [rows][d] fp32 row-major, boxes of box_rows x 32 floats, 128-byte swizzle,
// zero fill outside the array (rows >= rows, columns >= d).
CUtensorMap make_map(const float* base, int64_t rows, int d, int box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)d * 4};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims,
                                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(JHQ_EDEVICE, "coarse_scores_tc: tensor map encoding failed");
    return m;
}

}  // namespace

bool coarse_tc_supported(int d, int nlist) {
    // TMA: row stride 3d*4 a multiple of 16 bytes; 16-byte aligned bases.
    return d % 4 == 0 && d >= 4 && nlist >= 1;
}

void split3_rows(const float* x, int64_t n, int d, float* out, cudaStream_t s) {
    if (n <= 0) return;
    const int64_t tot = n * d;
    split3_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(x, n, d, out);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void split3_rows_host(const float* x, int64_t n, int d, int order, float* out) {
    for (int64_t r = 0; r < n; ++r) {
        float* o = out + r * 3 * d;
        for (int j = 0; j < d; ++j) {
            const float v = x[r * d + j];
            uint32_t u;
            std::memcpy(&u, &v, 4);
            u &= 0xFFFFE000u;
            float hi;
            std::memcpy(&hi, &u, 4);
            const float lo = v - hi;
            o[j] = hi;
            o[d + j] = order == 0 ? hi : lo;
            o[2 * d + j] = order == 0 ? lo : hi;
        }
    }
}

int coarse_tc_tiles(int nlist) { return (nlist + TC_BN - 1) / TC_BN; }

void coarse_scores_tc(const float* q3, int nq, const float* c3, const float* norms, int nlist,
                      int d, float* scores, float* tile_min, cudaStream_t s) {
    if (nq <= 0) return;
    if (!coarse_tc_supported(d, nlist) || ((uintptr_t)q3 | (uintptr_t)c3) % 16)
        fail(JHQ_EINVAL, "coarse_scores_tc: unsupported shape or alignment");
    const int gy = (nq + TC_BM - 1) / TC_BM;
    if (gy > 65535) fail(JHQ_EINVAL, "coarse_scores_tc: too many queries in one call");
    static std::once_flag attr;
    std::call_once(attr, [] {
        JHQ_CUDA(cudaFuncSetAttribute(coarse_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      TC_SMEM));
    });
    const CUtensorMap mq = make_map(q3, nq, 3 * d, TC_BM);
    const CUtensorMap mc = make_map(c3, nlist, 3 * d, TC_BN);
    dim3 grid((unsigned)((nlist + TC_BN - 1) / TC_BN), (unsigned)gy);
    coarse_tc_kernel<<<grid, TC_THREADS, TC_SMEM, s>>>(mq, mc, norms, scores, tile_min, nq, nlist,
                                                       3 * d);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

int coarse_tc_error(bool clear) {
    int v = 0;
    JHQ_CUDA(cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)));
    if (clear && v) {
        const int z = 0;
        JHQ_CUDA(cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int)));
    }
    return v;
}

}  // namespace jhq
