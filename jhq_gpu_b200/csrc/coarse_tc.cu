// coarse_tc.cu — approximate IVF coarse scores on the 5th-generation tensor
// cores (tcgen05.mma kind::f16 with bf16 operands, fp32 accumulator in TMEM,
// operands staged by TMA).
//
//   s~[q][c] = |c|^2 - 2 * (q3[q] . c3[c])      (bf16 inputs, fp32 sums)
//
// with a 2-piece bf16 split of each fp32 value, x = hi + lo + r (hi = bf16
// round-to-nearest-even of x, lo = the same rounding of x - hi, which is exact
// in fp32, |r| <= 2^-18 |x|); the rows are laid out as
//   q3 = [q_hi | q_hi | q_lo],  c3 = [c_hi | c_lo | c_hi]   (K = 3d, zero-padded to K3)
// so one GEMM over K3 sums q_hi.c_hi + q_hi.c_lo + q_lo.c_hi (bf16 products
// are exact in fp32), within about 3 * 2^-18 |q_i c_i| of each product. The
// scores are approximate within a bound that select_probes_margin (ivf.cu)
// states and turns into the EXACT top-nprobe lists of the
// fp32 fma-chain scores (the order the reference's coarse GEMM + selection
// define, jhq_v14_streaming_add/search.cu:13-62), so the probe lists stay
// bit-identical to the fp32 path while the contraction runs on tensor cores.
//
// Persistent kernel, one CTA per SM (192 threads), over 128-query x 256-list
// output tiles (tile t = query tile t % mt, list tile t / mt, so the CTAs
// resident together share one list tile and each is read from HBM about once):
//   warp 0 lane 0   TMA producer: K chunks of 64 bf16 (one 128-byte swizzle
//                   row) of the query tile [128][64] and list tile [256][64]
//                   into a 4-stage ring (4 x 48 KB);
//   warp 1 lane 0   MMA issuer: 4 x tcgen05.mma (M=128, N=256, K=16) per chunk
//                   into one of two 256-column fp32 accumulators in TMEM
//                   (512 columns), tcgen05.commit frees each stage and, after
//                   a tile's last chunk, hands the accumulator to the epilogue;
//   warps 2-9       epilogue: tcgen05.ld 32x32b (warp w reads TMEM lanes
//                   32 (w % 4) .. +31 = tile rows, warps w and w + 4 split the
//                   256 columns into two 128-list groups), transposed through
//                   shared memory so each warp stores 128-byte row segments of
//                   s~; each row's minimum over its group goes to tile_min
//                   [nq][ngroups] (the selection's threshold bound); then the
//                   accumulator is released to the MMA warp.
// The epilogue of tile i overlaps the loads and MMAs of tile i + 1.
//
// Every mbarrier wait is bounded (about a second of clock cycles); a wait that
// gives up sets g_tc_error and a shared abort flag that ends every role's
// loop; the producer then waits (bounded) for the copies it issued, the MMA
// warp for its MMAs (a final commit), and the CTA frees its TMEM and returns.
// Every TMA load here reads this GPU's own memory into its own CTA only.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "device_utils.cuh"
#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {

__device__ int g_tc_error;

namespace {

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64;       // BK in bf16 elements
constexpr int TC_STAGES = 4;
constexpr int TC_EPI_WARPS = 8;                            // two per TMEM lane quarter
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int TC_EPI_THREADS = 32 * TC_EPI_WARPS;
constexpr int TC_GROUP = COARSE_TILE_LISTS;                // lists per tile_min entry
static_assert(TC_BN == 2 * TC_GROUP, "each epilogue warp of a quarter owns one group");
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;              // 16 KB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;              // 32 KB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_EPI_BYTES = TC_EPI_WARPS * 32 * 32 * 4;   // per-warp 32 x 32 transposition
constexpr int TC_NBARS = 2 * TC_STAGES + 2 + 2 + 1;        // full, empty, tfull, tempty, drain
constexpr int TC_SMEM = TC_STAGES * TC_STAGE_BYTES + TC_EPI_BYTES + 1024 + 256;
constexpr uint32_t TC_TMEM_COLS = 512;
static_assert(TC_NBARS * 8 + 16 <= 256, "barrier area");
// Instruction descriptor: fp32 accumulate (bit 4), A and B bf16 (bits 7-9,
// 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t TC_IDESC = (1u << 4) | (1u << 7) | (1u << 10) |
                              ((uint32_t)(TC_BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
constexpr long long TC_WAIT_CYCLES = 1ll << 31;

// bf16 bits of x, rounded to nearest even (finite x).
__host__ __device__ __forceinline__ uint16_t bf16_rne(uint32_t u) {
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
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

// Bounded wait for the phase of parity `parity`; gives up (false) when the
// CTA's abort flag is set or after `limit` cycles, which sets the flag. The
// pipeline waits use the launch's limit (TC_WAIT_CYCLES unless a test shortens
// it); the drain waits (abort == nullptr) always use TC_WAIT_CYCLES.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                          long long limit = TC_WAIT_CYCLES) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (abort && *abort) return false;
        if (clock64() - t0 > limit) {
            atomicExch(&g_tc_error, 1);
            if (abort) *abort = 1;
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

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}

__global__ void __launch_bounds__(TC_THREADS, 1)
coarse_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_c,
                 const float* __restrict__ norms, float* __restrict__ scores,
                 float* __restrict__ tile_min, int nq, int nlist, int K, int mt, int ntiles,
                 long long wait_limit) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* epi = (float*)(smem + TC_STAGES * TC_STAGE_BYTES);
    uint64_t* bars = (uint64_t*)(smem + TC_STAGES * TC_STAGE_BYTES + TC_EPI_BYTES);
    uint32_t* tmem_slot = (uint32_t*)(bars + TC_NBARS);
    volatile int* abort = (volatile int*)(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nk = (K + TC_BK - 1) / TC_BK;
    const int ngr = (nlist + TC_GROUP - 1) / TC_GROUP;    // tile_min row length
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * TC_STAGES,
                   tfull0 = empty0 + 8 * TC_STAGES, tempty0 = tfull0 + 16, drain = tempty0 + 16;

    if (tid == 0) {
        for (int i = 0; i < TC_NBARS; ++i) {
            const uint32_t a = full0 + 8 * i;
            const uint32_t cnt = (a >= tempty0 && a < drain) ? TC_EPI_THREADS : 1;
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(a), "r"(cnt));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {                                   // TMA producer
            int it = 0;
            for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
                const int m0 = (t % mt) * TC_BM, n0 = (t / mt) * TC_BN;
                for (int kc = 0; kc < nk; ++kc, ++it) {
                    const int s = it % TC_STAGES;
                    if (it >= TC_STAGES &&
                        !mbar_wait(empty0 + 8 * s, ((it / TC_STAGES) - 1) & 1, abort, wait_limit))
                        break;
                    const uint32_t fb = full0 + 8 * s;
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                                 :: "r"(fb), "r"((uint32_t)TC_STAGE_BYTES) : "memory");
                    const uint32_t a_s = smem_u32(smem + s * TC_STAGE_BYTES);
                    tma_load_2d(a_s, &map_q, kc * TC_BK, m0, fb);
                    tma_load_2d(a_s + TC_A_BYTES, &map_c, kc * TC_BK, n0, fb);
                }
            }
            if (*abort)   // copies still in flight land before the shared memory is released
                for (int j = it > TC_STAGES ? it - TC_STAGES : 0; j < it; ++j)
                    mbar_wait(full0 + 8 * (j % TC_STAGES), (j / TC_STAGES) & 1, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {                                   // MMA issuer
            int it = 0, i = 0;
            for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++i) {
                const int acc = i & 1;
                if (i >= 2 && !mbar_wait(tempty0 + 8 * acc, ((i >> 1) - 1) & 1, abort, wait_limit))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d_tmem = tmem + (uint32_t)(acc * TC_BN);
                bool ok = true;
                for (int kc = 0; kc < nk; ++kc, ++it) {
                    const int s = it % TC_STAGES;
                    if (!mbar_wait(full0 + 8 * s, (it / TC_STAGES) & 1, abort, wait_limit)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a_s = smem_u32(smem + s * TC_STAGE_BYTES);
                    const uint64_t da = sw128_desc(a_s), db = sw128_desc(a_s + TC_A_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_BK / 16; ++k) {
                        // +32 bytes per K=16 step inside the swizzle row (16-byte units)
                        const uint32_t accum = (kc | k) != 0;
                        asm volatile(
                            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                            :: "r"(d_tmem), "l"(da + 2 * k), "l"(db + 2 * k), "r"(TC_IDESC),
                               "r"(accum));
                    }
                    mma_commit(empty0 + 8 * s);
                }
                if (!ok) break;
                mma_commit(tfull0 + 8 * acc);
            }
            mma_commit(drain);                             // every MMA issued has completed
            mbar_wait(drain, 0, nullptr);
        }
    } else {                                               // epilogue, warps 2..9
        const int q4 = warp & 3;                           // TMEM lane quarter
        const int half = (warp - 2) >> 2;                  // column half = list group
        float* tile = epi + (warp - 2) * (32 * 32);
        const bool vec = (nlist & 3) == 0;                 // 16-byte row segments
        int i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
            const int acc = i & 1;
            const bool ok = mbar_wait(tfull0 + 8 * acc, (i >> 1) & 1, abort, wait_limit);
            if (!__all_sync(0xffffffffu, ok)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int m0 = (t % mt) * TC_BM, n0 = (t / mt) * TC_BN;
            const int row0 = m0 + q4 * 32;
            // store layout: lane = (row sub-index rsub, 4-column group cg); a
            // warp instruction covers 4 rows x 32 columns (four 128-byte segments)
            const int cg = lane & 7, rsub = lane >> 3;
            float rmin[8];
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) rmin[rr] = __int_as_float(0x7f800000);
            for (int cb = half * TC_GROUP; cb < (half + 1) * TC_GROUP && n0 + cb < nlist; cb += 32) {
                uint32_t r[32];
                const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16) +
                                       (uint32_t)(acc * TC_BN + cb);
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
                // row layout (thread = row) -> shared memory; 16-byte chunk k of
                // row l sits at chunk k ^ (l & 7), conflict-free both ways
                float4* trow = reinterpret_cast<float4*>(tile + lane * 32);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    trow[k ^ (lane & 7)] = make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]),
                                          __uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3]));
                __syncwarp();
                const int col = n0 + cb + 4 * cg;
                const float inf = __int_as_float(0x7f800000);
                float4 nv;
                if (vec && col + 3 < nlist) {
                    nv = *reinterpret_cast<const float4*>(norms + col);
                } else {
                    nv.x = col < nlist ? norms[col] : inf;
                    nv.y = col + 1 < nlist ? norms[col + 1] : inf;
                    nv.z = col + 2 < nlist ? norms[col + 2] : inf;
                    nv.w = col + 3 < nlist ? norms[col + 3] : inf;
                }
#pragma unroll
                for (int rr = 0; rr < 8; ++rr) {
                    const int rl = rr * 4 + rsub;
                    const float4 a4 =
                        *reinterpret_cast<const float4*>(tile + rl * 32 + 4 * (cg ^ (rl & 7)));
                    float4 sv;
                    sv.x = nv.x - 2.0f * a4.x;
                    sv.y = nv.y - 2.0f * a4.y;
                    sv.z = nv.z - 2.0f * a4.z;
                    sv.w = nv.w - 2.0f * a4.w;
                    rmin[rr] = fminf(rmin[rr], fminf(fminf(sv.x, sv.y), fminf(sv.z, sv.w)));
                    const int row = row0 + rl;
                    if (row < nq) {
                        float* dst = scores + (int64_t)row * nlist + col;
                        if (vec && col + 3 < nlist) {
                            *reinterpret_cast<float4*>(dst) = sv;
                        } else {
                            if (col < nlist) dst[0] = sv.x;
                            if (col + 1 < nlist) dst[1] = sv.y;
                            if (col + 2 < nlist) dst[2] = sv.z;
                            if (col + 3 < nlist) dst[3] = sv.w;
                        }
                    }
                }
                __syncwarp();
            }
            const int g = (t / mt) * 2 + half;
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) {
                float m = rmin[rr];
                m = fminf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                m = fminf(m, __shfl_xor_sync(0xffffffffu, m, 2));
                m = fminf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                const int row = row0 + rr * 4 + rsub;
                if (cg == 0 && row < nq && g < ngr) tile_min[(int64_t)row * ngr + g] = m;
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(tempty0 + 8 * acc)
                         : "memory");
        }
    }
    __syncwarp();
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

// Rows of x -> [hi | hi | lo | 0...] bf16 rows of out (n x K3).
__global__ void split3_kernel(const float* __restrict__ x, int64_t n, int d, int K3,
                              uint16_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * K3) return;
    const int64_t r = i / K3;
    const int j = (int)(i - r * K3);
    const int part = j / d, jj = j - part * d;
    uint16_t v = 0;
    if (part < 3) {
        const float xv = x[r * d + jj];
        const uint16_t hi = bf16_rne(__float_as_uint(xv));
        v = part < 2 ? hi : bf16_rne(__float_as_uint(xv - __uint_as_float((uint32_t)hi << 16)));
    }
    out[i] = v;
}

// [rows][K] bf16 row-major, boxes of box_rows x 64 elements, 128-byte swizzle,
// zero fill outside the array.
CUtensorMap make_map(const uint16_t* base, int64_t rows, int K, int box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)base, dims,
                                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(JHQ_EDEVICE, "coarse_scores_tc: tensor map encoding failed");
    return m;
}

}  // namespace

bool coarse_tc_supported(int d, int nlist) { return d >= 1 && nlist >= 1; }

int coarse_tc_k3(int d) { return (3 * d + 7) / 8 * 8; }   // 16-byte row stride for TMA

void split3_rows(const float* x, int64_t n, int d, uint16_t* out, cudaStream_t s) {
    if (n <= 0) return;
    const int K3 = coarse_tc_k3(d);
    const int64_t tot = n * K3;
    split3_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(x, n, d, K3, out);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void split3_rows_host(const float* x, int64_t n, int d, int order, uint16_t* out) {
    const int K3 = coarse_tc_k3(d);
    for (int64_t r = 0; r < n; ++r) {
        uint16_t* o = out + r * K3;
        for (int j = 0; j < K3; ++j) o[j] = 0;
        for (int j = 0; j < d; ++j) {
            const float v = x[r * d + j];
            uint32_t u;
            std::memcpy(&u, &v, 4);
            const uint16_t hi = bf16_rne(u);
            const uint32_t hu = (uint32_t)hi << 16;
            float hf;
            std::memcpy(&hf, &hu, 4);
            const float rest = v - hf;
            std::memcpy(&u, &rest, 4);
            const uint16_t lo = bf16_rne(u);
            o[j] = hi;
            o[d + j] = order == 0 ? hi : lo;
            o[2 * d + j] = order == 0 ? lo : hi;
        }
    }
}

int coarse_tc_tiles(int nlist) { return (nlist + TC_GROUP - 1) / TC_GROUP; }

void coarse_scores_tc(const uint16_t* q3, int nq, const uint16_t* c3, const float* norms,
                      int nlist, int d, float* scores, float* tile_min, cudaStream_t s) {
    if (nq <= 0) return;
    if (!coarse_tc_supported(d, nlist) || ((uintptr_t)q3 | (uintptr_t)c3) % 16)
        fail(JHQ_EINVAL, "coarse_scores_tc: unsupported shape or alignment");
    const int mt = (nq + TC_BM - 1) / TC_BM, nlt = (nlist + TC_BN - 1) / TC_BN;   // MMA tiles
    const int64_t ntiles = (int64_t)mt * nlt;
    if (ntiles > INT32_MAX) fail(JHQ_EINVAL, "coarse_scores_tc: too many tiles");
    static std::atomic<uint64_t> attr{0};
    once_per_device(attr, [] {
        JHQ_CUDA(cudaFuncSetAttribute(coarse_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      TC_SMEM));
    });
    int dev = 0, nsm = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    const int K3 = coarse_tc_k3(d);
    const CUtensorMap mq = make_map(q3, nq, K3, TC_BM);
    const CUtensorMap mc = make_map(c3, nlist, K3, TC_BN);
    const int grid = (int)std::min<int64_t>(ntiles, nsm);
    // Test hook: JHQ_TEST_TC_WAIT_CYCLES shortens the pipeline waits of the
    // kernels launched (or captured) from now on, so that a test can make a wait
    // give up and check the JHQ_ETIMEDOUT report; the drain waits keep their limit.
    long long wait_limit = TC_WAIT_CYCLES;
    if (const char* e = std::getenv("JHQ_TEST_TC_WAIT_CYCLES")) wait_limit = std::atoll(e);
    coarse_tc_kernel<<<grid, TC_THREADS, TC_SMEM, s>>>(mq, mc, norms, scores, tile_min, nq, nlist,
                                                       K3, mt, (int)ntiles, wait_limit);
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


namespace {

// ===========================================================================
// Flat ADC scan on the tensor cores for 1-bit codes (K1D = 2: B = 8, Ds = 8).
//
// With two codewords c0 < c1 per dimension and b_j in {0, 1} the bit of dim j,
//   s_v = sum_j (q_j - c[b_j])^2 = S0 + D * pop(v) - 2 e * (q . b_v),
//   S0 = sum_j (q_j - c0)^2,  D = c1^2 - c0^2,  e = c1 - c0,  pop = popcount,
// so the ADC distance of every (vector, query) pair is one GEMM of the code
// bits with the queries. flat_tc_kernel computes g = q . b on tcgen05 in
// integer arithmetic (kind::i8, exact s32 accumulation):
//   * each query is quantised to Q = rint(q / s), s = max|q| / 32000, and Q is
//     split in two signed bytes Q = 256 Qh + Ql; the residual
//     R1 = sum_j |q_j - s Q_j| bounds |q . b - s Q . b| for every b;
//   * the B operand (the block's Qh rows, then its Ql rows, all K) is loaded
//     into shared memory once per CTA by TMA and stays there;
//   * the A operand (128 vectors x 128 dims per K chunk) is expanded from the
//     code bytes to s8 0/1 in shared memory by eight warps (two threads per
//     row), in the 128-byte swizzled K-major layout a TMA would produce (row r
//     at r * 128 bytes, 16-byte chunk c stored at c ^ (r & 7));
//   * one MMA of N' = 2N columns per 32-dim step: TMEM columns [0, N) collect
//     Qh . b and [N, 2N) Ql . b.
// Eight epilogue warps (two per TMEM lane quarter, alternating 32-column
// blocks) form s~ = S0 + D pop + (-2 e s) (256 Gh + Gl), store s~ [q][v] and
// the per-query minimum of each 128-vector tile. The scores are
// approximate; flat_select (below) turns them into the exact top-ck of the
// LUT-path keys. Same bounded-wait / abort / drain discipline as
// coarse_tc_kernel.
constexpr int FT_BM = 128, FT_BK = 128;       // BK in bytes = dims (u8 / s8 operands)
constexpr int FT_EXP = 256;                  // expander threads: two per tile row (64 dims each)
constexpr int FT_MMA_WARP = FT_EXP / 32;      // warp 8 issues the MMAs
constexpr int FT_EPI = 256;                   // epilogue threads: two warps per TMEM lane quarter
constexpr int FT_THREADS = FT_EXP + 32 + FT_EPI;
constexpr int FT_A_BYTES = FT_BM * FT_BK;     // 16 KB per stage
constexpr int FT_B_MAX = 128 * 1024;          // resident query block
constexpr int FT_SMEM_MAX = 227 * 1024;
constexpr float FT_QMAX = 32000.0f;           // |Q| bound: Qh in [-125, 125], Ql in [-128, 127]

// queries per block for dimension d: the resident 2N x d bytes fit FT_B_MAX
__host__ __device__ inline int ft_block_queries(int d) {
    const int n = FT_B_MAX / (2 * d) / 32 * 32;
    return n < 128 ? n : 128;
}
__host__ __device__ inline int ft_stages(int N, int d) {
    const int s = (FT_SMEM_MAX - 3072 - 2 * N * d) / FT_A_BYTES;
    return s < 6 ? s : 6;
}
__host__ __device__ inline int ft_smem_bytes(int N, int d) {
    return 2 * N * d + ft_stages(N, d) * FT_A_BYTES + 1024 + 256 + 1024;
}

// 32 consecutive 32-bit TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// bits 0-3 of x -> bytes 0-3 of the result, each 0 or 1 (the four shifted
// copies of x occupy disjoint bit ranges, so the product has no carries)
__device__ __forceinline__ uint32_t spread4(uint32_t x) { return (x * 0x00204081u) & 0x01010101u; }

__global__ void __launch_bounds__(FT_THREADS, 1)
flat_tc_kernel(const __grid_constant__ CUtensorMap map_q, const uint8_t* __restrict__ codes,
               const int32_t* __restrict__ pop, const float* __restrict__ S0,
               const float* __restrict__ qscale, int nvec, int M, int nq, int N, float Dc,
               float ec, float* __restrict__ scores, uint32_t* __restrict__ tile_min, int ntiles,
               long long wait_limit) {
    extern __shared__ uint8_t smem_raw[];
    const int d = M * 8, nk = d / FT_BK;
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* bsm = smem;                                   // [nk][2N][128] resident B
    uint8_t* asm_ = smem + 2 * N * d;                      // [S][128][128] A stages
    const int S = ft_stages(N, d);
    uint64_t* bars = (uint64_t*)(asm_ + S * FT_A_BYTES);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * S + 6);
    float* cst = (float*)(asm_ + S * FT_A_BYTES + 256);    // [2][128] epilogue constants
    volatile int* abort = (volatile int*)(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * S, tfull0 = empty0 + 8 * S,
                   tempty0 = tfull0 + 16, drain = tempty0 + 16, bfull = drain + 8;
    // s32 accumulate (bits 4-5 = 2), A and B s8 (bits 7-9, 10-12 = 1; the code
    // bits are 0 / 1), both K-major, N' = 2N at bit 17, M at bit 24
    const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(2 * N >> 3) << 17) |
                           ((uint32_t)(FT_BM >> 4) << 24);
    uint32_t cols = 32;
    while (cols < (uint32_t)(4 * N)) cols <<= 1;
    if (tid == 0) {
        for (int i = 0; i < 2 * S + 6; ++i) {
            const uint32_t a = full0 + 8 * i;
            uint32_t cnt = 1;
            if (a < empty0) cnt = FT_EXP;                  // the expanders
            else if (a >= tempty0 && a < drain) cnt = FT_EPI; // epilogue threads
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(a), "r"(cnt));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort = 0;
    }
    if (warp == FT_MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp < FT_MMA_WARP) {                              // A expansion (+ the B load)
        const int r = tid & (FT_BM - 1);                   // tile row = vector
        const int hf = tid >> 7;                           // dims 64 hf .. 64 hf + 63 of a chunk
        if (tid == 0) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                         :: "r"(bfull), "r"((uint32_t)(2 * N * d)) : "memory");
            for (int kb = 0; kb < nk; ++kb)
                tma_load_2d(smem_u32(bsm + kb * 2 * N * FT_BK), &map_q, kb * FT_BK, 0, bfull);
        }
        // the CTA's (tile, K chunk) items in order: item i is chunk i % nk of the
        // CTA's tile i / nk. The code bytes of a group of 8 items are loaded
        // while the previous group is expanded (8 loads in flight per thread).
        const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const int total = my_tiles * nk;
        auto load_item = [&](int item) {
            const int t = blockIdx.x + (item / nk) * gridDim.x, kc = item % nk;
            const int v = t * FT_BM + r;
            return (item < total && v < nvec)
                       ? __ldg(reinterpret_cast<const uint2*>(codes + (int64_t)v * M + kc * 16 + hf * 8))
                       : make_uint2(0u, 0u);
        };
        uint2 cur[8], nxt[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) cur[j] = load_item(j);
        bool stop = false;
        for (int g = 0; g * 8 < total && !stop && !*abort; ++g) {
#pragma unroll
            for (int j = 0; j < 8; ++j) nxt[j] = load_item((g + 1) * 8 + j);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int it = g * 8 + j;
                if (it >= total) break;
                const int s = it % S;
                if (it >= S && !mbar_wait(empty0 + 8 * s, ((it / S) - 1) & 1, abort, wait_limit)) {
                    stop = true;
                    break;
                }
                uint8_t* row = asm_ + s * FT_A_BYTES + (r >> 3) * 1024 + (r & 7) * 128;
                const uint32_t w[2] = {cur[j].x, cur[j].y};
#pragma unroll
                for (int c = 0; c < 4; ++c) {              // 16 dims = code bytes 2c, 2c + 1 of the half
                    const uint32_t b2 = w[c >> 1] >> ((c & 1) * 16);
                    const uint4 o = make_uint4(spread4(b2 & 15u), spread4((b2 >> 4) & 15u),
                                               spread4((b2 >> 8) & 15u), spread4((b2 >> 12) & 15u));
                    *reinterpret_cast<uint4*>(row + (((hf * 4 + c) ^ (r & 7)) << 4)) = o;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(full0 + 8 * s)
                             : "memory");
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
        }
        // the B copy must complete before the CTA exits
        if (tid == 0) mbar_wait(bfull, 0, nullptr);
    } else if (warp == FT_MMA_WARP) {
        if (lane == 0) {                                   // MMA issuer
            int it = 0, i = 0;
            bool ok = mbar_wait(bfull, 0, abort, wait_limit);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int t = blockIdx.x; ok && t < ntiles && !*abort; t += gridDim.x, ++i) {
                const int acc = i & 1;
                if (i >= 2 && !mbar_wait(tempty0 + 8 * acc, ((i >> 1) - 1) & 1, abort, wait_limit))
                    break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d_tmem = tmem + (uint32_t)(acc * 2 * N);
                for (int kc = 0; kc < nk; ++kc, ++it) {
                    const int s = it % S;
                    if (!mbar_wait(full0 + 8 * s, (it / S) & 1, abort, wait_limit)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t da = sw128_desc(smem_u32(asm_ + s * FT_A_BYTES));
                    const uint64_t db = sw128_desc(smem_u32(bsm + kc * 2 * N * FT_BK));  // Qh rows, then Ql
#pragma unroll
                    for (int k = 0; k < FT_BK / 32; ++k) {   // 32 dims = 32 bytes per MMA
                        const uint32_t accum = (kc | k) != 0;
                        asm volatile(
                            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                            :: "r"(d_tmem), "l"(da + 2 * k), "l"(db + 2 * k), "r"(idesc), "r"(accum));
                    }
                    mma_commit(empty0 + 8 * s);
                }
                if (!ok) break;
                mma_commit(tfull0 + 8 * acc);
            }
            mma_commit(drain);
            mbar_wait(drain, 0, nullptr);
        }
    } else {                                               // epilogue, warps 9-16
        const int q4 = warp & 3;          // TMEM lane quarter: a warp reads lanes 32 (warp % 4) ..
        const int half = (warp - FT_MMA_WARP - 1) >> 2;    // column blocks half, half + 2, ...
        // per query column: S0 and -2 e s (one rounding, like the product it replaces)
        for (int q = tid - FT_EXP - 32; q < N; q += FT_EPI) {
            cst[q] = q < nq ? S0[q] : 0.0f;
            cst[128 + q] = q < nq ? -2.0f * ec * qscale[q] : 0.0f;
        }
        asm volatile("bar.sync 1, %0;" :: "n"(FT_EPI) : "memory");
        int i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
            const int acc = i & 1;
            const bool ok = mbar_wait(tfull0 + 8 * acc, (i >> 1) & 1, abort, wait_limit);
            if (!__all_sync(0xffffffffu, ok)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int v = t * FT_BM + q4 * 32 + lane;
            const float pv = v < nvec ? (float)__ldg(pop + v) : 0.0f;
            for (int cb = half * 32; cb < N; cb += 64) {
                uint32_t rh[32], rl[32];
                const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(acc * 2 * N + cb);
                tmem_ld32(taddr, rh);
                tmem_ld32(taddr + (uint32_t)N, rl);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                float m[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int q = cb + c;
                    m[c] = __int_as_float(0x7f800000);
                    if (q < nq) {                                       // warp-uniform
                        // |256 Gh + Gl| <= 32000 d: exact in int32
                        const int gi = (int)rh[c] * 256 + (int)rl[c];
                        const float sv = __fmaf_rn(cst[128 + q], (float)gi, __fmaf_rn(Dc, pv, cst[q]));
                        if (v < nvec) {
                            scores[(int64_t)q * nvec + v] = sv;
                            m[c] = sv;
                        }
                    }
                }
                // transpose-reduce: after the 5 halving steps lane c holds the
                // minimum of column c over the warp's 32 rows (31 shuffles)
#pragma unroll
                for (int h = 16; h; h >>= 1) {
                    const bool up = lane & h;
#pragma unroll
                    for (int j = 0; j < h; ++j) {
                        const float send = up ? m[j] : m[j + h];
                        const float keep = up ? m[j + h] : m[j];
                        m[j] = fminf(keep, __shfl_xor_sync(0xffffffffu, send, h));
                    }
                }
                if (cb + lane < nq)
                    atomicMin(tile_min + (int64_t)(cb + lane) * ntiles + t, float_order(m[0]));
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(tempty0 + 8 * acc)
                         : "memory");
        }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == FT_MMA_WARP)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(cols));
}


// Per query block row q < nq: the signed byte planes q8[q] = Qh, q8[N + q] =
// Ql of Q = rint(q / s), s = max|q| / 32000 (rows nq..N-1 zero), and per query
// S0 = sum_j (q_j - c0)^2 (a per-query constant: its rounding shifts every s~
// of the query alike and cancels in the selection), the scale s and the
// quantisation residual R1 = sum_j |q_j - s Q_j|.
__global__ void flat_prep_kernel(const float* __restrict__ q_rot, int nq, int N, int d, float c0,
                                 int8_t* __restrict__ q8, float* __restrict__ S0,
                                 float* __restrict__ qscale, float* __restrict__ R1) {
    const int q = blockIdx.x;
    __shared__ float red[2][32];
    __shared__ float s_sh;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float amax = 0.0f;
    for (int j = threadIdx.x; j < d; j += blockDim.x)
        amax = fmaxf(amax, q < nq ? fabsf(q_rot[(int64_t)q * d + j]) : 0.0f);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[0][warp] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int w = 0; w < nw; ++w) a = fmaxf(a, red[0][w]);
        s_sh = a > 0.0f ? a / FT_QMAX : 1.0f;
    }
    __syncthreads();
    const float sc = s_sh;
    float acc = 0.0f, res = 0.0f;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        const float x = q < nq ? q_rot[(int64_t)q * d + j] : 0.0f;
        const float Qf = fminf(fmaxf(rintf(x / sc), -FT_QMAX), FT_QMAX);
        const int Q = (int)Qf;
        const int qh = (Q + 128) >> 8;                 // floor((Q + 128) / 256)
        q8[(int64_t)q * d + j] = (int8_t)qh;
        q8[((int64_t)N + q) * d + j] = (int8_t)(Q - qh * 256);
        res += fabsf(__fmaf_rn(-sc, Qf, x));
        const float t = x - c0;
        acc = __fmaf_rn(t, t, acc);
    }
    __syncthreads();
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        acc += __shfl_xor_sync(0xffffffffu, acc, o);
        res += __shfl_xor_sync(0xffffffffu, res, o);
    }
    if (lane == 0) { red[0][warp] = acc; red[1][warp] = res; }
    __syncthreads();
    if (threadIdx.x == 0 && q < nq) {
        float tot = 0.0f, rt = 0.0f;
        for (int w = 0; w < nw; ++w) { tot += red[0][w]; rt += red[1][w]; }
        S0[q] = tot;
        qscale[q] = sc;
        R1[q] = rt;
    }
}

// Exact top-ck from the approximate scores, one CTA (8 warps) per query:
//   tau = ck-th smallest tile minimum of s~ (ck distinct vectors have s~ <= tau);
//   every exact top-ck member has s~ <= tau + 2E (E bounds |s~ - s| per vector
//   up to a per-query constant), so only tiles whose minimum is <= tau + 2E are
//   read, their vectors with s~ <= tau + 2E are rescored with the scan's own
//   arithmetic (nibble tables lo + hi, in-order sum over m: the oracle's key),
//   and the exact top-ck by (distance, id) is written as the query's single
//   candidate slot for the refine. The keys are unique (they hold the id), so
//   the result does not depend on the order the threads find the candidates in.
constexpr int FS_THREADS = 256;
constexpr int FS_CAP = 1024;                 // exact keys held before a compaction (>= ck_pad + 256)
constexpr int FS_ROUND = 64;                 // hot tiles read per round (8 per warp)
constexpr int FS_CAND = FS_ROUND * FT_BM;    // window candidates of one round
constexpr int FS_TILES = 4096;               // tile minima per query (nvec <= 524,288)
constexpr int FS_SMEM_MAX = 200 * 1024;      // dynamic shared memory (the kernel has static too)

__host__ __device__ inline size_t fs_smem_bytes(int M, int ntiles_pad) {
    return (size_t)M * 32 * 4 + (size_t)FS_CAP * 8 + (size_t)ntiles_pad * 4 * 2 + (size_t)FS_CAND * 4;
}

__global__ void __launch_bounds__(FS_THREADS, 1)
flat_select_kernel(const float* __restrict__ q_rot, const float* __restrict__ c1d_g,
                   const uint8_t* __restrict__ codes, const float* __restrict__ scores,
                   const uint32_t* __restrict__ tile_min, const float* __restrict__ R1q, int nvec,
                   int M, int nq, int ck, int ck_pad, int ntiles, int ntiles_pad, float cmax,
                   float ec, float Dc, uint64_t* __restrict__ cand, uint64_t* __restrict__ gthr,
                   int64_t* __restrict__ qslot_off, const int* __restrict__ d_nvalid) {
    extern __shared__ __align__(16) unsigned char fs_smem[];
    __shared__ float red[3][FS_THREADS / 32];
    __shared__ int cnt[2][FS_THREADS / 32];
    __shared__ int nhot_s, nc_s, n_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = FS_THREADS / 32;
    const int q = blockIdx.x;
    if (q >= nq) return;
    if (tid == 0) {
        qslot_off[q + 1] = q + 1;
        if (q == 0) qslot_off[0] = 0;
    }
    if (d_nvalid && q >= *d_nvalid) {
        // padding row of a partial batch (zeros: every vector ties, so the
        // window would take them all): no candidates
        for (int i = tid; i < ck; i += FS_THREADS) cand[(int64_t)q * ck + i] = KEY_EMPTY;
        if (tid == 0) gthr[q] = KEY_EMPTY;
        return;
    }
    float* tab = reinterpret_cast<float*>(fs_smem);                              // [M][32]
    uint64_t* buf = reinterpret_cast<uint64_t*>(fs_smem + (size_t)M * 32 * 4);   // [FS_CAP] exact keys
    uint32_t* tk = reinterpret_cast<uint32_t*>(buf + FS_CAP);                    // [ntiles] tile minima
    int* hot = reinterpret_cast<int*>(tk + ntiles_pad);                          // tiles in the window
    int* cl = hot + ntiles_pad;                                                  // [FS_CAND] candidates
    const int d = M * 8;
    const float* qv = q_rot + (int64_t)q * d;
    const float c0 = c1d_g[0], c1 = c1d_g[1];
    const unsigned lt = (1u << lane) - 1u;

    // error bound (all but per-query constants): LUT-path rounding of s, the
    // quantisation of q (R1: exact integer products and sums after it), and the
    // roundings forming g~ and s~
    float V = 0.0f, L1 = 0.0f, S0 = 0.0f;
    for (int j = tid; j < d; j += FS_THREADS) {
        const float x = qv[j], a = fabsf(x) + cmax, t = x - c0;
        V += a * a;
        L1 += fabsf(x);
        S0 += t * t;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        V += __shfl_xor_sync(0xffffffffu, V, o);
        L1 += __shfl_xor_sync(0xffffffffu, L1, o);
        S0 += __shfl_xor_sync(0xffffffffu, S0, o);
    }
    if (lane == 0) { red[0][warp] = V; red[1][warp] = L1; red[2][warp] = S0; }
    if (tid == 0) { nhot_s = 0; n_s = 0; }

    // the query's nibble tables (the scan's mode-1 tables: lo dims 0-3, hi 4-7)
    for (int i = tid; i < M * 32; i += FS_THREADS) {
        const int m = i >> 5, t = i & 31, half = t >> 4, nb = t & 15;
        float acc = 0.0f;
        for (int k = 0; k < 4; ++k) {
            const float diff = qv[m * 8 + half * 4 + k] - ((nb >> k) & 1 ? c1 : c0);
            acc = __fmaf_rn(diff, diff, acc);
        }
        tab[i] = acc;
    }
    for (int i = tid; i < ntiles; i += FS_THREADS) tk[i] = tile_min[(int64_t)q * ntiles + i];
    __syncthreads();
    V = L1 = S0 = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) { V += red[0][w]; L1 += red[1][w]; S0 += red[2][w]; }
    // the 1.001 factors cover the fp32 rounding of V, S0 and R1 themselves
    const float u = 5.9604645e-08f;                                    // 2^-24
    const float aD = fabsf(Dc), ae = fabsf(ec), R1 = R1q[q] * 1.001f;
    const float G = (L1 + R1) * 1.001f;                                // bounds |g~|
    const float E = 1.1f * (V * 1.001f * (float)(2 * M + 16) * u + aD * (float)d * u +
                            2.0f * ae * (R1 + 2.0f * u * G) +
                            2.0f * u * (S0 * 1.001f + aD * (float)d + 2.0f * ae * G));

    // tau = the ck-th smallest tile minimum: bisection over the order keys
    // (one barrier per step: the warp counts alternate between two rows)
    float tau = __int_as_float(0x7f800000);
    if (ck <= ntiles) {
        uint32_t lo = 0, hi = 0xFFFFFFFFu;                 // smallest x with count(k <= x) >= ck
        int it = 0;
        while (lo < hi) {
            const uint32_t mid = lo + ((hi - lo) >> 1);
            int c = 0;
            for (int i = tid; i < ntiles; i += FS_THREADS) c += tk[i] <= mid;
            c = __reduce_add_sync(0xffffffffu, c);
            if (lane == 0) cnt[it & 1][warp] = c;
            __syncthreads();
            int tot = 0;
#pragma unroll
            for (int w = 0; w < NW; ++w) tot += cnt[it & 1][w];
            if (tot >= ck) hi = mid; else lo = mid + 1;
            ++it;
        }
        tau = order_float(lo);
    }
    const float T = __fadd_ru(tau, 2.0f * E);

    // tiles whose minimum is inside the window
    for (int b0 = 0; b0 < ntiles; b0 += FS_THREADS) {
        const int t = b0 + tid;
        const bool in = t < ntiles && order_float(tk[t]) <= T;
        const unsigned mk = __ballot_sync(0xffffffffu, in);
        int base = 0;
        if (lane == 0 && mk) base = atomicAdd(&nhot_s, __popc(mk));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (in) hot[base + __popc(mk & lt)] = t;
    }
    __syncthreads();
    const int nhot = nhot_s;
    const float* srow = scores + (int64_t)q * nvec;
    int n = 0;                                             // exact keys in buf (block-uniform)
    for (int h0 = 0; h0 < nhot; h0 += FS_ROUND) {
        if (tid == 0) nc_s = 0;
        __syncthreads();
        // gather: warp w reads hot tiles h0 + w + 8j, all loads issued first
        float sv[FS_ROUND / NW][4];
        int tt[FS_ROUND / NW];
#pragma unroll
        for (int j = 0; j < FS_ROUND / NW; ++j) {
            const int h = h0 + warp + NW * j;
            tt[j] = h < nhot ? hot[h] : -1;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                // rows past nvec (or no tile) read NaN: never <= T, even when T = +inf
                const int v = tt[j] * FT_BM + c * 32 + lane;
                sv[j][c] = (tt[j] >= 0 && v < nvec) ? __ldg(srow + v) : __int_as_float(0x7fc00000);
            }
        }
#pragma unroll
        for (int j = 0; j < FS_ROUND / NW; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const bool in = sv[j][c] <= T;
                const unsigned mk = __ballot_sync(0xffffffffu, in);
                if (!mk) continue;
                int base = 0;
                if (lane == 0) base = atomicAdd(&nc_s, __popc(mk));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (in) cl[base + __popc(mk & lt)] = tt[j] * FT_BM + c * 32 + lane;
            }
        __syncthreads();
        const int nc = nc_s;
        // rescore: one candidate per thread, appended to buf
        for (int c0i = 0; c0i < nc; c0i += FS_THREADS) {
            if (n + FS_THREADS > FS_CAP) {                 // keep the best ck_pad
                for (int i = n + tid; i < FS_CAP; i += FS_THREADS) buf[i] = KEY_EMPTY;
                __syncthreads();
                block_bitonic_sort(buf, FS_CAP);
                n = ck_pad;
                if (tid == 0) n_s = n;
            }
            uint64_t key = KEY_EMPTY;
            if (c0i + tid < nc) {
                const int id = cl[c0i + tid];
                const uint4* cv = reinterpret_cast<const uint4*>(codes + (int64_t)id * M);
                float dist = 0.0f;
                for (int g = 0; g < M / 16; ++g) {
                    const uint4 w4 = __ldg(cv + g);
                    const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                        for (int bb = 0; bb < 4; ++bb) {
                            const int m = g * 16 + wi * 4 + bb;
                            const uint32_t b = (ws[wi] >> (bb * 8)) & 0xFFu;
                            dist = __fadd_rn(dist, __fadd_rn(tab[m * 32 + (b & 15u)],
                                                              tab[m * 32 + 16 + (b >> 4)]));
                        }
                }
                key = make_key(dist, id);
            }
            const unsigned mk = __ballot_sync(0xffffffffu, key != KEY_EMPTY);
            int base = 0;
            if (lane == 0 && mk) base = atomicAdd(&n_s, __popc(mk));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (key != KEY_EMPTY) buf[base + __popc(mk & lt)] = key;
            __syncthreads();
            n = n_s;
        }
    }
    int P = ck_pad;
    while (P < n) P <<= 1;
    for (int i = n + tid; i < P; i += FS_THREADS) buf[i] = KEY_EMPTY;
    __syncthreads();
    block_bitonic_sort(buf, P);
    for (int i = tid; i < ck; i += FS_THREADS) cand[(int64_t)q * ck + i] = buf[i];
    if (tid == 0) gthr[q] = buf[ck - 1];
}

}  // namespace

bool flat_tc_supported(int d, int M, int B, int nvec) {
    return M > 0 && d == 8 * M && B == 8 && M % 16 == 0 && ft_block_queries(d) >= 32 &&
           nvec > 0 && (nvec + FT_BM - 1) / FT_BM <= FS_TILES;
}

namespace {
// scratch carve: q8 [2][Nb][d] s8, S0 / scale / R1 [Bq], scores [Bq][nvec],
// tile_min [Bq][ntiles], each 256-byte aligned
struct FlatScratch {
    int8_t* q8;
    float *S0, *qscale, *R1, *scores;
    uint32_t* tmin;
    size_t bytes;
};
FlatScratch flat_carve(void* base, int Bq, int d, int nvec) {
    const int Nb = std::min(ft_block_queries(d), (Bq + 31) / 32 * 32);
    const int ntiles = (nvec + FT_BM - 1) / FT_BM;
    const uintptr_t p = reinterpret_cast<uintptr_t>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        void* r = reinterpret_cast<void*>(p + off);
        off += (bytes + 255) & ~size_t(255);
        return r;
    };
    FlatScratch f;
    f.q8 = reinterpret_cast<int8_t*>(take((size_t)2 * Nb * d));
    f.S0 = reinterpret_cast<float*>(take((size_t)Bq * 4));
    f.qscale = reinterpret_cast<float*>(take((size_t)Bq * 4));
    f.R1 = reinterpret_cast<float*>(take((size_t)Bq * 4));
    f.scores = reinterpret_cast<float*>(take((size_t)Bq * nvec * 4));
    f.tmin = reinterpret_cast<uint32_t*>(take((size_t)Bq * ntiles * 4));
    f.bytes = off;
    return f;
}

// [rows][K] s8 row-major, boxes of box_rows x 128 bytes, 128-byte swizzle
CUtensorMap make_map_s8(const int8_t* base, int64_t rows, int K, int box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)FT_BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)base, dims,
                                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(JHQ_EDEVICE, "flat_search_tc: tensor map encoding failed");
    return m;
}
}  // namespace

float* flat_tc_scores_of(void* scratch, int Bq, int d, int nvec) {
    return flat_carve(scratch, Bq, d, nvec).scores;
}

size_t flat_tc_scratch_bytes(int Bq, int d, int nvec) {
    return flat_carve(nullptr, Bq, d, nvec).bytes + 256;
}

void flat_search_tc(const FlatTcArgs& a, cudaStream_t s) {
    if (a.nq <= 0) return;
    const int d = a.M * 8, ntiles = (a.nvec + FT_BM - 1) / FT_BM;
    if (!flat_tc_supported(d, a.M, 8, a.nvec)) fail(JHQ_EINVAL, "flat_search_tc: unsupported shape");
    int ntiles_pad = 32;
    while (ntiles_pad < ntiles) ntiles_pad <<= 1;
    const FlatScratch f = flat_carve(a.scratch, a.nq, d, a.nvec);
    JHQ_CUDA(cudaMemsetAsync(f.tmin, 0xFF, (size_t)a.nq * ntiles * 4, s));
    static std::atomic<uint64_t> attr{0};
    once_per_device(attr, [] {
        JHQ_CUDA(cudaFuncSetAttribute(flat_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      FT_SMEM_MAX));
        JHQ_CUDA(cudaFuncSetAttribute(flat_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      FS_SMEM_MAX));
    });
    int dev = 0, nsm = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    long long wait_limit = TC_WAIT_CYCLES;
    if (const char* e = std::getenv("JHQ_TEST_TC_WAIT_CYCLES")) wait_limit = std::atoll(e);
    const float c0 = a.c1d_host[0], c1 = a.c1d_host[1];
    const float Dc = c1 * c1 - c0 * c0, ec = c1 - c0;
    const float cmax = std::max(std::fabs(c0), std::fabs(c1));
    const int NB = ft_block_queries(d);
    for (int q0 = 0; q0 < a.nq; q0 += NB) {
        const int nqb = std::min(NB, a.nq - q0);
        const int N = (nqb + 31) / 32 * 32;        // the epilogue reads 32 TMEM columns at a time
        flat_prep_kernel<<<N, 256, 0, s>>>(a.q_rot + (int64_t)q0 * d, nqb, N, d, c0, f.q8,
                                           f.S0 + q0, f.qscale + q0, f.R1 + q0);
        JHQ_LAUNCH_CHECK();
        const CUtensorMap mq = make_map_s8(f.q8, 2 * N, d, 2 * N);
        const int grid = std::min(ntiles, nsm);
        if (ft_smem_bytes(N, d) > FT_SMEM_MAX || ft_stages(N, d) < 2)
            fail(JHQ_EINVAL, "flat_search_tc: shared memory plan");
        flat_tc_kernel<<<grid, FT_THREADS, ft_smem_bytes(N, d), s>>>(
            mq, a.codes, a.pop, f.S0 + q0, f.qscale + q0, a.nvec, a.M, nqb, N, Dc, ec,
            f.scores + (int64_t)q0 * a.nvec, f.tmin + (int64_t)q0 * ntiles, ntiles, wait_limit);
        JHQ_LAUNCH_CHECK();
        count_launch(2);
    }
    if (a.scores_only) return;                     // diagnostics: the approximate scores
    const size_t smem = fs_smem_bytes(a.M, ntiles_pad);
    if (smem > (size_t)FS_SMEM_MAX) fail(JHQ_EINVAL, "flat_search_tc: selection buffers too large");
    flat_select_kernel<<<(unsigned)a.nq, FS_THREADS, smem, s>>>(
        a.q_rot, a.c1d, a.codes, f.scores, f.tmin, f.R1, a.nvec, a.M, a.nq, a.ck, a.ck_pad, ntiles,
        ntiles_pad, cmax, ec, Dc, a.cand, a.gthr, a.qslot_off, a.d_nvalid);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

#include "ivf_tc.cuh"

bool ivf_tc_supported(int d, int M, int B, int nprobe) {
    return M > 0 && d % M == 0 && d / M == 4 && B == 8 && (M + 15) / 16 * 16 * 4 == 128 &&
           nprobe >= 1 && nprobe <= 128;
}

namespace {
struct IvfScratch {
    int8_t* qw;
    float4* qc;
    int64_t* qtile;
    uint32_t* tmin;
    size_t bytes;
};
IvfScratch ivf_carve(void* base, int Bq, int64_t max_tiles) {
    const uintptr_t p = reinterpret_cast<uintptr_t>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        void* r = reinterpret_cast<void*>(p + off);
        off += (bytes + 255) & ~size_t(255);
        return r;
    };
    IvfScratch f;
    f.qw = reinterpret_cast<int8_t*>(take((size_t)Bq * 2 * IT_KP));
    f.qc = reinterpret_cast<float4*>(take((size_t)Bq * sizeof(float4)));
    f.qtile = reinterpret_cast<int64_t*>(take((size_t)(Bq + 1) * 8));
    f.tmin = reinterpret_cast<uint32_t*>(take((size_t)std::max<int64_t>(1, max_tiles) * 4));
    f.bytes = off;
    return f;
}
}  // namespace

size_t ivf_tc_scratch_bytes(int Bq, int64_t max_tiles) {
    return ivf_carve(nullptr, Bq, max_tiles).bytes + 256;
}

void ivf_search_tc(const IvfTcArgs& a, cudaStream_t s) {
    if (a.nq <= 0) return;
    if (!ivf_tc_supported(a.d, a.M, 8, a.nprobe)) fail(JHQ_EINVAL, "ivf_search_tc: unsupported shape");
    const int Mp = (a.M + 15) / 16 * 16;
    const IvfScratch f = ivf_carve(a.scratch, a.nq, a.max_tiles);
    PlanBufs pb = a.plan;
    pb.qslot_off = f.qtile;                        // tile offsets per query (the refine's stay apart)
    plan_build(a.probes, a.nq, a.nprobe, a.nlist, a.list_page_off, a.d_nvalid, 4, IT_NQ, pb, s);
    static std::atomic<uint64_t> attr{0};
    once_per_device(attr, [Mp] {
        JHQ_CUDA(cudaFuncSetAttribute(ivf_tc_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      it_smem_bytes<3>()));
        JHQ_CUDA(cudaFuncSetAttribute(ivf_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      it_smem_bytes<2>()));
        JHQ_CUDA(cudaFuncSetAttribute(ivf_tc_select_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)is_smem_bytes(128)));
    });
    int nsm0 = 0, dev0 = 0;
    JHQ_CUDA(cudaGetDevice(&dev0));
    JHQ_CUDA(cudaDeviceGetAttribute(&nsm0, cudaDevAttrMultiProcessorCount, dev0));
    const float* c = a.c1d_host;
    // a symmetric codebook (the Lloyd-Max levels are) has no L&H term: its true
    // weight is 0, and the pass-1 GEMM then runs on the L and H planes only
    const bool sym = c[0] == -c[3] && c[1] == -c[2];
    const float e1 = c[1] - c[0], e2 = c[2] - c[0], e3 = sym ? 0.0f : c[3] - c[2] - c[1] + c[0];
    float cmax = 0.0f;
    for (int i = 0; i < 4; ++i) cmax = std::max(cmax, std::fabs(c[i]));
    tmin_fill_kernel<<<4 * nsm0, 256, 0, s>>>(f.tmin, f.qtile, a.nq);
    JHQ_LAUNCH_CHECK();
    ivf_prep_kernel<<<a.nq, IP_THREADS, 0, s>>>(a.q_rot, a.nq, a.d, Mp, c[0], e1, e2, e3, cmax,
                                                f.qw, f.qc);
    JHQ_LAUNCH_CHECK();
    int dev = 0, nsm = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    long long wait_limit = TC_WAIT_CYCLES;
    if (const char* e = std::getenv("JHQ_TEST_TC_WAIT_CYCLES")) wait_limit = std::atoll(e);
    const bool two = sym && !std::getenv("JHQ_IVF_TC_3PLANES");
    auto pass1 = two ? ivf_tc_kernel<2> : ivf_tc_kernel<3>;
    const int per_sm = two ? it_ctas_per_sm<2>() : it_ctas_per_sm<3>();
    pass1<<<per_sm * nsm, IT_THREADS, two ? it_smem_bytes<2>() : it_smem_bytes<3>(), s>>>(
        a.pages, a.slot_ids, a.list_page_off, pb, f.qw, f.qc, a.nlist, a.nprobe, a.d, Mp,
        c[0] * c[0], c[1] * c[1], c[2] * c[2], c[3] * c[3], f.tmin, wait_limit);
    JHQ_LAUNCH_CHECK();
    ivf_tc_select_kernel<<<a.nq, IS_THREADS, is_smem_bytes(Mp), s>>>(
        a.q_rot, a.c1d, a.pages, a.slot_ids, a.list_page_off, a.probes, pb, f.qc, f.tmin, a.nq,
        a.nprobe, a.d, a.M, Mp, a.ck, a.ck_pad, a.cand, a.gthr, a.qslot_out, a.d_nvalid);
    JHQ_LAUNCH_CHECK();
    count_launch(4);
}

}  // namespace jhq
