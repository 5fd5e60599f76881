// ivf.cu — IVF probe selection and the page partition of the ADC scan.
//
// select_probes_kernel: exact top-nprobe lists per query (see the kernel).
//
// The plan kernels invert the (query, probe) pairs into per-list buckets and
// number the scan's work units and candidate slots (see kernels.cuh).
#include "device_utils.cuh"
#include "jhq_common.h"
#include "kernels.cuh"

#include <algorithm>
#include <mutex>

namespace jhq {
namespace {

constexpr int SP_THREADS = 512;
constexpr int SP_CAP = 4096;                 // keys held in shared memory per query
constexpr int SPM_DMAX = 2048;               // largest d of select_probes_margin
constexpr int TL_CAP = 1024;                 // candidate tiles read selectively

// Exact top-nprobe of one score row by (score, list id) — composite uint64
// keys (order-preserving score << 32 | id) make the order a plain integer one.
//  - nlist <= SP_CAP: the whole row is sorted in shared memory;
//  - otherwise the first SP_CAP scores are sorted and their nprobe-th key T is
//    an upper bound of the row's nprobe-th key, so every winner has key <= T;
//    one pass collects those keys (about nprobe * nlist / SP_CAP of them) and
//    a final sort picks the winners. If more than SP_CAP keys tie below T the
//    row falls back to a 4-pass 8-bit radix select (select_probes_radix).
// The reference's select_probes_kernel (jhq_v14_streaming_add/search.cu:13-62)
// runs nprobe block-argmin rounds over the row in shared memory and cannot
// launch above ~11.7k lists; the order here is jhq_v3_ivf/search.cu:46-85's.
__device__ void select_probes_radix(const float* row, int nlist, int nprobe, int np_pad,
                                    uint64_t* sp_buf, int32_t* out);

// Exact selection of one row into out[nprobe]; buf = SP_CAP keys of shared memory.
__device__ void select_row_exact(const float* row, int nlist, int nprobe, int32_t* out,
                                 uint64_t* buf) {
    __shared__ unsigned int cnt;
    const int tid = threadIdx.x;
    const int n0 = min(nlist, SP_CAP);
    int P = 1;
    while (P < n0) P <<= 1;
    for (int i = tid; i < P; i += SP_THREADS)
        buf[i] = i < n0 ? (((uint64_t)float_order(row[i]) << 32) | (uint32_t)i) : KEY_EMPTY;
    __syncthreads();
    block_bitonic_sort(buf, P);
    if (nlist > SP_CAP) {
        const uint64_t T = buf[nprobe - 1];
        __syncthreads();
        if (tid == 0) cnt = 0;
        __syncthreads();
        for (int c = tid; c < nlist; c += SP_THREADS) {
            const uint64_t key = ((uint64_t)float_order(row[c]) << 32) | (uint32_t)c;
            if (key <= T) {
                const unsigned int pos = atomicAdd(&cnt, 1u);
                if (pos < SP_CAP) buf[pos] = key;
            }
        }
        __syncthreads();
        const unsigned int n = cnt;
        if (n > SP_CAP) {                      // pathological ties: radix select
            int np_pad = 1;
            while (np_pad < nprobe) np_pad <<= 1;
            select_probes_radix(row, nlist, nprobe, np_pad, buf, out);
            return;
        }
        P = 1;
        while (P < (int)n) P <<= 1;
        for (int i = n + tid; i < P; i += SP_THREADS) buf[i] = KEY_EMPTY;
        __syncthreads();
        block_bitonic_sort(buf, P);
    }
    for (int p = tid; p < nprobe; p += SP_THREADS) {
        const uint64_t e = buf[p];
        out[p] = (e == KEY_EMPTY) ? 0 : (int32_t)(e & 0xffffffffu);
    }
}

__global__ void __launch_bounds__(SP_THREADS)
select_probes_kernel(const float* __restrict__ s, int nlist, int nprobe, int32_t* __restrict__ probes) {
    __shared__ uint64_t buf[SP_CAP];
    const int q = blockIdx.x;
    select_row_exact(s + (int64_t)q * nlist, nlist, nprobe, probes + (int64_t)q * nprobe, buf);
}

// 2E of select_probes_margin for |q|^2 = qn2 (the bound is derived there).
__device__ __forceinline__ float coarse_margin2(float qn2, int d, float cmax) {
    const float qn = sqrtf(qn2) * 1.001f;
    const float eps = 2.2888184e-05f + (float)d * 8.3446503e-07f;   // 6*2^-18 + d (3*2^-22 + 2^-23)
    const float E = (2.0f * eps * qn * cmax + 4.7683716e-07f * (cmax * cmax + 2.0f * qn * cmax)) *
                    1.01f;
    return 2.0f * E;
}

// The fp32 chain score norms[c] - 2 * fma-chain_j(q[j] * cent_c[j]), j ascending
// (the order of gemm_rows' EPI_COARSE and of the oracle).
__device__ __forceinline__ float exact_coarse(const float* q, const float* __restrict__ cents,
                                              const float* __restrict__ norms, int c, int d) {
    float acc = 0.0f;
    if (d % 4) {
        const float* cr = cents + (int64_t)c * d;
        for (int j = 0; j < d; ++j) acc = __fmaf_rn(q[j], cr[j], acc);
        return norms[c] - 2.0f * acc;
    }
    // eight 16-byte loads in flight per round; the fma chain stays in order
    const float4* cr = reinterpret_cast<const float4*>(cents + (int64_t)c * d);
    const int d4 = d / 4;
    for (int j0 = 0; j0 < d4; j0 += 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (j0 + u < d4) v[u] = __ldg(cr + j0 + u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (j0 + u < d4) {
                const float* qq = q + 4 * (j0 + u);
                acc = __fmaf_rn(qq[0], v[u].x, acc);
                acc = __fmaf_rn(qq[1], v[u].y, acc);
                acc = __fmaf_rn(qq[2], v[u].z, acc);
                acc = __fmaf_rn(qq[3], v[u].w, acc);
            }
        }
    }
    return norms[c] - 2.0f * acc;
}

// Exact top-nprobe from APPROXIMATE scores s~ (the tensor-core coarse GEMM,
// coarse_tc.cu). With |s~_c - s_c| <= E for every list c (s = the fp32 chain
// score norms[c] - 2 * fma-chain(q, cent_c)), and t~ the nprobe-th smallest s~:
//   a winner w has s_w <= t (the nprobe-th smallest s), and t <= t~ + E (the
//   nprobe lists with s~ <= t~ have s <= t~ + E), so s~_w <= s_w + E <= t~ + 2E.
// Hence the lists with s~ <= t~ + 2E contain every winner; they are rescored
// with the exact chain and the exact (s, list id) order picks the winners.
// E bounds, for the bf16 split of coarse_tc.cu (x = hi + lo + r with
// |r| <= 2^-18 |x|; the three bf16 products are exact in fp32 and come within
// 3 * 2^-18 |q_i c_i| of q_i c_i), fp32 accumulation of the 3d products inside
// the tensor core (at most 3d * 2^-23 of the absolute sum, allowing truncating
// adds), the fp32 chain (d * 2^-24) and the final subtractions:
//   |q3.c3 - q.c| <= (3 * 2^-18 + 3d * 2^-23 + d * 2^-24) |q| |c|, doubled for
//   safety: eps = 6 * 2^-18 + d * (3 * 2^-22 + 2^-23),
//   E = (2 eps |q| cmax + 2^-21 (cmax^2 + 2 |q| cmax)) * 1.01,
// with cmax >= max |c|. Step 1 bounds t~ by T >= t~: the nprobe-th smallest of
// the per-tile minima of s~ (nprobe distinct lists lie at or below it) when the
// GEMM supplied at least nprobe of them, else the nprobe-th smallest of the
// first SP_CAP scores. One pass then collects every s~ <= T + 2E (>= t~ + 2E),
// reading only the tiles whose minimum is within that bound when tile minima exist;
// those are sorted to find t~. If more than SP_CAP lists fall in the window the
// row is rescored in full (in place) and selected exactly.
__global__ void __launch_bounds__(SP_THREADS)
select_probes_margin_kernel(float* __restrict__ s, const float* __restrict__ q_rot,
                            const float* __restrict__ cents, const float* __restrict__ norms,
                            const float* __restrict__ tile_min, int ntiles,
                            int nlist, int d, int nprobe, float cmax,
                            int32_t* __restrict__ probes, int only_flagged) {
    if (only_flagged && probes[(int64_t)blockIdx.x * nprobe] != -1) return;
    __shared__ uint64_t buf[SP_CAP];
    __shared__ float qs[SPM_DMAX];
    __shared__ float red[SP_THREADS / 32];
    __shared__ unsigned int cnt, m_sh;
    __shared__ int tl[TL_CAP];
    const int q = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float* row = s + (int64_t)q * nlist;
    int32_t* out = probes + (int64_t)q * nprobe;
    const float* qr = q_rot + (int64_t)q * d;
    float ss = 0.0f;
    for (int j = tid; j < d; j += SP_THREADS) {
        const float v = qr[j];
        qs[j] = v;
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    if (tid == 0) { cnt = 0; m_sh = 0; }
    __syncthreads();
    float qn2 = 0.0f;
    for (int w = 0; w < SP_THREADS / 32; ++w) qn2 += red[w];
    const float twoE = coarse_margin2(qn2, d, cmax);
    auto exact = [&](int c) { return exact_coarse(qs, cents, norms, c, d); };

    const bool use_tiles = tile_min && nlist > SP_CAP && ntiles >= nprobe && ntiles <= SP_CAP;
    const float* src = use_tiles ? tile_min + (int64_t)q * ntiles : row;
    const int n0 = use_tiles ? ntiles : min(nlist, SP_CAP);
    int P = 1;
    while (P < n0) P <<= 1;
    for (int i = tid; i < P; i += SP_THREADS)
        buf[i] = i < n0 ? (((uint64_t)float_order(src[i]) << 32) | (uint32_t)i) : KEY_EMPTY;
    __syncthreads();
    block_bitonic_sort(buf, P);
    int n = n0;
    if (nlist > SP_CAP) {
        const float T = key_dist(buf[nprobe - 1]);
        const float thr = __fadd_ru(T, twoE);
        // Only tiles whose minimum is <= thr can hold a list with s~ <= thr.
        int ntc = TL_CAP + 1;
        if (use_tiles) {
            for (int i = tid; i < n0; i += SP_THREADS)
                if (key_dist(buf[i]) <= thr && (i + 1 == n0 || !(key_dist(buf[i + 1]) <= thr)))
                    m_sh = (unsigned)(i + 1);
            __syncthreads();
            ntc = (int)m_sh;
            if (ntc <= TL_CAP)
                for (int i = tid; i < ntc; i += SP_THREADS) tl[i] = key_id(buf[i]);
        }
        __syncthreads();
        auto take = [&](int c) {
            const float v = row[c];
            if (v <= thr) {
                const unsigned int pos = atomicAdd(&cnt, 1u);
                if (pos < SP_CAP) buf[pos] = ((uint64_t)float_order(v) << 32) | (uint32_t)c;
            }
        };
        if (ntc <= TL_CAP) {
            for (int e = tid; e < ntc * COARSE_TILE_LISTS; e += SP_THREADS) {
                const int c = tl[e / COARSE_TILE_LISTS] * COARSE_TILE_LISTS + e % COARSE_TILE_LISTS;
                if (c < nlist) take(c);
            }
        } else {
            for (int c = tid; c < nlist; c += SP_THREADS) take(c);
        }
        __syncthreads();
        if (tid == 0) m_sh = 0;
        n = (int)cnt;
        if (n > SP_CAP) {                      // window too wide: rescore the row exactly
            for (int c = tid; c < nlist; c += SP_THREADS) row[c] = exact(c);
            __syncthreads();
            select_row_exact(row, nlist, nprobe, out, buf);
            return;
        }
        P = 1;
        while (P < n) P <<= 1;
        for (int i = n + tid; i < P; i += SP_THREADS) buf[i] = KEY_EMPTY;
        __syncthreads();
        block_bitonic_sort(buf, P);
    }
    const float thr2 = __fadd_ru(key_dist(buf[nprobe - 1]), twoE);
    for (int i = tid; i < n; i += SP_THREADS)
        if (key_dist(buf[i]) <= thr2 && (i + 1 == n || !(key_dist(buf[i + 1]) <= thr2)))
            m_sh = (unsigned)(i + 1);
    __syncthreads();
    const int m = (int)m_sh;
    for (int i = tid; i < m; i += SP_THREADS) {
        const int c = key_id(buf[i]);
        buf[i] = ((uint64_t)float_order(exact(c)) << 32) | (uint32_t)c;
    }
    P = 1;
    while (P < m) P <<= 1;
    for (int i = m + tid; i < P; i += SP_THREADS) buf[i] = KEY_EMPTY;
    __syncthreads();
    block_bitonic_sort(buf, P);
    for (int p = tid; p < nprobe; p += SP_THREADS) {
        const uint64_t e = buf[p];
        out[p] = (e == KEY_EMPTY) ? 0 : (int32_t)(e & 0xffffffffu);
    }
}

// One warp per query for the common case of select_probes_margin_kernel
// (group minima present, at most SW_CAP groups and SW_CAP collected lists):
// the same steps with warp-synchronous sorts in shared memory and ballot-based
// appends. A query whose window holds more than SW_CAP lists is flagged
// (probes[q][0] = -1) and finished by the block kernel.
constexpr int SW_WARPS = 8;
constexpr int SW_CAP = 512;

__global__ void __launch_bounds__(SW_WARPS * 32)
select_probes_margin_warp_kernel(const float* __restrict__ s, const float* __restrict__ q_rot,
                                 const float* __restrict__ cents, const float* __restrict__ norms,
                                 const float* __restrict__ tile_min, int ngr, int nq, int nlist,
                                 int d, int nprobe, float cmax, int32_t* __restrict__ probes) {
    extern __shared__ uint64_t sw_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * SW_WARPS + warp;
    if (q >= nq) return;                                   // warp-uniform; no block barriers below
    uint64_t* gb = sw_smem + (size_t)warp * 2 * SW_CAP;    // group minima, sorted
    uint64_t* cb = gb + SW_CAP;                            // collected lists
    const float* qr = q_rot + (int64_t)q * d;
    const float* row = s + (int64_t)q * nlist;
    int32_t* out = probes + (int64_t)q * nprobe;
    const unsigned lt = (1u << lane) - 1u;
    float ss = 0.0f;
    for (int j = lane; j < d; j += 32) {
        const float v = qr[j];
        ss += v * v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float twoE = coarse_margin2(ss, d, cmax);

    int P = 32;
    while (P < ngr) P <<= 1;
    const float* tm = tile_min + (int64_t)q * ngr;
    for (int i0 = 0; i0 < P; i0 += 128) {                 // four loads in flight per lane
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = i0 + 32 * u + lane;
            x[u] = i < ngr ? tm[i] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = i0 + 32 * u + lane;
            if (i < P) gb[i] = i < ngr ? (((uint64_t)float_order(x[u]) << 32) | (uint32_t)i) : KEY_EMPTY;
        }
    }
    __syncwarp();
    warp_bitonic_sort(gb, P, lane);
    const float thr = __fadd_ru(key_dist(gb[nprobe - 1]), twoE);
    int ntc = 0;                                           // sorted: groups with min <= thr lead
    for (int base = 0; base < ngr; base += 32) {
        const int i = base + lane;
        const unsigned b = __ballot_sync(0xffffffffu, i < ngr && key_dist(gb[i]) <= thr);
        ntc += __popc(b);
        if (b != 0xffffffffu) break;
    }
    // groups 8 at a time, lane l holding lists 4l..4l+3 of each (loads in flight together)
    static_assert(COARSE_TILE_LISTS == 128, "one 16-byte load per lane per group");
    const bool vec = (nlist & 3) == 0;
    const float inf = __int_as_float(0x7f800000);
    int cnt = 0;
    for (int t0 = 0; t0 < ntc; t0 += 8) {
        float4 v[8];
        int cc[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            cc[u] = t0 + u < ntc ? key_id(gb[t0 + u]) * COARSE_TILE_LISTS + 4 * lane : nlist;
            const int c = cc[u];
            if (vec && c + 3 < nlist) {
                v[u] = __ldcs(reinterpret_cast<const float4*>(row + c));
            } else {
                v[u].x = c < nlist ? row[c] : inf;
                v[u].y = c + 1 < nlist ? row[c + 1] : inf;
                v[u].z = c + 2 < nlist ? row[c + 2] : inf;
                v[u].w = c + 3 < nlist ? row[c + 3] : inf;
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float x = e == 0 ? v[u].x : e == 1 ? v[u].y : e == 2 ? v[u].z : v[u].w;
                const bool in = cc[u] + e < nlist && x <= thr;
                const unsigned b = __ballot_sync(0xffffffffu, in);
                const int pos = cnt + __popc(b & lt);
                if (in && pos < SW_CAP)
                    cb[pos] = ((uint64_t)float_order(x) << 32) | (uint32_t)(cc[u] + e);
                cnt += __popc(b);
            }
        }
    }
    if (cnt > SW_CAP) {
        if (lane == 0) out[0] = -1;                        // left to the block kernel
        return;
    }
    P = 32;
    while (P < cnt) P <<= 1;
    for (int i = cnt + lane; i < P; i += 32) cb[i] = KEY_EMPTY;
    __syncwarp();
    warp_bitonic_sort(cb, P, lane);
    const float thr2 = __fadd_ru(key_dist(cb[nprobe - 1]), twoE);
    int m = 0;
    for (int base = 0; base < cnt; base += 32) {
        const int i = base + lane;
        const unsigned b = __ballot_sync(0xffffffffu, i < cnt && key_dist(cb[i]) <= thr2);
        m += __popc(b);
        if (b != 0xffffffffu) break;
    }
    for (int i = lane; i < m; i += 32) {
        const int c = key_id(cb[i]);
        cb[i] = ((uint64_t)float_order(exact_coarse(qr, cents, norms, c, d)) << 32) | (uint32_t)c;
    }
    int P3 = 32;
    while (P3 < m) P3 <<= 1;
    for (int i = m + lane; i < P3; i += 32) cb[i] = KEY_EMPTY;
    __syncwarp();
    warp_bitonic_sort(cb, P3, lane);
    for (int p = lane; p < nprobe; p += 32) {
        const uint64_t e = cb[p];                          // never -1: a list id in range
        out[p] = (e == KEY_EMPTY) ? 0 : key_id(e);
    }
}

// 4-pass 8-bit radix select of the nprobe-th key, then the winners (ties at
// the threshold taken in ascending list id), sorted. Uses sp_buf[np_pad].
__device__ void select_probes_radix(const float* row, int nlist, int nprobe, int np_pad,
                                    uint64_t* sp_buf, int32_t* out) {
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sh_prefix, sh_rank, sh_nbuf, sh_eq_taken;
    __shared__ uint32_t warp_eq[SP_THREADS / 32];
    const int tid = threadIdx.x;
    __syncthreads();
    uint32_t prefix = 0, pmask = 0;
    uint32_t rank = (uint32_t)nprobe;               // 1-based rank of the threshold
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += SP_THREADS) hist[i] = 0;
        __syncthreads();
        for (int c = tid; c < nlist; c += SP_THREADS) {
            uint32_t k = float_order(row[c]);
            if ((k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t acc = 0;
            int dgt = 0;
            for (; dgt < 256; ++dgt) {
                if (acc + hist[dgt] >= rank) break;
                acc += hist[dgt];
            }
            sh_prefix = prefix | ((uint32_t)dgt << shift);
            sh_rank = rank - acc;
        }
        __syncthreads();
        prefix = sh_prefix;
        rank = sh_rank;
        pmask |= 255u << shift;
        __syncthreads();
    }
    const uint32_t T = prefix;                       // key of the nprobe-th smallest
    // rank = how many entries equal to T are needed (lowest list ids first)
    if (tid == 0) { sh_nbuf = 0; sh_eq_taken = 0; }
    for (int i = tid; i < np_pad; i += SP_THREADS) sp_buf[i] = KEY_EMPTY;
    __syncthreads();
    const uint32_t need_eq = rank;
    const int lane = tid & 31, warp = tid / 32;
    for (int base = 0; base < nlist; base += SP_THREADS) {
        int c = base + tid;
        uint32_t k = (c < nlist) ? float_order(row[c]) : 0xffffffffu;
        bool less = c < nlist && k < T;
        bool eq = c < nlist && k == T;
        if (less) {
            uint32_t pos = atomicAdd(&sh_nbuf, 1u);
            sp_buf[pos] = ((uint64_t)k << 32) | (uint32_t)c;
        }
        // equal keys taken in ascending c order
        unsigned eb = __ballot_sync(0xffffffffu, eq);
        if (lane == 0) warp_eq[warp] = __popc(eb);
        __syncthreads();
        uint32_t before = sh_eq_taken;
        for (int w = 0; w < warp; ++w) before += warp_eq[w];
        before += __popc(eb & ((1u << lane) - 1u));
        if (eq && before < need_eq) {
            uint32_t pos = atomicAdd(&sh_nbuf, 1u);
            sp_buf[pos] = ((uint64_t)k << 32) | (uint32_t)c;
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t tot = 0;
            for (int w = 0; w < SP_THREADS / 32; ++w) tot += warp_eq[w];
            sh_eq_taken += tot;
        }
        __syncthreads();
    }
    block_bitonic_sort(sp_buf, np_pad);
    for (int p = tid; p < nprobe; p += SP_THREADS) {
        uint64_t e = sp_buf[p];
        out[p] = (e == KEY_EMPTY) ? 0 : (int32_t)(e & 0xffffffffu);
    }
}

constexpr int PLAN_THREADS = 1024;

__device__ __forceinline__ int chunks_of(const int32_t* lpo, int l, int chunk_pages) {
    return (lpo[l + 1] - lpo[l] + chunk_pages - 1) / chunk_pages;
}

// Per pair: count per list. Per query: chunk prefix over its probes, slot
// count (into qslot_off[q+1]) and a fresh pruning bound.
__global__ void plan_count_kernel(const int32_t* __restrict__ probes, int nq, int nprobe,
                                  const int32_t* __restrict__ lpo, const int* __restrict__ d_nvalid,
                                  int chunk_pages, PlanBufs b) {
    const int nvalid = d_nvalid ? *d_nvalid : nq;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < (int64_t)nq * nprobe) {
        const int q = (int)(t / nprobe);
        if (q < nvalid) atomicAdd(&b.cnt[probes[t]], 1);
    }
    if (t < nq) {
        const int q = (int)t;
        int32_t* po = b.cpo + (int64_t)q * (nprobe + 1);
        int acc = 0;
        po[0] = 0;
        for (int p = 0; p < nprobe; ++p) {
            if (q < nvalid) acc += chunks_of(lpo, probes[(int64_t)q * nprobe + p], chunk_pages);
            po[p + 1] = acc;
        }
        b.qslot_off[q + 1] = acc;
        b.gthr[q] = KEY_EMPTY;
    }
}

// Exclusive scan of value_of(0..n) into out[0..n) with one block (warp
// shuffles inside a warp, one shared round across warps); returns the total.
template <class T, class F>
__device__ T block_exclusive_scan(int n, F&& value_of, T* out) {
    __shared__ T wsum[PLAN_THREADS / 32];
    __shared__ T carry;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < n; base += PLAN_THREADS) {
        const int i = base + threadIdx.x;
        const T v = i < n ? value_of(i) : T(0);
        T x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const T y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[warp] = x;
        __syncthreads();
        if (warp == 0) {
            T t = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const T y = __shfl_up_sync(0xffffffffu, t, o);
                if (lane >= o) t += y;
            }
            wsum[lane] = t;                    // inclusive over warps
        }
        __syncthreads();
        const T before = carry + (warp ? wsum[warp - 1] : T(0));
        if (i < n) out[i] = before + x - v;
        __syncthreads();
        if (threadIdx.x == 0) carry += wsum[PLAN_THREADS / 32 - 1];
        __syncthreads();
    }
    return carry;
}

__global__ void __launch_bounds__(PLAN_THREADS)
plan_scan_kernel(int nq, int nlist, const int32_t* __restrict__ lpo, int chunk_pages, int qg,
                 PlanBufs b) {
    const int32_t nb = block_exclusive_scan<int32_t>(nlist, [&](int l) { return b.cnt[l]; },
                                                     b.bucket_off);
    if (threadIdx.x == 0) b.bucket_off[nlist] = nb;
    const int32_t nu = block_exclusive_scan<int32_t>(nlist, [&](int l) {
        const int c = b.cnt[l];
        return c ? ((c + qg - 1) / qg) * chunks_of(lpo, l, chunk_pages) : 0;
    }, b.unit_off);
    if (threadIdx.x == 0) b.unit_off[nlist] = nu;
    for (int l = threadIdx.x; l < nlist; l += PLAN_THREADS) b.fill[l] = b.bucket_off[l];
    // qslot_off[q+1] holds the count of query q: turn it into offsets
    const int64_t ns = block_exclusive_scan<int64_t>(nq, [&](int q) { return b.qslot_off[q + 1]; },
                                                     b.qslot_off);
    if (threadIdx.x == 0) b.qslot_off[nq] = ns;
}

__global__ void plan_fill_kernel(const int32_t* __restrict__ probes, int nq, int nprobe,
                                 const int* __restrict__ d_nvalid, PlanBufs b) {
    const int nvalid = d_nvalid ? *d_nvalid : nq;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)nq * nprobe) return;
    const int q = (int)(t / nprobe), p = (int)(t % nprobe);
    if (q >= nvalid) return;
    const int pos = atomicAdd(&b.fill[probes[t]], 1);
    b.bucket[pos] = make_int2(q, p);
}

}  // namespace

void select_probes(const float* s, int nq, int nlist, int nprobe, int32_t* probes,
                   cudaStream_t st) {
    if (nq <= 0) return;
    if (nprobe > SP_CAP) fail(JHQ_EINVAL, "select_probes: nprobe too large");
    select_probes_kernel<<<nq, SP_THREADS, 0, st>>>(s, nlist, nprobe, probes);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void select_probes_margin(float* s, const float* q_rot, const float* cents, const float* norms,
                          const float* tile_min, int ntiles, int nq, int nlist, int d, int nprobe,
                          float cmax, int32_t* probes, cudaStream_t st) {
    if (nq <= 0) return;
    if (nprobe > SP_CAP || nprobe > nlist) fail(JHQ_EINVAL, "select_probes_margin: bad nprobe");
    if (d > SPM_DMAX) fail(JHQ_EINVAL, "select_probes_margin: unsupported d");
    if (tile_min && ntiles >= nprobe && ntiles <= SW_CAP && nprobe <= SW_CAP && nlist > SP_CAP) {
        const size_t smem = (size_t)SW_WARPS * 2 * SW_CAP * sizeof(uint64_t);
        static std::atomic<uint64_t> attr{0};
        once_per_device(attr, [smem] {
            JHQ_CUDA(cudaFuncSetAttribute(select_probes_margin_warp_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        });
        select_probes_margin_warp_kernel<<<(nq + SW_WARPS - 1) / SW_WARPS, SW_WARPS * 32, smem, st>>>(
            s, q_rot, cents, norms, tile_min, ntiles, nq, nlist, d, nprobe, cmax, probes);
        JHQ_LAUNCH_CHECK();
        count_launch();
        select_probes_margin_kernel<<<nq, SP_THREADS, 0, st>>>(s, q_rot, cents, norms, tile_min,
                                                               ntiles, nlist, d, nprobe, cmax,
                                                               probes, 1);
    } else {
        select_probes_margin_kernel<<<nq, SP_THREADS, 0, st>>>(s, q_rot, cents, norms, tile_min,
                                                               ntiles, nlist, d, nprobe, cmax,
                                                               probes, 0);
    }
    JHQ_LAUNCH_CHECK();
    count_launch();
}

namespace {

// Per query: page prefix over its probes, item count, fresh bound.
__global__ void plan_qmajor_kernel(const int32_t* __restrict__ probes, int nq, int nprobe,
                                   const int32_t* __restrict__ lpo, const int* __restrict__ d_nvalid,
                                   int item_pages, PlanBufs b) {
    const int nvalid = d_nvalid ? *d_nvalid : nq;
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    int32_t* po = b.cpo + (int64_t)q * (nprobe + 1);
    int acc = 0;
    po[0] = 0;
    for (int p = 0; p < nprobe; ++p) {
        if (q < nvalid) {
            const int l = probes[(int64_t)q * nprobe + p];
            acc += lpo[l + 1] - lpo[l];
        }
        po[p + 1] = acc;
    }
    b.qslot_off[q + 1] = (acc + item_pages - 1) / item_pages;
    b.gthr[q] = KEY_EMPTY;
}

__global__ void __launch_bounds__(PLAN_THREADS)
plan_qmajor_scan_kernel(int nq, PlanBufs b) {
    const int64_t ns = block_exclusive_scan<int64_t>(nq, [&](int q) { return b.qslot_off[q + 1]; },
                                                     b.qslot_off);
    if (threadIdx.x == 0) b.qslot_off[nq] = ns;
}

}  // namespace

void plan_build_qmajor(const int32_t* probes, int nq, int nprobe, const int32_t* list_page_off,
                       const int* d_nvalid, int item_pages, const PlanBufs& b, cudaStream_t st) {
    if (nq <= 0) return;
    plan_qmajor_kernel<<<(unsigned)ceil_div(nq, 256), 256, 0, st>>>(probes, nq, nprobe,
                                                                   list_page_off, d_nvalid,
                                                                   item_pages, b);
    JHQ_LAUNCH_CHECK();
    plan_qmajor_scan_kernel<<<1, PLAN_THREADS, 0, st>>>(nq, b);
    JHQ_LAUNCH_CHECK();
    count_launch(2);
}

void plan_build(const int32_t* probes, int nq, int nprobe, int nlist,
                const int32_t* list_page_off, const int* d_nvalid, int chunk_pages, int qg,
                const PlanBufs& b, cudaStream_t st) {
    if (nq <= 0) return;
    JHQ_CUDA(cudaMemsetAsync(b.cnt, 0, (size_t)(nlist + 1) * sizeof(int32_t), st));
    const int64_t pairs = std::max<int64_t>((int64_t)nq * nprobe, nq);
    plan_count_kernel<<<(unsigned)ceil_div(pairs, 256), 256, 0, st>>>(
        probes, nq, nprobe, list_page_off, d_nvalid, chunk_pages, b);
    JHQ_LAUNCH_CHECK();
    plan_scan_kernel<<<1, PLAN_THREADS, 0, st>>>(nq, nlist, list_page_off, chunk_pages, qg, b);
    JHQ_LAUNCH_CHECK();
    plan_fill_kernel<<<(unsigned)ceil_div((int64_t)nq * nprobe, 256), 256, 0, st>>>(
        probes, nq, nprobe, d_nvalid, b);
    JHQ_LAUNCH_CHECK();
    count_launch(3);
}

}  // namespace jhq
