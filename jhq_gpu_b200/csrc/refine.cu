// refine.cu — per query: merge the scan's candidate slots into the exact
// top-ck, refine them with the Br-bit residual code and return the top-k.
// Replaces build_residual_lut_batched_kernel + residual_refine_batched_kernel
// + batched_topk_final_kernel of the reference (jhq_v14_streaming_add/
// search.cu:198-291) with one kernel, one CTA per query:
//   1. the scan wrote one sorted top-ck list per (probe, chunk) of query q into
//      its slots; the keys at or below the query's final bound are gathered and
//      sorted (slot-by-slot bitonic merges when ties make them too many);
//   2. warp per candidate: lane l reads 16-byte chunks l, l+32, ... of the
//      candidate's residual row (coalesced), accumulates (q_j - res_c1d[r_j])^2
//      as an in-order fma chain, and the warp reduces with an xor butterfly
//      (offsets 16..1) — the order fixed in oracle/jhq_oracle.c;
//      comp = (primary + residual) + corr (search.cu:240);
//   3. block bitonic sort of the ck composite keys; the first k are written,
//      missing ones as (+inf, -1) (search.cu:285-286).
//   4. (exact rerank, when the index keeps its vectors) the first kr composite
//      keys are re-scored by exact L2 against the stored vectors — warp per
//      candidate, lane l takes float4 chunks l, l+32, ... of the row as an
//      in-order fma chain, xor butterfly 16..1 — and the k smallest (distance,
//      id) keys are written instead. This is the exact L2 rerank over stored
//      vectors of the reference's hblock indexes (hblock_v34/search.cu:531-690)
//      applied behind the JHQ refine.
#include <cstdlib>
#include <cstring>

#include "device_utils.cuh"
#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {
namespace {

constexpr int RF_THREADS = 512;
constexpr int RF_WARPS = RF_THREADS / 32;
constexpr int RF_CAP = 2048;          // gathered candidates kept for the sort

__global__ void __launch_bounds__(RF_THREADS)
refine_kernel(RefineArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t* top = reinterpret_cast<uint64_t*>(smem);            // 2 * ck_pad
    uint64_t* comp = top + 2 * a.ck_pad;                           // ck_pad
    uint64_t* buf = comp + a.ck_pad;                               // RF_CAP
    int* nbuf = reinterpret_cast<int*>(buf + RF_CAP);              // 1 (16 bytes reserved)
    // q_rot padded by one float per 32: lane l reads dims 32l.. of its chunk,
    // and the padding puts the 32 lanes in 32 different banks.
    float* qs = reinterpret_cast<float*>(buf + RF_CAP + 2);        // d + d/32 + 1
    float* rc1d = qs + a.d + a.d / 32 + 1;                         // nres (Kr, or M*Kr)
    const int Kr = 1 << a.Br;
    const int nres = a.res_per_sub ? a.M * Kr : Kr;
    float* qraw = qs + ((a.d + a.d / 32 + 1 + nres + 3) & ~3);     // d (rerank only), 16-byte aligned

    const int q = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (q >= a.nq) return;
    for (int i = tid; i < a.ck_pad; i += RF_THREADS) top[i] = KEY_EMPTY;
    for (int i = tid; i < a.d; i += RF_THREADS) qs[i + (i >> 5)] = a.q_rot[(int64_t)q * a.d + i];
    for (int i = tid; i < nres; i += RF_THREADS) rc1d[i] = a.res_c1d[i];
    if (a.raw)
        for (int i = tid; i < a.d; i += RF_THREADS) qraw[i] = a.q_raw[(int64_t)q * a.d + i];
    __syncthreads();

    // candidates of query q: its slots [qslot_off[q], qslot_off[q+1]), ck keys
    // each. Keys above the query's final bound gthr[q] cannot be in its top-ck
    // (ck keys <= gthr[q] sit in one slot), so only the others are gathered.
    const int64_t s0 = a.qslot_off[q], s1 = a.qslot_off[q + 1];
    const uint64_t bound = a.gthr[q];
    if (tid == 0) *nbuf = 0;
    __syncthreads();
    const int64_t nkeys = (s1 - s0) * a.ck;
    const uint64_t* src = a.cand + s0 * a.ck;
    for (int64_t i = tid; i < nkeys; i += RF_THREADS) {
        const uint64_t key = src[i];
        if (key != KEY_EMPTY && key <= bound) {
            const int pos = atomicAdd(nbuf, 1);
            if (pos < RF_CAP) buf[pos] = key;
        }
    }
    __syncthreads();
    const int n = *nbuf;
    if (n <= RF_CAP) {
        int P = a.ck_pad;
        while (P < n) P <<= 1;
        for (int i = n + tid; i < P; i += RF_THREADS) buf[i] = KEY_EMPTY;
        __syncthreads();
        block_bitonic_sort(buf, P);
        for (int i = tid; i < a.ck_pad; i += RF_THREADS) top[i] = buf[i];
        __syncthreads();
    } else {                                   // many ties at the bound: merge slot by slot
        for (int64_t sl = s0; sl < s1; ++sl) {
            const uint64_t* sp = a.cand + sl * a.ck;
            for (int i = tid; i < a.ck_pad; i += RF_THREADS)
                top[a.ck_pad + i] = (i < a.ck) ? sp[i] : KEY_EMPTY;
            __syncthreads();
            block_merge_halves(top, a.ck_pad);
        }
    }

    // residual refine, warp per candidate
    const int chunks = a.bpv_pad / 16, dpw = 32 / a.Br, mask = Kr - 1;
    const int Ds = a.d / a.M;
    for (int i = warp; i < a.ck_pad; i += RF_WARPS) {
        const uint64_t key = (i < a.ck) ? top[i] : KEY_EMPTY;
        if (key == KEY_EMPTY) {
            if (lane == 0) comp[i] = KEY_EMPTY;
            continue;
        }
        const int id = key_id(key);
        const uint4* row = reinterpret_cast<const uint4*>(a.rcodes + (int64_t)id * a.bpv_pad);
        float acc = 0.0f;
        for (int c = lane; c < chunks; c += 32) {
            const uint4 v = __ldg(row + c);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                for (int t = 0; t < dpw; ++t) {
                    const int j = (c * 4 + w) * dpw + t;
                    if (j >= a.d) break;
                    const int cb = a.res_per_sub ? (j / Ds) * Kr : 0;
                    const float diff = qs[j + (j >> 5)] - rc1d[cb + ((wv[w] >> (t * a.Br)) & mask)];
                    acc = __fmaf_rn(diff, diff, acc);
                }
            }
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) {
            const float c = __fadd_rn(__fadd_rn(key_dist(key), acc), __ldg(a.corr + id));
            comp[i] = make_key(c, id);
        }
    }
    __syncthreads();
    block_bitonic_sort(comp, a.ck_pad);
    uint64_t* fin = comp;
    if (a.raw) {                               // exact rerank of the kr best
        int kr_pad = 32;
        while (kr_pad < a.kr) kr_pad <<= 1;
        const float4* q4 = reinterpret_cast<const float4*>(qraw);
        const int c4 = a.d / 4;
        for (int i = warp; i < kr_pad; i += RF_WARPS) {
            const uint64_t key = (i < a.kr) ? comp[i] : KEY_EMPTY;
            if (key == KEY_EMPTY) {
                if (lane == 0) buf[i] = KEY_EMPTY;
                continue;
            }
            const int id = key_id(key);
            const float4* row = reinterpret_cast<const float4*>(a.raw + (int64_t)id * a.d);
            float acc = 0.0f;
            for (int c = lane; c < c4; c += 32) {
                const float4 v = __ldg(row + c), w = q4[c];
                float t = w.x - v.x; acc = __fmaf_rn(t, t, acc);
                t = w.y - v.y; acc = __fmaf_rn(t, t, acc);
                t = w.z - v.z; acc = __fmaf_rn(t, t, acc);
                t = w.w - v.w; acc = __fmaf_rn(t, t, acc);
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
            if (lane == 0) buf[i] = make_key(acc, id);
        }
        __syncthreads();
        block_bitonic_sort(buf, kr_pad);
        fin = buf;
    }
    for (int i = tid; i < a.k; i += RF_THREADS) {
        const uint64_t key = fin[i];
        const bool ok = key != KEY_EMPTY;
        a.out_dists[(int64_t)q * a.k + i] = ok ? key_dist(key) : __int_as_float(0x7f800000);
        a.out_ids[(int64_t)q * a.k + i] = ok ? key_id(key) : -1;
    }
}

// ---------------------------------------------------------------------------
// Warp-per-query refine (8 queries per CTA, no block-wide synchronisation),
// used when the top-ck fits a warp's shared region (ck_pad <= 128). Same
// arithmetic as refine_kernel: the residual distance of a candidate is the
// 32-lane chunk partial sums joined by the xor butterfly; for short residual
// rows (fewer than 16 chunks of 16 bytes) one lane computes a whole candidate,
// forming the same 32 partials and the same butterfly tree (lane 0's path:
// p[l] + p[l^16], then ^8, ^4, ^2, ^1), so the result is bit-identical.
constexpr int RW_WARPS = 8;
constexpr int RW_CAP = 256;                // gathered keys per warp before a compaction

__device__ __forceinline__ float butterfly_lane0(float (&p)[32]) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
        for (int l = 0; l < o; ++l) p[l] = __fadd_rn(p[l], p[l + o]);
    return p[0];
}

__global__ void __launch_bounds__(RW_WARPS * 32)
refine_warp_kernel(RefineArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int Kr = 1 << a.Br;
    const int nres = a.res_per_sub ? a.M * Kr : Kr;
    // shared: rc1d [nres], then per warp: buf [RW_CAP] keys, comp [ck_pad] keys,
    // q_rot [d], q_raw [d] (rerank)
    float* rc1d = reinterpret_cast<float*>(smem);
    const size_t per_warp = (size_t)(RW_CAP + a.ck_pad) * 8 + (size_t)a.d * 4 * (a.raw ? 2 : 1);
    unsigned char* wbase = smem + (((size_t)nres * 4 + 15) & ~size_t(15)) + warp * ((per_warp + 15) & ~size_t(15));
    uint64_t* buf = reinterpret_cast<uint64_t*>(wbase);
    uint64_t* comp = buf + RW_CAP;
    float* qs = reinterpret_cast<float*>(comp + a.ck_pad);
    float* qraw = qs + a.d;
    for (int i = threadIdx.x; i < nres; i += blockDim.x) rc1d[i] = a.res_c1d[i];
    __syncthreads();
    const int q = blockIdx.x * RW_WARPS + warp;
    if (q >= a.nq) return;
    for (int i = lane; i < a.d; i += 32) qs[i] = a.q_rot[(int64_t)q * a.d + i];
    if (a.raw)
        for (int i = lane; i < a.d; i += 32) qraw[i] = a.q_raw[(int64_t)q * a.d + i];

    // 1. gather the keys at or below the query's final bound (ballot append);
    //    when the buffer fills, sort it and keep its best ck_pad (rare: ties)
    const int64_t s0 = a.qslot_off[q], s1 = a.qslot_off[q + 1];
    uint64_t bound = a.gthr[q];
    const int64_t nkeys = (s1 - s0) * a.ck;
    const uint64_t* src = a.cand + s0 * a.ck;
    int n = 0;
    for (int64_t base = 0; base < nkeys; base += 32) {
        const int64_t i = base + lane;
        const uint64_t key = i < nkeys ? src[i] : KEY_EMPTY;
        const bool take = key != KEY_EMPTY && key <= bound;
        const unsigned m = __ballot_sync(0xffffffffu, take);
        if (m == 0) continue;
        if (n + __popc(m) > RW_CAP) {
            for (int t = n + lane; t < RW_CAP; t += 32) buf[t] = KEY_EMPTY;
            __syncwarp();
            warp_bitonic_sort(buf, RW_CAP, lane);
            n = a.ck_pad;
            const uint64_t kth = buf[a.ck - 1];
            bound = kth < bound ? kth : bound;
        }
        const bool take2 = key != KEY_EMPTY && key <= bound;
        const unsigned m2 = __ballot_sync(0xffffffffu, take2);
        if (take2) buf[n + __popc(m2 & ((1u << lane) - 1u))] = key;
        n += __popc(m2);
        __syncwarp();
    }
    // pad to at least ck_pad: buf[0..ck) is read below even when fewer keys came in
    int P = a.ck_pad;
    while (P < n) P <<= 1;
    for (int t = n + lane; t < P; t += 32) buf[t] = KEY_EMPTY;
    __syncwarp();
    warp_bitonic_sort(buf, P, lane);             // buf[0..ck) = exact top-ck

    // 2. residual refine: comp = (primary + residual) + corr
    const int chunks = a.bpv_pad / 16, dpw = 32 / a.Br, mask = Kr - 1, Ds = a.d / a.M;
    if (chunks >= 16) {                          // warp per candidate (lane = chunk)
        for (int i = 0; i < a.ck_pad; ++i) {
            const uint64_t key = i < a.ck ? buf[i] : KEY_EMPTY;
            if (key == KEY_EMPTY) {
                if (lane == 0) comp[i] = KEY_EMPTY;
                continue;
            }
            const int id = key_id(key);
            const uint4* row = reinterpret_cast<const uint4*>(a.rcodes + (int64_t)id * a.bpv_pad);
            float acc = 0.0f;
            for (int c = lane; c < chunks; c += 32) {
                const uint4 v = __ldg(row + c);
                const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int w = 0; w < 4; ++w)
                    for (int t = 0; t < dpw; ++t) {
                        const int j = (c * 4 + w) * dpw + t;
                        if (j >= a.d) break;
                        const int cb = a.res_per_sub ? (j / Ds) * Kr : 0;
                        const float diff = qs[j] - rc1d[cb + ((wv[w] >> (t * a.Br)) & mask)];
                        acc = __fmaf_rn(diff, diff, acc);
                    }
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
            if (lane == 0)
                comp[i] = make_key(__fadd_rn(__fadd_rn(key_dist(key), acc), __ldg(a.corr + id)), id);
        }
    } else {                                     // lane per candidate, the same partials and tree
        for (int i = lane; i < a.ck_pad; i += 32) {
            const uint64_t key = i < a.ck ? buf[i] : KEY_EMPTY;
            if (key == KEY_EMPTY) { comp[i] = KEY_EMPTY; continue; }
            const int id = key_id(key);
            const uint4* row = reinterpret_cast<const uint4*>(a.rcodes + (int64_t)id * a.bpv_pad);
            float p[32];
#pragma unroll
            for (int l = 0; l < 32; ++l) p[l] = 0.0f;
#pragma unroll
            for (int c = 0; c < 16; ++c) {           // chunks < 16: chunk c is lane c's only one
                if (c >= chunks) break;
                const uint4 v = __ldg(row + c);
                const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
                float acc = 0.0f;
#pragma unroll
                for (int w = 0; w < 4; ++w)
                    for (int t = 0; t < dpw; ++t) {
                        const int j = (c * 4 + w) * dpw + t;
                        if (j >= a.d) break;
                        const int cb = a.res_per_sub ? (j / Ds) * Kr : 0;
                        const float diff = qs[j] - rc1d[cb + ((wv[w] >> (t * a.Br)) & mask)];
                        acc = __fmaf_rn(diff, diff, acc);
                    }
                p[c] = acc;
            }
            const float r = butterfly_lane0(p);
            comp[i] = make_key(__fadd_rn(__fadd_rn(key_dist(key), r), __ldg(a.corr + id)), id);
        }
    }
    __syncwarp();
    warp_bitonic_sort(comp, a.ck_pad, lane);
    uint64_t* fin = comp;
    if (a.raw) {                                 // 3. exact rerank of the kr best (warp per candidate)
        int kr_pad = 32;
        while (kr_pad < a.kr) kr_pad <<= 1;
        const int c4 = a.d / 4;
        const float4* q4 = reinterpret_cast<const float4*>(qraw);
        for (int i = 0; i < kr_pad; ++i) {
            const uint64_t key = i < a.kr ? comp[i] : KEY_EMPTY;
            if (key == KEY_EMPTY) {
                if (lane == 0) buf[i] = KEY_EMPTY;
                continue;
            }
            const int id = key_id(key);
            const float4* row = reinterpret_cast<const float4*>(a.raw + (int64_t)id * a.d);
            float acc = 0.0f;
            for (int c = lane; c < c4; c += 32) {
                const float4 v = __ldg(row + c), w = q4[c];
                float t = w.x - v.x; acc = __fmaf_rn(t, t, acc);
                t = w.y - v.y; acc = __fmaf_rn(t, t, acc);
                t = w.z - v.z; acc = __fmaf_rn(t, t, acc);
                t = w.w - v.w; acc = __fmaf_rn(t, t, acc);
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
            if (lane == 0) buf[i] = make_key(acc, id);
        }
        __syncwarp();
        warp_bitonic_sort(buf, kr_pad, lane);
        fin = buf;
    }
    for (int i = lane; i < a.k; i += 32) {
        const uint64_t key = fin[i];
        const bool ok = key != KEY_EMPTY;
        a.out_dists[(int64_t)q * a.k + i] = ok ? key_dist(key) : __int_as_float(0x7f800000);
        a.out_ids[(int64_t)q * a.k + i] = ok ? key_id(key) : -1;
    }
}

size_t refine_warp_smem(const RefineArgs& a) {
    const int nres = a.res_per_sub ? a.M * (1 << a.Br) : (1 << a.Br);
    const size_t per_warp = (size_t)(RW_CAP + a.ck_pad) * 8 + (size_t)a.d * 4 * (a.raw ? 2 : 1);
    return (((size_t)nres * 4 + 15) & ~size_t(15)) + RW_WARPS * ((per_warp + 15) & ~size_t(15));
}

__global__ void __launch_bounds__(RF_THREADS)
merge_shards_kernel(const float* __restrict__ in_d, const int32_t* __restrict__ in_i,
                    int nshards, int64_t nq, int k, int n_pad,
                    float* __restrict__ out_d, int32_t* __restrict__ out_i) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint64_t* s = reinterpret_cast<uint64_t*>(smem);
    const int64_t q = blockIdx.x;
    for (int i = threadIdx.x; i < n_pad; i += RF_THREADS) {
        uint64_t key = KEY_EMPTY;
        if (i < nshards * k) {
            const int sh = i / k, j = i % k;
            const int64_t at = ((int64_t)sh * nq + q) * k + j;
            const int32_t id = in_i[at];
            if (id >= 0) key = make_key(in_d[at], id);
        }
        s[i] = key;
    }
    __syncthreads();
    block_bitonic_sort(s, n_pad);
    for (int i = threadIdx.x; i < k; i += RF_THREADS) {
        const uint64_t key = s[i];
        const bool ok = key != KEY_EMPTY;
        out_d[q * k + i] = ok ? key_dist(key) : __int_as_float(0x7f800000);
        out_i[q * k + i] = ok ? key_id(key) : -1;
    }
}

}  // namespace

void refine_topk(const RefineArgs& a, cudaStream_t st) {
    if (a.nq <= 0) return;
    const char* e = std::getenv("JHQ_REFINE");          // tuning / test override
    const bool cta_only = e && std::strcmp(e, "cta") == 0;
    // one warp per query pays off when the batch alone fills the GPU; small
    // batches (C1: 64 queries) keep one CTA of 16 warps per query
    const bool warp_only = e && std::strcmp(e, "warp") == 0;
    if (!cta_only && (a.nq >= 1024 || warp_only) && a.ck_pad <= 128 &&
        refine_warp_smem(a) <= 200 * 1024) {
        refine_warp_kernel<<<(unsigned)ceil_div(a.nq, RW_WARPS), RW_WARPS * 32,
                             refine_warp_smem(a), st>>>(a);
        JHQ_LAUNCH_CHECK();
        count_launch();
        return;
    }
    const int nres = a.res_per_sub ? a.M * (1 << a.Br) : (1 << a.Br);
    size_t smem = (size_t)a.ck_pad * 3 * 8 + (size_t)(a.d + a.d / 32 + 1 + nres + 3) * 4 +
                  (size_t)RF_CAP * 8 + 16 + (a.raw ? (size_t)a.d * 4 + 16 : 0);
    refine_kernel<<<a.nq, RF_THREADS, smem, st>>>(a);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void refine_configure() {
    JHQ_CUDA(cudaFuncSetAttribute(refine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  227 * 1024));
    JHQ_CUDA(cudaFuncSetAttribute(refine_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  227 * 1024));
}

namespace {
__global__ void remap_ids_kernel(int32_t* __restrict__ ids, int64_t n, int mul, int add) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const int32_t v = ids[i];
        if (v >= 0) ids[i] = v * mul + add;
    }
}
}  // namespace

void remap_ids(int32_t* ids, int64_t n, int mul, int add, cudaStream_t st) {
    if (n <= 0) return;
    remap_ids_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, n, mul, add);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void merge_shard_lists(const float* in_d, const int32_t* in_i, int nshards, int64_t nq,
                       int k, float* out_d, int32_t* out_i, cudaStream_t st) {
    if (nq <= 0 || k <= 0) return;
    int n_pad = next_pow2(nshards * k);
    size_t smem = (size_t)n_pad * 8;
    if (smem > 48 * 1024) fail(JHQ_EINVAL, "merge_shards: nshards * k too large");
    merge_shards_kernel<<<(unsigned)nq, RF_THREADS, smem, st>>>(in_d, in_i, nshards, nq, k, n_pad,
                                                               out_d, out_i);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq
