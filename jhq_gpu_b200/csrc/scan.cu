// scan.cu — ADC scan over page-tiled primary codes with exact top-ck
// selection, list-major and amortised over query groups. Replaces
// build_byte_lut_kernel + scan_ivf_coalesced_kernel of the reference
// (jhq_v14_streaming_add/search.cu:65-195) and the full-N thrust::sort of its
// flat path (jhq_v1_plain/search.cu:193-194).
//
// Layout. Primary codes live in pages of 32 vectors. A page holds the codes of
// its 32 slots as [Mp/16][32 lanes][16 bytes]: lane l of a warp loads its
// vector's 16 codes of subspace group g with one 16-byte load, and the warp's
// 32 loads cover 512 contiguous bytes (fully coalesced). Mp = M rounded up to
// 16; pad subspaces have code 0 and zero tables, so they add exactly 0.
//
// Work units (built on the device by plan_build in ivf.cu). The queries that
// probe list l are grouped QG at a time; a unit is (list l, one query group,
// one chunk of at most chunk_pages pages of l). Units are numbered list-major,
// group-major, so a CTA's contiguous range of units mostly keeps one query
// group and rebuilds its tables only when the group changes. For each unit the
// CTA
//   1. (re)builds the QG queries' lookup tables in shared memory. When the bits
//      of a dimension never straddle a nibble (bits_per_dim in {1, 2, 4}: every
//      BASELINE config) the byte-LUT entry LUT[m][b] is lo[m][b & 15] +
//      hi[m][b >> 4], lo/hi being in-order fma chains of (q - c1d)^2 over the
//      dims of each nibble (the order fixed in oracle/jhq_oracle.c), and only
//      these 16-entry tables are stored, for two queries side by side
//      (float2). A 16-entry table of float2 fills one 128-byte bank row, so a
//      warp's 64-bit lookups are conflict-free whatever the codes (a random
//      256-entry gather costs ~3.5 bank-conflict wavefronts per warp load).
//      The entry is formed as lo + hi before it is added, so every distance is
//      bit-identical to the byte-LUT sum. Other bit widths keep the byte LUT
//      (one query per unit);
//   2. lets each warp score PPW pages at a time: lane = slot, one distance per
//      query of the group, each the in-order sum over m (search.cu:146-151).
//      The nibble offsets of four codes come from two shift+mask ops and one
//      byte-permute per code, shared by all queries of the group;
//   3. keeps per warp and query an exact top-ck of packed (distance, id) keys
//      (ballot + popc append into a shared buffer, merged by a warp bitonic
//      sort when full) — the replacement of the reference's per-thread top-4
//      + ck serial block-argmin rounds (search.cu:153-194), which can drop
//      true top-ck. Candidates are pruned against min(warp ck-th, CTA ck-th,
//      the query's global ck-th): a key above any of them has ck better keys
//      already kept somewhere, so it cannot reach the query's top-ck. Every
//      warp flush publishes its ck-th key to both bounds (a CTA's merged list
//      keeps ck keys at or below any of its warps' ck-th keys), so CTAs that
//      scan the same query tighten each other's bounds while they run;
//   4. at the end of a run (consecutive units of one list and query group on
//      this CTA) merges its warps' lists per query, writes the top-ck to the
//      run's first slot (the run's other slots hold empty lists) and lowers
//      the query's global bound (64-bit atomicMin). refine.cu merges the slots.
#include "device_utils.cuh"
#include "jhq_common.h"
#include "kernels.cuh"

#include <type_traits>

namespace jhq {
namespace {

#ifndef JHQ_SCAN_MIN_BLOCKS
#define JHQ_SCAN_MIN_BLOCKS 3
#endif
#ifndef JHQ_SCAN_PPW
#define JHQ_SCAN_PPW 1
#endif
constexpr int SCAN_THREADS = 256;
constexpr int PPW = JHQ_SCAN_PPW;                      // pages per warp step
constexpr int SCAN_WARPS = SCAN_THREADS / 32;
constexpr size_t SCAN_SMEM_LIMIT = 227 * 1024 - 1024;   // dynamic bytes left after statics

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

// keys of one warp top-ck region: two list halves and the append buffer (WarpTop)
__host__ __device__ inline int merge_n_of(int ck_pad) { return 2 * ck_pad + 64; }

// MODE: 0 = byte LUT (one query), 1/2/4 = nibble tables for 1/2/4 queries.
__host__ __device__ constexpr int qg_of(int mode) { return mode == 0 ? 1 : mode; }
__host__ __device__ inline size_t table_floats(int Mp, int mode) {
    return (size_t)Mp * (mode == 0 ? 256 : 32 * qg_of(mode));
}

struct ScanSmem {
    size_t tab, qs, c1d, wl, mrg, tau, total;
};

// The table sits at offset 0 of dynamic shared memory, so its address is a
// link-time constant and the lookups need no base register.
__host__ __device__ inline ScanSmem scan_smem_layout(int Mp, int d, int ck_pad, int mode) {
    ScanSmem s;
    size_t off = 0;
    const int qg = qg_of(mode);
    s.tab = off; off = align16(off + table_floats(Mp, mode) * 4);
    s.qs = off;  off = align16(off + (size_t)d * 4);
    s.c1d = off; off = align16(off + 256 * 4);
    s.wl = off;  off = align16(off + (size_t)SCAN_WARPS * qg * merge_n_of(ck_pad) * 8);
    s.mrg = off; off = align16(off + (size_t)SCAN_WARPS * ck_pad * 8);
    s.tau = off; off = align16(off + (size_t)qg * 8);
    s.total = off;
    return s;
}

__host__ __device__ inline bool nibble_split(int d, int M, int B) {
    const int bpd = B / (d / M);
    return bpd <= 4 && (4 % bpd) == 0;
}

// Tables of query slot j (q_rot already in shared qs).
//  mode 0: tab[m][256] byte LUT;  mode 1: tab[m][32] (lo 0..15, hi 16..31);
//  mode 2/4: tab[m][pair][32][2] — queries 2*pair and 2*pair+1 side by side.
template <int MODE>
__device__ void build_tables(float* tab, int j, const float* qs, const float* c1d, int d, int M,
                             int Mp, int B, bool valid) {
    const int Ds = d / M, bpd = B / Ds, kmask = (1 << bpd) - 1;
    if (MODE == 0) {
        for (int i = threadIdx.x; i < Mp * 256; i += blockDim.x) {
            const int m = i >> 8, b = i & 255;
            float acc = 0.0f;
            if (valid && m < M)
                for (int k = 0; k < Ds; ++k) {
                    const float diff = qs[m * Ds + k] - c1d[(b >> (k * bpd)) & kmask];
                    acc = __fmaf_rn(diff, diff, acc);
                }
            tab[i] = acc;
        }
        return;
    }
    constexpr int QG = qg_of(MODE);
    const int kpn = 4 / bpd;                          // dims per nibble
    for (int i = threadIdx.x; i < Mp * 32; i += blockDim.x) {
        const int m = i >> 5, t = i & 31, half = t >> 4, n = t & 15;
        float acc = 0.0f;
        if (valid && m < M) {
            const int k0 = half ? kpn : 0;
            const int k1 = half ? Ds : min(kpn, Ds);
            for (int k = k0; k < k1; ++k) {
                const float diff = qs[m * Ds + k] - c1d[(n >> ((k - k0) * bpd)) & kmask];
                acc = __fmaf_rn(diff, diff, acc);
            }
        }
        if (QG == 1) tab[i] = acc;
        else tab[((m * (QG / 2) + (j >> 1)) * 32 + t) * 2 + (j & 1)] = acc;
    }
}

// Adds the 16 subspaces of one code group (16 bytes of one vector) to the
// group's QG distances, in m order. tg points at subspace g*16 of the table.
template <int MODE>
__device__ __forceinline__ void add_group(float* dist, const unsigned char* tg, const uint4& v) {
    constexpr int QG = qg_of(MODE);
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const uint32_t w = wi == 0 ? v.x : wi == 1 ? v.y : wi == 2 ? v.z : v.w;
        if (MODE == 0) {
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                const int b = wi * 4 + bb;
                const float* row = reinterpret_cast<const float*>(tg) + b * 256;
                dist[0] = __fadd_rn(dist[0], row[(w >> (bb * 8)) & 255u]);
            }
        } else {
            // byte offsets of the lo / hi nibble entries of the 4 codes of w
            constexpr int SH = QG == 1 ? 2 : 3;           // entry size 4 or 8 bytes
            constexpr uint32_t MASK = QG == 1 ? 0x3C3C3C3Cu : 0x78787878u;
            const uint32_t Lo = (w << SH) & MASK;
            const uint32_t Hi = (w >> (4 - SH)) & MASK;
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                const int b = wi * 4 + bb;
                const uint32_t olo = __byte_perm(Lo, 0u, 0x4440u | bb);
                const uint32_t ohi = __byte_perm(Hi, 0u, 0x4440u | bb);
                if (QG == 1) {
                    const unsigned char* row = tg + b * 128;
                    const float lo = *reinterpret_cast<const float*>(row + olo);
                    const float hi = *reinterpret_cast<const float*>(row + 64 + ohi);
                    dist[0] = __fadd_rn(dist[0], __fadd_rn(lo, hi));
                } else {
#pragma unroll
                    for (int pr = 0; pr < QG / 2; ++pr) {
                        const unsigned char* row = tg + (b * (QG / 2) + pr) * 256;
                        const float2 lo = *reinterpret_cast<const float2*>(row + olo);
                        const float2 hi = *reinterpret_cast<const float2*>(row + 128 + ohi);
                        dist[2 * pr] = __fadd_rn(dist[2 * pr], __fadd_rn(lo.x, hi.x));
                        dist[2 * pr + 1] = __fadd_rn(dist[2 * pr + 1], __fadd_rn(lo.y, hi.y));
                    }
                }
            }
        }
    }
}

#ifdef JHQ_SCAN_STATS
}  // namespace
__device__ unsigned long long g_scan_stats[8];
namespace {   // pushes, inserts, flushes, runs, units
#define SCAN_STAT(i, v) atomicAdd(&g_scan_stats[i], (unsigned long long)(v))
#else
#define SCAN_STAT(i, v) ((void)0)
#endif

// Per-warp exact top-ck of one query. Region (merge_n_of(ck_pad) keys):
// two list halves of ck_pad keys (the current sorted list and the target of
// the next merge) and a 64-key append buffer. thr = pruning bound (uniform in
// the warp). A flush sorts the buffer in registers (two keys per lane, bitonic
// network over shuffles), then merges it into the list by rank: list key i
// goes to i + #(buffer keys below it), buffer key e to e + #(list keys below
// it) — keys are unique (distance, id) pairs, so the ranks are a permutation;
// positions >= ck_pad drop out. Cost ~ (log 64 + log ck_pad) shared loads per
// key instead of a bitonic sort of list + buffer.
constexpr int TOP_BUF = 64;

__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int m) {
    const unsigned hi = __shfl_xor_sync(0xffffffffu, (unsigned)(v >> 32), m);
    const unsigned lo = __shfl_xor_sync(0xffffffffu, (unsigned)v, m);
    return ((uint64_t)hi << 32) | lo;
}

// Ascending sort of 64 keys held two per lane (element 2*lane + r in x_r).
__device__ __forceinline__ void warp_sort64(uint64_t& x0, uint64_t& x1, int lane) {
#pragma unroll
    for (int k = 2; k <= 64; k <<= 1) {
        const bool up = ((2 * lane) & k) == 0;
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j == 1) {
                const uint64_t lo = x0 < x1 ? x0 : x1, hi = x0 < x1 ? x1 : x0;
                x0 = up ? lo : hi;
                x1 = up ? hi : lo;
            } else {
                const int m = j >> 1;
                const uint64_t p0 = shfl_xor64(x0, m), p1 = shfl_xor64(x1, m);
                const bool keep_min = ((lane & m) == 0) == up;
                x0 = keep_min ? (p0 < x0 ? p0 : x0) : (p0 > x0 ? p0 : x0);
                x1 = keep_min ? (p1 < x1 ? p1 : x1) : (p1 > x1 ? p1 : x1);
            }
        }
    }
}

// number of keys in sorted a[0..n) strictly below v (n a power of two)
__device__ __forceinline__ int rank_below(const uint64_t* a, int n, uint64_t v) {
    int lo = 0;
    for (int step = n >> 1; step > 0; step >>= 1)
        if (a[lo + step - 1] < v) lo += step;
    return lo + (a[lo] < v ? 1 : 0);
}

struct WarpTop {
    uint64_t* base;    // region start
    uint64_t* s;       // current sorted list [ck_pad]
    uint64_t* alt;     // merge target [ck_pad]
    uint64_t* buf;     // append buffer [TOP_BUF]
    uint64_t thr;
    int count;

    __device__ __forceinline__ void init(uint64_t* region, int ck_pad) {
        base = region;
        s = region;
        alt = region + ck_pad;
        buf = region + 2 * ck_pad;
    }
    __device__ __forceinline__ void reset(int lane, int merge_n, uint64_t bound) {
        for (int i = lane; i < merge_n; i += 32) base[i] = KEY_EMPTY;
        thr = bound;
        count = 0;
        __syncwarp();
    }
    // Merge the buffer into the list; publish the warp's ck-th key to the CTA
    // bound and pick up the tightest bound.
    __device__ __forceinline__ void flush(int lane, int ck, int ck_pad, int merge_n, uint64_t* tau,
                                          uint64_t* gbound = nullptr) {
        (void)merge_n;
        if (lane == 0) SCAN_STAT(2, 1);
        uint64_t b0 = lane < count ? buf[lane] : KEY_EMPTY;
        uint64_t b1 = lane + 32 < count ? buf[lane + 32] : KEY_EMPTY;
        warp_sort64(b0, b1, lane);
        __syncwarp();
        buf[2 * lane] = b0;
        buf[2 * lane + 1] = b1;
        __syncwarp();
        for (int i = lane; i < ck_pad; i += 32) {
            const uint64_t v = s[i];
            const int pos = i + rank_below(buf, TOP_BUF, v);
            if (pos < ck_pad) alt[pos] = v;
        }
        const int p0 = 2 * lane + rank_below(s, ck_pad, b0);
        const int p1 = 2 * lane + 1 + rank_below(s, ck_pad, b1);
        if (p0 < ck_pad) alt[p0] = b0;
        if (p1 < ck_pad) alt[p1] = b1;
        __syncwarp();
        uint64_t* t = s; s = alt; alt = t;
        const uint64_t kth = s[ck - 1];
        if (lane == 0 && kth != KEY_EMPTY) {
            atomicMin(reinterpret_cast<unsigned long long*>(tau), (unsigned long long)kth);
            if (gbound) atomicMin(reinterpret_cast<unsigned long long*>(gbound), (unsigned long long)kth);
        }
        __syncwarp();
        uint64_t tb = *reinterpret_cast<volatile uint64_t*>(tau);
        if (gbound) {
            const uint64_t g = *reinterpret_cast<volatile uint64_t*>(gbound);
            tb = g < tb ? g : tb;
        }
        thr = kth < tb ? kth : tb;
        count = 0;
    }
    __device__ __forceinline__ void push(uint64_t key, int lane, int ck, int ck_pad, int merge_n,
                                         uint64_t* tau, uint64_t* gbound = nullptr) {
        bool take = key < thr;
        unsigned mask = __ballot_sync(0xffffffffu, take);
        if (lane == 0) { SCAN_STAT(0, 32); SCAN_STAT(1, __popc(mask)); }
        if (mask == 0) return;
        if (count + __popc(mask) > TOP_BUF) {
            flush(lane, ck, ck_pad, merge_n, tau, gbound);
            take = key < thr;
            mask = __ballot_sync(0xffffffffu, take);
            if (mask == 0) return;
        }
        if (take) buf[count + __popc(mask & ((1u << lane) - 1u))] = key;
        count += __popc(mask);
        __syncwarp();
    }
};

struct UnitInfo {
    int64_t pb, pe;          // physical page range
    int list;
    int q[4];                // member queries (-1 = none)
    int64_t slot[4];         // candidate slot of each member
};

// Three CTAs per SM (registers capped at 85): the lookups are latency-bound;
// measured on C1, 2 / 3 / 4 CTAs per SM give 6.36 / 5.78 / 6.53 ms per step.
template <int G_T, int MODE>
__global__ void __launch_bounds__(SCAN_THREADS, JHQ_SCAN_MIN_BLOCKS)
scan_kernel(ScanArgs a) {
    constexpr int QG = qg_of(MODE);
    constexpr int TROW = MODE == 0 ? 1024 : (QG == 1 ? 128 : 256 * (QG / 2));  // bytes per m
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ UnitInfo unit;
    __shared__ int cur_q[4];
    const ScanSmem L = scan_smem_layout(a.Mp, a.d, a.ck_pad, MODE);
    float* tab = reinterpret_cast<float*>(smem);                 // offset 0
    float* qs = reinterpret_cast<float*>(smem + L.qs);
    float* c1d = reinterpret_cast<float*>(smem + L.c1d);
    uint64_t* wl = reinterpret_cast<uint64_t*>(smem + L.wl);
    uint64_t* mrg = reinterpret_cast<uint64_t*>(smem + L.mrg);
    uint64_t* tau = reinterpret_cast<uint64_t*>(smem + L.tau);

    const int G = G_T > 0 ? G_T : a.Mp / 16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int merge_n = merge_n_of(a.ck_pad);
    const int nunits = a.unit_off[a.nlist];
    const int u0 = (int)((int64_t)blockIdx.x * nunits / a.grid);
    const int u1 = (int)((int64_t)(blockIdx.x + 1) * nunits / a.grid);
    if (u0 >= u1) return;

    const int K1D = 1 << (a.B / (a.d / a.M));
    for (int i = tid; i < K1D; i += SCAN_THREADS) c1d[i] = a.c1d[i];
    if (tid < 4) cur_q[tid] = -2;

    // list of unit u0: last l with unit_off[l] <= u0
    int lst = 0;
    {
        int lo = 0, hi = a.nlist;
        while (hi - lo > 1) {
            int mid = (lo + hi) >> 1;
            if (a.unit_off[mid] <= u0) lo = mid; else hi = mid;
        }
        lst = lo;
    }
    WarpTop top[QG];
#pragma unroll
    for (int j = 0; j < QG; ++j) top[j].init(wl + ((size_t)warp * QG + j) * merge_n, a.ck_pad);

    // A run = consecutive units of this CTA with the same list and query group
    // (chunks of one list). The warps' top-ck lists live across the whole run;
    // the merged result goes to the run's first slot, the other slots of the
    // run get empty lists.
    __shared__ int64_t run_slot[4];
    __shared__ int run_list;
    bool run_open = false;
    auto close_run = [&]() {
#pragma unroll
        for (int j = 0; j < QG; ++j)
            top[j].flush(lane, a.ck, a.ck_pad, merge_n, tau + j,
                         cur_q[j] >= 0 ? a.gthr + cur_q[j] : nullptr);
        for (int j = 0; j < QG; ++j) {
            if (cur_q[j] < 0) continue;        // uniform across the block
            __syncthreads();
            for (int i = lane; i < a.ck_pad; i += 32) mrg[warp * a.ck_pad + i] = top[j].s[i];
            __syncthreads();
            block_bitonic_sort(mrg, SCAN_WARPS * a.ck_pad);
            uint64_t* out = a.cand + run_slot[j] * a.ck;
            for (int i = tid; i < a.ck; i += SCAN_THREADS) out[i] = mrg[i];
            if (tid == 0 && mrg[a.ck - 1] != KEY_EMPTY)
                atomicMin(reinterpret_cast<unsigned long long*>(a.gthr + cur_q[j]),
                          (unsigned long long)mrg[a.ck - 1]);
        }
    };

    for (int u = u0; u < u1; ++u) {
        __syncthreads();                       // previous unit done with unit/tables/mrg
        if (tid == 0) {
            while (a.unit_off[lst + 1] <= u) ++lst;
            const int pages0 = a.list_page_off[lst], pages1 = a.list_page_off[lst + 1];
            const int nch = (pages1 - pages0 + a.chunk_pages - 1) / a.chunk_pages;
            const int v = u - a.unit_off[lst];
            const int grp = v / nch, ch = v % nch;
            const int b0 = a.bucket_off[lst], cnt = a.bucket_off[lst + 1] - b0;
            unit.pb = pages0 + (int64_t)ch * a.chunk_pages;
            unit.pe = min((int64_t)pages1, unit.pb + a.chunk_pages);
            unit.list = lst;
            for (int j = 0; j < 4; ++j) {
                unit.q[j] = -1;
                unit.slot[j] = -1;
                if (j < QG && grp * QG + j < cnt) {
                    const int2 qp = a.bucket[b0 + grp * QG + j];
                    unit.q[j] = qp.x;
                    unit.slot[j] = a.qslot_off[qp.x] + a.cpo[(int64_t)qp.x * (a.nprobe + 1) + qp.y] + ch;
                }
            }
        }
        __syncthreads();
        bool same = true;
#pragma unroll
        for (int j = 0; j < QG; ++j) same = same && (unit.q[j] == cur_q[j]);
        const bool cont = run_open && same && unit.list == run_list;
        if (!cont) {
            if (run_open) close_run();
            __syncthreads();
            if (!same) {                       // tables of the new query group
                for (int j = 0; j < QG; ++j) {
                    const int q = unit.q[j];
                    if (q >= 0)
                        for (int i = tid; i < a.d; i += SCAN_THREADS) qs[i] = a.q_rot[(int64_t)q * a.d + i];
                    __syncthreads();
                    build_tables<MODE>(tab, j, qs, c1d, a.d, a.M, a.Mp, a.B, q >= 0);
                    __syncthreads();
                }
            }
            if (tid < QG) {
                cur_q[tid] = unit.q[tid];
                run_slot[tid] = unit.slot[tid];
                tau[tid] = unit.q[tid] >= 0 ? a.gthr[unit.q[tid]] : KEY_EMPTY;
            }
            if (tid == 0) run_list = unit.list;
            __syncthreads();
#pragma unroll
            for (int j = 0; j < QG; ++j) top[j].reset(lane, merge_n, tau[j]);
            run_open = true;
            if (tid == 0) SCAN_STAT(3, 1);
        } else {                               // continuation: this unit's slots stay empty
            for (int j = 0; j < QG; ++j) {
                if (unit.q[j] < 0) continue;
                uint64_t* out = a.cand + unit.slot[j] * a.ck;
                for (int i = tid; i < a.ck; i += SCAN_THREADS) out[i] = KEY_EMPTY;
            }
        }

        // ---- score PPW pages at a time: warp w takes pb + PPW*(w + W*i)
        const int64_t pb = unit.pb, pe = unit.pe;
        // the first group and slot ids of the warp's next pages are in flight
        // while the current pages are looked up
        int32_t id[PPW];
        uint4 cur[PPW];
        auto fetch_page = [&](int64_t p0, int32_t (&ids)[PPW], uint4 (&c0)[PPW]) {
#pragma unroll
            for (int u = 0; u < PPW; ++u) {
                const bool ok = p0 + u < pe;
                ids[u] = ok ? __ldg(a.slot_ids + (p0 + u) * 32 + lane) : -1;
                c0[u] = ok ? __ldg(reinterpret_cast<const uint4*>(a.pages) + (p0 + u) * G * 32 + lane)
                           : make_uint4(0, 0, 0, 0);
            }
        };
        fetch_page(pb + PPW * warp, id, cur);
        for (int64_t pg = pb + PPW * warp; pg < pe; pg += PPW * SCAN_WARPS) {
            int32_t idn[PPW];
            uint4 curn[PPW];
            fetch_page(pg + PPW * SCAN_WARPS, idn, curn);
            float dd[PPW][QG];
            const uint4* pp[PPW];
#pragma unroll
            for (int u = 0; u < PPW; ++u) {
                pp[u] = reinterpret_cast<const uint4*>(a.pages) + (pg + u) * G * 32 + lane;
#pragma unroll
                for (int j = 0; j < QG; ++j) dd[u][j] = 0.0f;
            }
            bool pruned = false;
            // group g+1 of every page is in flight while group g is looked up
#pragma unroll (G_T > 0 ? G_T : 1)
            for (int g = 0; g < G; ++g) {
                uint4 nxt[PPW];
#pragma unroll
                for (int u = 0; u < PPW; ++u) {
                    nxt[u] = cur[u];
                    if (g + 1 < G && pg + u < pe) nxt[u] = __ldg(pp[u] + (g + 1) * 32);
                }
                const unsigned char* tg = smem + (size_t)g * 16 * TROW;
#pragma unroll
                for (int u = 0; u < PPW; ++u) add_group<MODE>(dd[u], tg, cur[u]);
#pragma unroll
                for (int u = 0; u < PPW; ++u) cur[u] = nxt[u];
                // Early exit (bounds seeded by pilot.cu): table entries are sums of
                // squares (>= 0), so a partial distance never exceeds the final one;
                // once every slot's partial is above its query's bound, none can enter.
                if (a.prune && g + 1 < G) {
                    bool dead = true;
#pragma unroll
                    for (int u = 0; u < PPW; ++u)
#pragma unroll
                        for (int j = 0; j < QG; ++j)
                            dead = dead && (id[u] < 0 || unit.q[j] < 0 ||
                                            float_order(dd[u][j]) > (uint32_t)(top[j].thr >> 32));
                    if (__all_sync(0xffffffffu, dead)) { pruned = true; break; }
                }
            }
            if (!pruned) {
#pragma unroll
                for (int j = 0; j < QG; ++j) {
                    if (unit.q[j] < 0) continue;
#pragma unroll
                    for (int u = 0; u < PPW; ++u)
                        top[j].push(id[u] >= 0 ? make_key(dd[u][j], id[u]) : KEY_EMPTY, lane, a.ck,
                                    a.ck_pad, merge_n, tau + j, a.gthr + unit.q[j]);
                }
            }
#pragma unroll
            for (int u = 0; u < PPW; ++u) { id[u] = idn[u]; cur[u] = curn[u]; }
        }
    }
    if (run_open) close_run();
}

// ---------------------------------------------------------------------------
// Query-major warp items, for IVF with small lists (a few pages per list),
// where list-major units would be dominated by their per-unit block-wide work.
// A warp owns one item = (query, up to item_pages consecutive pages of the
// query's probe sequence): it builds the query's nibble tables in its own
// shared region (kept while consecutive items share the query), scans the
// pages, keeps an exact top-ck (pruned by the query's global bound) and
// writes it to the item's slot — no block-wide synchronisation. The per-warp
// table base is folded into the byte-permute that extracts each nibble offset
// (the bases are multiples of 256 bytes), so a lookup needs no extra add.
constexpr int QM_WARPS = 8;
constexpr int QM_GMAX = 8;                  // code groups per page (Mp <= 128)
#ifndef JHQ_QM_PPS
#define JHQ_QM_PPS 1
#endif
#ifndef JHQ_QM_MINB
#define JHQ_QM_MINB 2
#endif
constexpr int QM_PPS = JHQ_QM_PPS;          // pages scored per warp step
constexpr int QM_THREADS = QM_WARPS * 32;

__host__ __device__ inline size_t qm_table_bytes(int Mp) { return ((size_t)Mp * 128 + 255) & ~size_t(255); }
__host__ __device__ inline size_t qm_smem_bytes(int Mp, int ck_pad) {
    return QM_WARPS * qm_table_bytes(Mp) + (size_t)QM_WARPS * merge_n_of(ck_pad) * 8 + 256 * 4;
}

template <int G_T>
__global__ void __launch_bounds__(QM_THREADS, JHQ_QM_MINB)
scan_qmajor_kernel(ScanArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int G = G_T > 0 ? G_T : a.Mp / 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t tb = qm_table_bytes(a.Mp);
    const int merge_n = merge_n_of(a.ck_pad);
    float* tab = reinterpret_cast<float*>(smem + warp * tb);
    uint64_t* wl = reinterpret_cast<uint64_t*>(smem + QM_WARPS * tb) + (size_t)warp * merge_n;
    float* c1d = reinterpret_cast<float*>(smem + QM_WARPS * tb + (size_t)QM_WARPS * merge_n * 8);
    const uint32_t base = (uint32_t)(warp * tb);            // byte offset of this warp's table

    const int K1D = 1 << (a.B / (a.d / a.M));
    for (int i = threadIdx.x; i < K1D; i += QM_THREADS) c1d[i] = a.c1d[i];
    __syncthreads();

    const int Ds = a.d / a.M, bpd = a.B / Ds, kmask = (1 << bpd) - 1, kpn = 4 / bpd;
    const int64_t total = a.qslot_off[a.nq];
    const int64_t nw = (int64_t)gridDim.x * QM_WARPS;
    const int64_t wid = (int64_t)blockIdx.x * QM_WARPS + warp;
    // A contiguous range of items per warp: consecutive items of one query form
    // a run that shares the tables and one top-ck list (written to the run's
    // first slot; the run's other slots get empty lists, merged away by refine).
    const int64_t it0 = total * wid / nw, it1 = total * (wid + 1) / nw;
    int cur_q = -1;
    int64_t run_slot = -1;
    WarpTop top;
    top.init(wl, a.ck_pad);
    auto close_run = [&]() {
        top.flush(lane, a.ck, a.ck_pad, merge_n, reinterpret_cast<uint64_t*>(&a.gthr[cur_q]));
        uint64_t* out = a.cand + run_slot * a.ck;
        for (int i = lane; i < a.ck; i += 32) out[i] = top.s[i];
        __syncwarp();
    };
    for (int64_t it = it0; it < it1; ++it) {
        int lo = 0, hi = a.nq;                                // last q with qslot_off[q] <= it
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (a.qslot_off[mid] <= it) lo = mid; else hi = mid;
        }
        const int q = lo;
        const int32_t* po = a.cpo + (int64_t)q * (a.nprobe + 1);
        const int32_t* pr = a.probes + (int64_t)q * a.nprobe;
        const int first = (int)(it - a.qslot_off[q]) * a.chunk_pages;
        const int last = min(first + a.chunk_pages, po[a.nprobe]);
        if (q != cur_q) {                                     // a new run: this query's tables
            if (cur_q >= 0) close_run();
            if (lane == 0) SCAN_STAT(4, 1);
            __syncwarp();
            const float* qv = a.q_rot + (int64_t)q * a.d;
            for (int i = lane; i < a.Mp * 32; i += 32) {
                const int m = i >> 5, t = i & 31, half = t >> 4, n = t & 15;
                float acc = 0.0f;
                if (m < a.M) {
                    const int k0 = half ? kpn : 0;
                    const int k1 = half ? Ds : min(kpn, Ds);
                    for (int k = k0; k < k1; ++k) {
                        const float diff = __ldg(qv + m * Ds + k) - c1d[(n >> ((k - k0) * bpd)) & kmask];
                        acc = __fmaf_rn(diff, diff, acc);
                    }
                }
                tab[i] = acc;
            }
            __syncwarp();
            cur_q = q;
            run_slot = it;
            top.reset(lane, merge_n, a.gthr[q]);
        } else {                                              // continuation: empty slot
            uint64_t* out = a.cand + it * a.ck;
            for (int i = lane; i < a.ck; i += 32) out[i] = KEY_EMPTY;
            const uint64_t g = *reinterpret_cast<volatile uint64_t*>(&a.gthr[q]);
            top.thr = g < top.thr ? g : top.thr;
        }
        // The item's page addresses, 32 at a time, one per lane (a binary search
        // over the query's page prefix, then the list's first page): the
        // dependent index loads are paid once per 32 pages, in parallel. Pages
        // are scored QM_PPS at a time with independent accumulators (the chains
        // of the in-order sums interleave), and the next QM_PPS pages' codes and
        // slot ids are in flight while the current ones are looked up.
        constexpr int GM = G_T > 0 ? G_T : QM_GMAX;
        for (int b0 = first; b0 < last; b0 += 32) {
            const int npg = min(32, last - b0);
            int64_t mypg = 0;
            if (lane < npg) {
                const int lp = b0 + lane;
                int plo = 0, phi = a.nprobe;                  // last p with po[p] <= lp
                while (phi - plo > 1) {
                    const int mid = (plo + phi) >> 1;
                    if (po[mid] <= lp) plo = mid; else phi = mid;
                }
                mypg = a.list_page_off[pr[plo]] + (lp - po[plo]);
            }
            auto fetch = [&](int j, int32_t (&id)[QM_PPS], uint4 (&code)[QM_PPS][GM]) {
#pragma unroll
                for (int u = 0; u < QM_PPS; ++u) {
                    const int64_t pg = __shfl_sync(0xffffffffu, mypg, (j + u) & 31);
                    const bool ok = j + u < npg;
                    id[u] = ok ? __ldg(a.slot_ids + pg * 32 + lane) : -1;
                    const uint4* pp = reinterpret_cast<const uint4*>(a.pages) + pg * G * 32 + lane;
#pragma unroll
                    for (int g = 0; g < GM; ++g)
                        code[u][g] = (ok && g < G) ? __ldg(pp + g * 32) : make_uint4(0, 0, 0, 0);
                }
            };
            int32_t id_c[QM_PPS];
            uint4 code_c[QM_PPS][GM];
            fetch(0, id_c, code_c);
            for (int j = 0; j < npg; j += QM_PPS) {
                int32_t id_n[QM_PPS];
                uint4 code_n[QM_PPS][GM];
                fetch(j + QM_PPS, id_n, code_n);
                float dist[QM_PPS];
#pragma unroll
                for (int u = 0; u < QM_PPS; ++u) dist[u] = 0.0f;
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g >= G) break;
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi) {
                        uint32_t Lo[QM_PPS], Hi[QM_PPS];
#pragma unroll
                        for (int u = 0; u < QM_PPS; ++u) {
                            const uint4 cur = code_c[u][g];
                            const uint32_t w = wi == 0 ? cur.x : wi == 1 ? cur.y : wi == 2 ? cur.z : cur.w;
                            Lo[u] = (w << 2) & 0x3C3C3C3Cu;
                            Hi[u] = (w >> 2) & 0x3C3C3C3Cu;
                        }
#pragma unroll
                        for (int bb = 0; bb < 4; ++bb) {
                            const int b = g * 16 + wi * 4 + bb;           // subspace
#pragma unroll
                            for (int u = 0; u < QM_PPS; ++u) {
                                // low byte from the nibble offset, upper bytes from the warp base
                                const uint32_t olo = __byte_perm(Lo[u], base, 0x7650u | bb);
                                const uint32_t ohi = __byte_perm(Hi[u], base, 0x7650u | bb);
                                const float lo_v = *reinterpret_cast<const float*>(smem + olo + b * 128);
                                const float hi_v = *reinterpret_cast<const float*>(smem + ohi + b * 128 + 64);
                                dist[u] = __fadd_rn(dist[u], __fadd_rn(lo_v, hi_v));
                            }
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < QM_PPS; ++u)
                    if (j + u < npg)                                  // uniform in the warp
                        top.push(id_c[u] >= 0 ? make_key(dist[u], id_c[u]) : KEY_EMPTY, lane, a.ck,
                                 a.ck_pad, merge_n, reinterpret_cast<uint64_t*>(&a.gthr[q]));
#pragma unroll
                for (int u = 0; u < QM_PPS; ++u) {
                    id_c[u] = id_n[u];
#pragma unroll
                    for (int g = 0; g < GM; ++g) code_c[u][g] = code_n[u][g];
                }
            }
        }
    }
    if (cur_q >= 0) close_run();
}

template <int G_T, int MODE>
void launch_scan(const ScanArgs& a, size_t smem, cudaStream_t st) {
    scan_kernel<G_T, MODE><<<a.grid, SCAN_THREADS, smem, st>>>(a);
}

// Opt-in dynamic shared memory: the per-block limit (227 KB) minus the
// kernel's static shared variables.
template <int G_T, int MODE>
void configure_one() {
    cudaFuncAttributes fa;
    JHQ_CUDA(cudaFuncGetAttributes(&fa, scan_kernel<G_T, MODE>));
    JHQ_CUDA(cudaFuncSetAttribute(scan_kernel<G_T, MODE>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  227 * 1024 - (int)fa.sharedSizeBytes));
}

template <int G_T, int MODE>
int blocks_per_sm(size_t smem) {
    int n = 0;
    JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_kernel<G_T, MODE>, SCAN_THREADS,
                                                           smem));
    return n;
}

template <int G, class F>
auto dispatch_mode(int mode, F&& f) {
    switch (mode) {
        case 0: return f(std::integral_constant<int, G>{}, std::integral_constant<int, 0>{});
        case 1: return f(std::integral_constant<int, G>{}, std::integral_constant<int, 1>{});
        case 2: return f(std::integral_constant<int, G>{}, std::integral_constant<int, 2>{});
        default: return f(std::integral_constant<int, G>{}, std::integral_constant<int, 4>{});
    }
}

// Dispatch on (Mp/16, mode) to the compile-time instantiations.
template <class F>
auto dispatch(int Mp, int mode, F&& f) {
    switch (Mp / 16) {
        case 1: return dispatch_mode<1>(mode, f);
        case 2: return dispatch_mode<2>(mode, f);
        case 4: return dispatch_mode<4>(mode, f);
        case 6: return dispatch_mode<6>(mode, f);
        case 8: return dispatch_mode<8>(mode, f);
        default: return dispatch_mode<0>(mode, f);
    }
}

}  // namespace

void scan_configure() {
    for (int g : {1, 2, 4, 6, 8, 0})
        for (int mode : {0, 1, 2, 4})
            dispatch(g * 16, mode, [](auto G, auto Md) { configure_one<G.value, Md.value>(); return 0; });
}

// Query groups of 2 or 4 (float2 tables) issue fewer instructions per lookup
// but measured slower on B200 than one query per lane (C1: 7.4 / 11.4 ms vs
// 6.4 ms per 1,000 queries), so one query per unit is the default; the wider
// groups stay selectable (JHQ_SCAN_MODE) for tuning.
int scan_mode_for(int d, int M, int B, double queries_per_list) {
    (void)queries_per_list;
    return nibble_split(d, M, B) ? 1 : 0;
}

size_t scan_smem_bytes(int Mp, int d, int ck_pad, int mode) {
    // reported with the static-variable reserve, so callers compare with 227 KB
    return scan_smem_layout(Mp, d, ck_pad, mode).total + 1024;
}

int scan_grid_for(int Mp, int d, int ck_pad, int mode) {
    int dev = 0, sms = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const size_t smem = scan_smem_layout(Mp, d, ck_pad, mode).total;
    const int per_sm = dispatch(Mp, mode, [&](auto G, auto Md) { return blocks_per_sm<G.value, Md.value>(smem); });
    if (per_sm < 1) fail(JHQ_EINVAL, "scan: kernel does not fit on an SM (reduce M or d)");
    return sms * per_sm;
}

template <int G_T>
void qm_configure_one() {
    JHQ_CUDA(cudaFuncSetAttribute(scan_qmajor_kernel<G_T>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
}

size_t scan_qmajor_smem_bytes(int Mp, int ck_pad) { return qm_smem_bytes(Mp, ck_pad); }

int scan_qmajor_grid_for(int Mp, int ck_pad) {
    int dev = 0, sms = 0, per_sm = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const size_t smem = qm_smem_bytes(Mp, ck_pad);
    switch (Mp / 16) {
        case 1: qm_configure_one<1>();
                JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_qmajor_kernel<1>, QM_THREADS, smem)); break;
        case 2: qm_configure_one<2>();
                JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_qmajor_kernel<2>, QM_THREADS, smem)); break;
        case 4: qm_configure_one<4>();
                JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_qmajor_kernel<4>, QM_THREADS, smem)); break;
        case 8: qm_configure_one<8>();
                JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_qmajor_kernel<8>, QM_THREADS, smem)); break;
        default: qm_configure_one<0>();
                JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_qmajor_kernel<0>, QM_THREADS, smem)); break;
    }
    if (per_sm < 1) fail(JHQ_EINVAL, "scan: query-major kernel does not fit on an SM");
    return sms * per_sm;
}

void scan_topck(const ScanArgs& a, cudaStream_t st) {
    if (a.qmajor) {
        const size_t smem = qm_smem_bytes(a.Mp, a.ck_pad);
        switch (a.Mp / 16) {
            case 1: scan_qmajor_kernel<1><<<a.grid, QM_THREADS, smem, st>>>(a); break;
            case 2: scan_qmajor_kernel<2><<<a.grid, QM_THREADS, smem, st>>>(a); break;
            case 4: scan_qmajor_kernel<4><<<a.grid, QM_THREADS, smem, st>>>(a); break;
            case 8: scan_qmajor_kernel<8><<<a.grid, QM_THREADS, smem, st>>>(a); break;
            default: scan_qmajor_kernel<0><<<a.grid, QM_THREADS, smem, st>>>(a); break;
        }
        JHQ_LAUNCH_CHECK();
        count_launch();
        return;
    }
    const size_t smem = scan_smem_layout(a.Mp, a.d, a.ck_pad, a.mode).total;
    if (smem > SCAN_SMEM_LIMIT) fail(JHQ_EINVAL, "scan: shared-memory tables too large (reduce M)");
    dispatch(a.Mp, a.mode, [&](auto G, auto Md) { launch_scan<G.value, Md.value>(a, smem, st); return 0; });
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq

#ifdef JHQ_SCAN_STATS
extern "C" int jhq_debug_scan_stats(unsigned long long* out, int reset) {
    cudaMemcpyFromSymbol(out, jhq::g_scan_stats, sizeof(unsigned long long) * 8);
    if (reset) {
        unsigned long long z[8] = {};
        cudaMemcpyToSymbol(jhq::g_scan_stats, z, sizeof z);
    }
    return 0;
}
#endif
