// scan.cu — per-query byte LUT in shared memory + ADC scan over page-tiled
// primary codes + exact top-ck selection. Replaces build_byte_lut_kernel and
// scan_ivf_coalesced_kernel of the reference (jhq_v14_streaming_add/
// search.cu:65-195) and the full-N thrust::sort of the flat path
// (jhq_v1_plain/search.cu:193-194).
//
// Layout. Primary codes live in pages of 32 vectors. A page holds the codes
// of its 32 slots as [Mp/16][32 lanes][16 bytes]: lane l of a warp loads its
// vector's 16 codes of subspace group g with one 16-byte load, and the warp's
// 32 loads cover 512 contiguous bytes (fully coalesced). Mp = M rounded up to
// 16; pad subspaces have code 0 and a zero LUT row, so they add exactly 0.
//
// Work split. The probed pages of all queries of a batch form one sequence
// (query-major, probe order inside a query, qpage_off = its offsets). A
// persistent grid of `grid` CTAs splits it evenly: CTA c owns pages
// [c*T/grid, (c+1)*T/grid). For every query segment it touches, the CTA
//   1. builds that query's lookup tables in shared memory. When the bits of a
//      dimension never straddle a nibble (bits_per_dim in {1, 2, 4}, i.e. every
//      BASELINE config), the byte LUT entry LUT[m][b] is lo[m][b&15] +
//      hi[m][b>>4], with lo/hi in-order fma chains of (q - c1d)^2 over the dims
//      of each nibble — the order fixed in oracle/jhq_oracle.c — and only the two
//      16-entry tables are stored (32 floats per subspace). A 16-entry table
//      spans 16 distinct banks, so a warp's lookups are conflict-free whatever
//      the codes: two conflict-free loads per code byte instead of a random
//      256-way gather (~3.5 bank-conflict wavefronts per warp load). The
//      entry is formed as lo + hi before it is added, so the sum is bit-identical
//      to the byte-LUT sum. Other bit widths keep the full byte LUT;
//   2. lets each warp scan pages two at a time: lane = slot, distance = sum
//      over m in order of LUT[m][code_m] (search.cu:146-151 order);
//   3. keeps a per-warp exact top-ck of packed (distance, id) keys: lanes whose
//      key beats the warp's current ck-th key append to a shared buffer (ballot
//      + popc), and a full buffer is merged into the list by a warp bitonic
//      sort — the replacement of the reference's per-thread top-4 + ck serial
//      block-argmin rounds (search.cu:153-194), which can drop true top-ck;
//   4. merges its warps' lists with a block bitonic sort and writes the
//      segment's top-ck keys to slot (c + q) of the candidate buffer. Slots are
//      unique because (c, q) pairs advance monotonically in both coordinates.
// refine.cu merges the slots of each query.
#include "device_utils.cuh"
#include "jhq_common.h"
#include "kernels.cuh"

#include <type_traits>

namespace jhq {
namespace {

constexpr int SCAN_THREADS = 512;
constexpr int SCAN_WARPS = SCAN_THREADS / 32;

struct ScanSmem {
    size_t tab, qs, c1d, wl, mrg, total;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline int merge_n_of(int ck_pad) {
    int n = 1;
    while (n < ck_pad + 64) n <<= 1;
    return n;
}

// The lookup table sits at offset 0 of dynamic shared memory, so its address
// is a link-time constant and the lookups need no base register.
__host__ __device__ inline ScanSmem scan_smem_layout(int Mp, int d, int ck_pad, bool nib) {
    ScanSmem s;
    size_t off = 0;
    s.tab = off; off = align16(off + (size_t)Mp * (nib ? 32 : 256) * 4);
    s.qs = off;  off = align16(off + (size_t)d * 4);
    s.c1d = off; off = align16(off + 256 * 4);
    s.wl = off;  off = align16(off + (size_t)SCAN_WARPS * merge_n_of(ck_pad) * 8);
    s.mrg = off; off = align16(off + (size_t)SCAN_WARPS * ck_pad * 8);
    s.total = off;
    return s;
}

__host__ __device__ inline bool nibble_split(int d, int M, int B) {
    const int bpd = B / (d / M);
    return bpd <= 4 && (4 % bpd) == 0;
}

// Tables of query q_rot (already in shared qs): nibble tables tab[Mp][32]
// (lo at 0..15, hi at 16..31) when NIB, else the byte LUT tab[Mp][256].
template <bool NIB>
__device__ void build_tables(float* tab, const float* qs, const float* c1d, int d, int M, int Mp,
                             int B) {
    const int Ds = d / M, bpd = B / Ds, kmask = (1 << bpd) - 1;
    if (NIB) {
        const int kpn = 4 / bpd;                      // dims per nibble
        for (int i = threadIdx.x; i < Mp * 32; i += blockDim.x) {
            const int m = i >> 5, t = i & 31, half = t >> 4, n = t & 15;
            float acc = 0.0f;
            if (m < M) {
                const int k0 = half ? kpn : 0;
                const int k1 = half ? Ds : min(kpn, Ds);
                for (int k = k0; k < k1; ++k) {
                    const float diff = qs[m * Ds + k] - c1d[(n >> ((k - k0) * bpd)) & kmask];
                    acc = __fmaf_rn(diff, diff, acc);
                }
            }
            tab[i] = acc;
        }
    } else {
        for (int i = threadIdx.x; i < Mp * 256; i += blockDim.x) {
            const int m = i >> 8, b = i & 255;
            float acc = 0.0f;
            if (m < M)
                for (int k = 0; k < Ds; ++k) {
                    const float diff = qs[m * Ds + k] - c1d[(b >> (k * bpd)) & kmask];
                    acc = __fmaf_rn(diff, diff, acc);
                }
            tab[i] = acc;
        }
    }
    __syncthreads();
}

// Adds the 16 subspaces of one code group (16 bytes) to dist, in m order.
template <bool NIB>
__device__ __forceinline__ float add_group(float dist, const float* tg, const uint4& v) {
#pragma unroll
    for (int b = 0; b < 16; ++b) {
        const uint32_t w = (b < 4) ? v.x : (b < 8) ? v.y : (b < 12) ? v.z : v.w;
        const int sh = (b & 3) * 8;
        float e;
        if (NIB) {
            const float* nm = tg + b * 32;
            e = __fadd_rn(nm[(w >> sh) & 15u], nm[16 + ((w >> (sh + 4)) & 15u)]);
        } else {
            e = tg[b * 256 + ((w >> sh) & 255u)];
        }
        dist = __fadd_rn(dist, e);
    }
    return dist;
}

// Per-warp exact top-ck state: s[0..ck_pad) sorted list, s[ck_pad..merge_n) buffer.
struct WarpTop {
    uint64_t* s;
    uint64_t thr;     // current ck-th key (uniform in the warp)
    int count;        // buffered entries (uniform)
    int ck, ck_pad, merge_n;

    __device__ __forceinline__ void reset(int lane) {
        for (int i = lane; i < merge_n; i += 32) s[i] = KEY_EMPTY;
        thr = KEY_EMPTY;
        count = 0;
        __syncwarp();
    }
    __device__ __forceinline__ void flush(int lane) {
        const int cap = merge_n - ck_pad;
        for (int i = count + lane; i < cap; i += 32) s[ck_pad + i] = KEY_EMPTY;
        __syncwarp();
        warp_bitonic_sort(s, merge_n, lane);
        thr = s[ck - 1];
        count = 0;
    }
    __device__ __forceinline__ void push(uint64_t key, int lane) {
        bool take = key < thr;
        unsigned mask = __ballot_sync(0xffffffffu, take);
        if (mask == 0) return;
        if (count + __popc(mask) > merge_n - ck_pad) {
            flush(lane);
            take = key < thr;
            mask = __ballot_sync(0xffffffffu, take);
            if (mask == 0) return;
        }
        if (take) s[ck_pad + count + __popc(mask & ((1u << lane) - 1u))] = key;
        count += __popc(mask);
        __syncwarp();
    }
};

template <int G_T, bool NIB>
__global__ void __launch_bounds__(SCAN_THREADS, 1)
scan_kernel(ScanArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const ScanSmem L = scan_smem_layout(a.Mp, a.d, a.ck_pad, NIB);
    float* tab = reinterpret_cast<float*>(smem);                 // offset 0
    float* qs = reinterpret_cast<float*>(smem + L.qs);
    float* c1d = reinterpret_cast<float*>(smem + L.c1d);
    uint64_t* wl = reinterpret_cast<uint64_t*>(smem + L.wl);
    uint64_t* mrg = reinterpret_cast<uint64_t*>(smem + L.mrg);
    constexpr int TSTRIDE = NIB ? 32 : 256;                       // floats per subspace

    const int G = G_T > 0 ? G_T : a.Mp / 16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int merge_n = merge_n_of(a.ck_pad);
    const int64_t T = a.qpage_off[a.nq];
    const int64_t c = blockIdx.x;
    const int64_t start = c * T / a.grid, end = (c + 1) * T / a.grid;
    if (start >= end) return;

    const int K1D = 1 << (a.B / (a.d / a.M));
    for (int i = tid; i < K1D; i += SCAN_THREADS) c1d[i] = a.c1d[i];

    // query containing page `start`: last q with qpage_off[q] <= start
    int lo = 0, hi = a.nq;                                   // qpage_off[hi] > start
    while (hi - lo > 1) {
        int mid = (lo + hi) >> 1;
        if (a.qpage_off[mid] <= start) lo = mid; else hi = mid;
    }
    int q = lo;

    WarpTop top;
    top.s = wl + (size_t)warp * merge_n;
    top.ck = a.ck; top.ck_pad = a.ck_pad; top.merge_n = merge_n;

    int64_t pos = start;
    while (pos < end) {
        const int64_t qbase = a.qpage_off[q];
        const int64_t seg_end = min(end, a.qpage_off[q + 1]);
        // ---- tables of query q
        __syncthreads();
        for (int i = tid; i < a.d; i += SCAN_THREADS) qs[i] = a.q_rot[(int64_t)q * a.d + i];
        __syncthreads();
        build_tables<NIB>(tab, qs, c1d, a.d, a.M, a.Mp, a.B);
        top.reset(lane);

        // ---- scan: warp w takes page pairs (lp, lp+1), lp = first + 2*(w + W*i)
        const int32_t* ppo = a.probe_page_off + (int64_t)q * (a.nprobe + 1);
        const int32_t* pr = a.probes + (int64_t)q * a.nprobe;
        const int first = (int)(pos - qbase), last = (int)(seg_end - qbase);
        int p = 0;                                        // probe cursor (monotone per warp)
        for (int lp = first + 2 * warp; lp < last; lp += 2 * SCAN_WARPS) {
            int64_t phys[2];
            bool valid[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                int l = lp + u;
                valid[u] = l < last;
                phys[u] = 0;
                if (valid[u]) {
                    while (l >= ppo[p + 1]) ++p;
                    phys[u] = a.list_page_off[pr[p]] + (l - ppo[p]);
                }
            }
            const int32_t id0 = __ldg(a.slot_ids + phys[0] * 32 + lane);
            const int32_t id1 = valid[1] ? __ldg(a.slot_ids + phys[1] * 32 + lane) : -1;
            float d0 = 0.0f, d1 = 0.0f;
            const uint4* pg0 = reinterpret_cast<const uint4*>(a.pages) + phys[0] * G * 32 + lane;
            const uint4* pg1 = reinterpret_cast<const uint4*>(a.pages) + phys[1] * G * 32 + lane;
            // group g+1 of both pages is in flight while group g is looked up
            uint4 c0 = __ldg(pg0), c1 = valid[1] ? __ldg(pg1) : make_uint4(0, 0, 0, 0);
#pragma unroll (G_T > 0 ? G_T : 1)
            for (int g = 0; g < G; ++g) {
                uint4 n0 = c0, n1 = c1;
                if (g + 1 < G) {
                    n0 = __ldg(pg0 + (g + 1) * 32);
                    if (valid[1]) n1 = __ldg(pg1 + (g + 1) * 32);
                }
                const float* tg = tab + g * 16 * TSTRIDE;
                d0 = add_group<NIB>(d0, tg, c0);
                d1 = add_group<NIB>(d1, tg, c1);
                c0 = n0;
                c1 = n1;
            }
            top.push(id0 >= 0 ? make_key(d0, id0) : KEY_EMPTY, lane);
            top.push(id1 >= 0 ? make_key(d1, id1) : KEY_EMPTY, lane);
        }
        top.flush(lane);
        __syncwarp();
        for (int i = lane; i < a.ck_pad; i += 32) mrg[warp * a.ck_pad + i] = top.s[i];
        __syncthreads();
        block_bitonic_sort(mrg, SCAN_WARPS * a.ck_pad);
        uint64_t* out = a.cand + (c + q) * a.ck;
        for (int i = tid; i < a.ck; i += SCAN_THREADS) out[i] = mrg[i];

        pos = seg_end;
        if (pos < end) {                                   // next query with pages
            ++q;
            while (a.qpage_off[q + 1] <= pos) ++q;
        }
    }
}

template <int G_T, bool NIB>
void launch_scan(const ScanArgs& a, size_t smem, cudaStream_t st) {
    scan_kernel<G_T, NIB><<<a.grid, SCAN_THREADS, smem, st>>>(a);
}

template <int G_T, bool NIB>
void configure_one() {
    JHQ_CUDA(cudaFuncSetAttribute(scan_kernel<G_T, NIB>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
}

template <int G_T, bool NIB>
int blocks_per_sm(size_t smem) {
    int n = 0;
    JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_kernel<G_T, NIB>, SCAN_THREADS,
                                                           smem));
    return n;
}

// Dispatch on (Mp/16, nibble) to the compile-time instantiations.
template <class F>
auto dispatch(int Mp, bool nib, F&& f) {
    switch (Mp / 16) {
        case 1: return nib ? f(std::integral_constant<int, 1>{}, std::true_type{})
                           : f(std::integral_constant<int, 1>{}, std::false_type{});
        case 2: return nib ? f(std::integral_constant<int, 2>{}, std::true_type{})
                           : f(std::integral_constant<int, 2>{}, std::false_type{});
        case 4: return nib ? f(std::integral_constant<int, 4>{}, std::true_type{})
                           : f(std::integral_constant<int, 4>{}, std::false_type{});
        case 6: return nib ? f(std::integral_constant<int, 6>{}, std::true_type{})
                           : f(std::integral_constant<int, 6>{}, std::false_type{});
        case 8: return nib ? f(std::integral_constant<int, 8>{}, std::true_type{})
                           : f(std::integral_constant<int, 8>{}, std::false_type{});
        default: return nib ? f(std::integral_constant<int, 0>{}, std::true_type{})
                            : f(std::integral_constant<int, 0>{}, std::false_type{});
    }
}

}  // namespace

void scan_configure() {
    for (int g : {1, 2, 4, 6, 8, 0})
        for (bool nib : {true, false})
            dispatch(g * 16, nib, [](auto G, auto N) { configure_one<G.value, N.value>(); return 0; });
}

size_t scan_smem_bytes(int Mp, int d, int ck_pad, bool nib) {
    return scan_smem_layout(Mp, d, ck_pad, nib).total;
}

bool scan_uses_nibbles(int d, int M, int B) { return nibble_split(d, M, B); }

int scan_grid_for(int Mp, int d, int ck_pad, bool nib) {
    int dev = 0, sms = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const size_t smem = scan_smem_layout(Mp, d, ck_pad, nib).total;
    const int per_sm = dispatch(Mp, nib, [&](auto G, auto N) { return blocks_per_sm<G.value, N.value>(smem); });
    if (per_sm < 1) fail(JHQ_EINVAL, "scan: kernel does not fit on an SM (reduce M or d)");
    return sms * per_sm;
}

void scan_topck(const ScanArgs& a, cudaStream_t st) {
    const bool nib = nibble_split(a.d, a.M, a.B);
    const size_t smem = scan_smem_layout(a.Mp, a.d, a.ck_pad, nib).total;
    if (smem > 227 * 1024) fail(JHQ_EINVAL, "scan: shared-memory LUT too large (reduce M)");
    dispatch(a.Mp, nib, [&](auto G, auto N) { launch_scan<G.value, N.value>(a, smem, st); return 0; });
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq
