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
//   1. builds that query's byte LUT in shared memory (LUT[m][b] = lo[m][b&15]
//      + hi[m][b>>4], lo/hi = in-order fma chains of (q - c1d)^2 over the dims
//      of each nibble — the order fixed in oracle/jhq_oracle.c);
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

namespace jhq {
namespace {

constexpr int SCAN_THREADS = 512;
constexpr int SCAN_WARPS = SCAN_THREADS / 32;

struct ScanSmem {
    size_t lut, nib, qs, c1d, wl, mrg, total;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline int merge_n_of(int ck_pad) {
    int n = 1;
    while (n < ck_pad + 64) n <<= 1;
    return n;
}

__host__ __device__ inline ScanSmem scan_smem_layout(int Mp, int d, int ck_pad) {
    ScanSmem s;
    size_t off = 0;
    s.lut = off; off = align16(off + (size_t)Mp * 256 * 4);
    s.nib = off; off = align16(off + (size_t)Mp * 32 * 4);
    s.qs = off;  off = align16(off + (size_t)d * 4);
    s.c1d = off; off = align16(off + 256 * 4);
    s.wl = off;  off = align16(off + (size_t)SCAN_WARPS * merge_n_of(ck_pad) * 8);
    s.mrg = off; off = align16(off + (size_t)SCAN_WARPS * ck_pad * 8);
    s.total = off;
    return s;
}

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int b) {
    uint32_t w = (b < 4) ? v.x : (b < 8) ? v.y : (b < 12) ? v.z : v.w;
    return (w >> ((b & 3) * 8)) & 0xffu;
}

// Build the byte LUT of query q_rot (already in shared qs) into lut[Mp][256].
__device__ void build_lut(float* lut, float* nib, const float* qs, const float* c1d,
                          int d, int M, int Mp, int B) {
    const int Ds = d / M, bpd = B / Ds, kmask = (1 << bpd) - 1;
    const bool split = (bpd <= 4) && (4 % bpd == 0);
    if (split) {
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
            nib[i] = acc;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < Mp * 256; i += blockDim.x) {
            const int m = i >> 8, b = i & 255;
            lut[i] = (m < M) ? __fadd_rn(nib[m * 32 + (b & 15)], nib[m * 32 + 16 + (b >> 4)]) : 0.0f;
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
            lut[i] = acc;
        }
    }
    __syncthreads();
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

// Small LUTs (Mp <= 32) leave room for two CTAs per SM: cap registers at 64.
template <int G_T>
__global__ void __launch_bounds__(SCAN_THREADS, (G_T > 0 && G_T <= 2) ? 2 : 1)
scan_kernel(ScanArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const ScanSmem L = scan_smem_layout(a.Mp, a.d, a.ck_pad);
    float* lut = reinterpret_cast<float*>(smem + L.lut);
    float* nib = reinterpret_cast<float*>(smem + L.nib);
    float* qs = reinterpret_cast<float*>(smem + L.qs);
    float* c1d = reinterpret_cast<float*>(smem + L.c1d);
    uint64_t* wl = reinterpret_cast<uint64_t*>(smem + L.wl);
    uint64_t* mrg = reinterpret_cast<uint64_t*>(smem + L.mrg);

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
        // ---- LUT of query q
        __syncthreads();
        for (int i = tid; i < a.d; i += SCAN_THREADS) qs[i] = a.q_rot[(int64_t)q * a.d + i];
        __syncthreads();
        build_lut(lut, nib, qs, c1d, a.d, a.M, a.Mp, a.B);
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
            float dist[2] = {0.0f, 0.0f};
            const uint4* pg0 = reinterpret_cast<const uint4*>(a.pages) + phys[0] * G * 32 + lane;
            const uint4* pg1 = reinterpret_cast<const uint4*>(a.pages) + phys[1] * G * 32 + lane;
            if (G_T > 0) {
                // all code groups of both pages in flight before the first lookup
                constexpr int GG = G_T > 0 ? G_T : 1;
                uint4 v0[GG], v1[GG];
#pragma unroll
                for (int g = 0; g < GG; ++g) v0[g] = __ldg(pg0 + g * 32);
                if (valid[1]) {
#pragma unroll
                    for (int g = 0; g < GG; ++g) v1[g] = __ldg(pg1 + g * 32);
                } else {
#pragma unroll
                    for (int g = 0; g < GG; ++g) v1[g] = make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int g = 0; g < GG; ++g) {
                    const float* lg = lut + g * 16 * 256;
#pragma unroll
                    for (int b = 0; b < 16; ++b) {
                        dist[0] = __fadd_rn(dist[0], lg[b * 256 + byte_of(v0[g], b)]);
                        dist[1] = __fadd_rn(dist[1], lg[b * 256 + byte_of(v1[g], b)]);
                    }
                }
            } else {
                for (int g = 0; g < G; ++g) {
                    const uint4 v0 = __ldg(pg0 + g * 32);
                    const uint4 v1 = valid[1] ? __ldg(pg1 + g * 32) : make_uint4(0, 0, 0, 0);
                    const float* lg = lut + g * 16 * 256;
#pragma unroll
                    for (int b = 0; b < 16; ++b) {
                        dist[0] = __fadd_rn(dist[0], lg[b * 256 + byte_of(v0, b)]);
                        dist[1] = __fadd_rn(dist[1], lg[b * 256 + byte_of(v1, b)]);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                int32_t id = valid[u] ? __ldg(a.slot_ids + phys[u] * 32 + lane) : -1;
                top.push(id >= 0 ? make_key(dist[u], id) : KEY_EMPTY, lane);
            }
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

template <int G_T>
void launch_scan(const ScanArgs& a, size_t smem, cudaStream_t st) {
    scan_kernel<G_T><<<a.grid, SCAN_THREADS, smem, st>>>(a);
}

template <int G_T>
void configure_one() {
    JHQ_CUDA(cudaFuncSetAttribute(scan_kernel<G_T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  227 * 1024));
}

}  // namespace

void scan_configure() {
    configure_one<0>(); configure_one<1>(); configure_one<2>();
    configure_one<4>(); configure_one<6>(); configure_one<8>();
}

size_t scan_smem_bytes(int Mp, int d, int ck_pad) { return scan_smem_layout(Mp, d, ck_pad).total; }

template <int G_T>
int blocks_per_sm(size_t smem) {
    int n = 0;
    JHQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_kernel<G_T>, SCAN_THREADS, smem));
    return n;
}

int scan_grid_for(int Mp, int d, int ck_pad) {
    int dev = 0, sms = 0;
    JHQ_CUDA(cudaGetDevice(&dev));
    JHQ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const size_t smem = scan_smem_layout(Mp, d, ck_pad).total;
    int per_sm = 0;
    switch (Mp / 16) {
        case 1: per_sm = blocks_per_sm<1>(smem); break;
        case 2: per_sm = blocks_per_sm<2>(smem); break;
        case 4: per_sm = blocks_per_sm<4>(smem); break;
        case 6: per_sm = blocks_per_sm<6>(smem); break;
        case 8: per_sm = blocks_per_sm<8>(smem); break;
        default: per_sm = blocks_per_sm<0>(smem); break;
    }
    if (per_sm < 1) fail(JHQ_EINVAL, "scan: kernel does not fit on an SM (reduce M or d)");
    return sms * per_sm;
}

void scan_topck(const ScanArgs& a, cudaStream_t st) {
    const size_t smem = scan_smem_layout(a.Mp, a.d, a.ck_pad).total;
    if (smem > 227 * 1024) fail(JHQ_EINVAL, "scan: shared-memory LUT too large (reduce M)");
    switch (a.Mp / 16) {
        case 1: launch_scan<1>(a, smem, st); break;
        case 2: launch_scan<2>(a, smem, st); break;
        case 4: launch_scan<4>(a, smem, st); break;
        case 6: launch_scan<6>(a, smem, st); break;
        case 8: launch_scan<8>(a, smem, st); break;
        default: launch_scan<0>(a, smem, st); break;
    }
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq
