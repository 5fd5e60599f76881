// ivf.cu — IVF probe selection and the page partition of the ADC scan.
//
// select_probes_kernel replaces select_probes_kernel of the reference
// (jhq_v14_streaming_add/search.cu:13-62), which runs nprobe rounds of
// block-wide argmin with the whole score row in shared memory and cannot
// launch above ~11.7k lists (48 KB default). Here one CTA per query finds the
// nprobe-th smallest score by a 4-pass 8-bit radix select over
// order-preserving keys read from global memory (no size limit), gathers the
// winners — ties at the threshold resolved by ascending list id — and sorts
// them by (score, list id), the exact order of jhq_v3_ivf/search.cu:46-85.
//
// scan_prepare_kernel turns the chosen lists into page counts: per query the
// prefix sums of pages over its probes, and over queries the exclusive scan
// qpage_off that the persistent scan kernel partitions evenly across CTAs.
#include "device_utils.cuh"
#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {
namespace {

constexpr int SP_THREADS = 256;

__global__ void __launch_bounds__(SP_THREADS)
select_probes_kernel(const float* __restrict__ s, int nlist, int nprobe, int np_pad,
                     int32_t* __restrict__ probes) {
    extern __shared__ uint64_t sp_buf[];           // np_pad entries
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sh_prefix, sh_rank, sh_nbuf, sh_eq_taken;
    const int q = blockIdx.x, tid = threadIdx.x;
    const float* row = s + (int64_t)q * nlist;

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
    __shared__ uint32_t warp_eq[SP_THREADS / 32];
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
        probes[(int64_t)q * nprobe + p] = (e == KEY_EMPTY) ? 0 : (int32_t)(e & 0xffffffffu);
    }
}

constexpr int PREP_THREADS = 1024;

__global__ void __launch_bounds__(PREP_THREADS)
scan_prepare_kernel(const int32_t* __restrict__ probes, int nq, int nprobe,
                    const int32_t* __restrict__ list_page_off, const int* __restrict__ d_nvalid,
                    int32_t* __restrict__ probe_page_off, int64_t* __restrict__ qpage_off) {
    __shared__ int64_t part[PREP_THREADS];
    __shared__ int64_t carry;
    const int nvalid = d_nvalid ? *d_nvalid : nq;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < nq; base += PREP_THREADS) {
        int q = base + threadIdx.x;
        int64_t tot = 0;
        if (q < nq) {
            int32_t* po = probe_page_off + (int64_t)q * (nprobe + 1);
            int acc = 0;
            po[0] = 0;
            for (int p = 0; p < nprobe; ++p) {
                if (q < nvalid) {
                    int l = probes[(int64_t)q * nprobe + p];
                    acc += list_page_off[l + 1] - list_page_off[l];
                }
                po[p + 1] = acc;
            }
            tot = acc;
        }
        part[threadIdx.x] = tot;
        __syncthreads();
        // inclusive Hillis-Steele scan of this chunk
        for (int o = 1; o < PREP_THREADS; o <<= 1) {
            int64_t v = (threadIdx.x >= o) ? part[threadIdx.x - o] : 0;
            __syncthreads();
            part[threadIdx.x] += v;
            __syncthreads();
        }
        if (q < nq) qpage_off[q + 1] = carry + part[threadIdx.x];
        __syncthreads();
        if (threadIdx.x == PREP_THREADS - 1) carry += part[PREP_THREADS - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0) qpage_off[0] = 0;
}

}  // namespace

void select_probes(const float* s, int nq, int nlist, int nprobe, int32_t* probes,
                   cudaStream_t st) {
    if (nq <= 0) return;
    int np_pad = next_pow2(nprobe);
    size_t smem = (size_t)np_pad * sizeof(uint64_t);
    select_probes_kernel<<<nq, SP_THREADS, smem, st>>>(s, nlist, nprobe, np_pad, probes);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

void scan_prepare(const int32_t* probes, int nq, int nprobe, const int32_t* list_page_off,
                  const int* d_nvalid, int32_t* probe_page_off, int64_t* qpage_off,
                  cudaStream_t st) {
    scan_prepare_kernel<<<1, PREP_THREADS, 0, st>>>(probes, nq, nprobe, list_page_off, d_nvalid,
                                                    probe_page_off, qpage_off);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq
