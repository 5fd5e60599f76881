// noalloc.cu — search without any device allocation.
//
// Some callers cannot allocate device memory while they search: code running
// inside a host that owns a fixed memory pool and forbids cudaMalloc after
// start-up, real-time paths where an allocation may block or fail at the worst
// moment, or plug-ins whose framework has already reserved the whole GPU. For
// them, jhq_search_device_noalloc runs the ordinary search pipeline (rotate,
// coarse scores + probes, scan partition, ADC scan, refine) but places every
// per-batch temporary — rotated queries, coarse scores, probe lists, page
// offsets, candidate lists — in one fixed array that is part of the library
// image, so each GPU that loads the library holds NOALLOC_SCRATCH_BYTES of it
// until the process exits. The caller passes the queries and the outputs; the
// index's own stored data (codes, codebooks) were allocated by train/add.
//
// Rules of use:
//  - the first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (and sets kernel attributes) for that device; make that
//    first call before any stream capture;
//  - a batch whose temporaries exceed NOALLOC_SCRATCH_BYTES is rejected with
//    JHQ_EINVAL (reduce batch_size or k);
//  - all calls on a device share the one array and it keeps the previous call's
//    contents: two calls that overlap on the GPU (different streams, or two
//    indexes on different host threads) race and corrupt each other's results.
//    Serialise them. The flat-index probe list, the only part that must start
//    at a fixed value, is cleared by every call.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>

#include "index.h"
#include "kernels.cuh"

namespace jhq {

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = 16u << 20;      // 16 MiB per GPU

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_setup_mu;
unsigned char* g_scratch_ptr[MAX_DEVICES] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
unsigned char* scratch_for(int dev) {
    if (dev < 0 || dev >= MAX_DEVICES) fail(JHQ_EINVAL, "noalloc: device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        JHQ_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        scan_configure();
        refine_configure();
        g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
    }
    return g_scratch_ptr[dev];
}

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

void Index::search_device_noalloc(const float* d_q, int64_t nq, int k, float* d_dists,
                                  int32_t* d_ids, cudaStream_t stream) {
    DeviceGuard g(dev_);
    check_search_args(nq, k);
    if (nq == 0) return;
    if (!d_q || !d_dists || !d_ids) fail(JHQ_EINVAL, "search_device_noalloc: null buffer");
    unsigned char* base = scratch_for(dev_);
    cudaStream_t s = stream ? stream : stream_;

    const int ck = std::max(k, (int)std::ceil(p_.alpha * (float)k));
    const int ck_pad = std::max(32, next_pow2(ck));
    const bool nib = scan_uses_nibbles(d_, M_, B_);
    const int grid = scan_grid_for(Mp_, d_, ck_pad, nib);
    const int Bq = (int)std::min<int64_t>(p_.batch_size, nq);
    const int np = p_.nprobe, nl = p_.nlist;

    // carve the batch temporaries out of the fixed array
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = up256(off + bytes); return base + o; };
    float* q_rot = reinterpret_cast<float*>(take((size_t)Bq * d_ * 4));
    float* scores = nl > 1 ? reinterpret_cast<float*>(take((size_t)Bq * nl * 4)) : nullptr;
    int32_t* probes = reinterpret_cast<int32_t*>(take((size_t)Bq * np * 4));
    int32_t* ppo = reinterpret_cast<int32_t*>(take((size_t)Bq * (np + 1) * 4));
    int64_t* qpage_off = reinterpret_cast<int64_t*>(take((size_t)(Bq + 1) * 8));
    uint64_t* cand = reinterpret_cast<uint64_t*>(take((size_t)(grid + Bq) * ck * 8));
    if (off > NOALLOC_SCRATCH_BYTES)
        fail(JHQ_EINVAL, "search_device_noalloc: batch needs " + std::to_string(off) +
                         " bytes of scratch, the fixed array holds " +
                         std::to_string(NOALLOC_SCRATCH_BYTES) + " (reduce batch_size or k)");
    if (nl == 1) JHQ_CUDA(cudaMemsetAsync(probes, 0, (size_t)Bq * np * 4, s));

    for (int64_t q0 = 0; q0 < nq; q0 += Bq) {
        const int nv = (int)std::min<int64_t>(Bq, nq - q0);
        rotate_device(d_q + q0 * d_, nv, q_rot, s);
        if (nl > 1) {
            gemm_rows(q_rot, dcentsT_.get(), scores, nv, d_, nl, EPI_COARSE, dnorms_.get(), s);
            select_probes(scores, nv, nl, np, probes, s);
        }
        scan_prepare(probes, nv, np, dlist_page_off_.get(), nullptr, ppo, qpage_off, s);
        ScanArgs sa;
        sa.q_rot = q_rot; sa.c1d = dc1d_.get(); sa.probes = probes;
        sa.probe_page_off = ppo; sa.qpage_off = qpage_off;
        sa.list_page_off = dlist_page_off_.get(); sa.pages = dpages_.get();
        sa.slot_ids = dslot_ids_.get(); sa.cand = cand;
        sa.nq = nv; sa.d = d_; sa.M = M_; sa.Mp = Mp_; sa.B = B_; sa.nprobe = np;
        sa.ck = ck; sa.ck_pad = ck_pad; sa.grid = grid;
        scan_topck(sa, s);
        RefineArgs ra;
        ra.q_rot = q_rot; ra.res_c1d = dres_.get(); ra.cand = cand;
        ra.qpage_off = qpage_off; ra.rcodes = drcodes_.get(); ra.corr = dcorr_.get();
        ra.out_dists = d_dists + q0 * k; ra.out_ids = d_ids + q0 * k;
        ra.nq = nv; ra.d = d_; ra.Br = Br_; ra.bpv_pad = bpv_pad_; ra.ck = ck;
        ra.ck_pad = ck_pad; ra.k = k; ra.grid = grid;
        refine_topk(ra, s);
    }
}

}  // namespace jhq
