// noalloc.cu — search without any device allocation.
//
// Some callers cannot allocate device memory while they search: code running
// inside a host that owns a fixed memory pool and forbids cudaMalloc after
// start-up, real-time paths where an allocation may block or fail at the worst
// moment, or plug-ins whose framework has already reserved the whole GPU. For
// them, jhq_search_device_noalloc runs the ordinary search pipeline (rotate,
// coarse scores + probes, scan plan, ADC scan, refine) but places every
// per-batch temporary — rotated queries, coarse scores, probe lists, page
// buckets, candidate lists — in one fixed array that is part of the library
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
//    Serialise them. What must start at a fixed value is reset by every call:
//    the flat-index probe list, the per-list pair counters and the per-query
//    pruning bounds.
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
    if (paging()) fail(JHQ_ESTATE, "search_device_noalloc: not available with list paging");
    unsigned char* base = scratch_for(dev_);
    cudaStream_t s = stream ? stream : stream_;

    const int Bq = (int)std::min<int64_t>(p_.batch_size, nq);
    const BatchShape sh = batch_shape(Bq, k);
    const int np = p_.nprobe, nl = p_.nlist;

    // carve the batch temporaries out of the fixed array
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = up256(off + bytes); return base + o; };
    BatchBufs b;
    b.q_rot = reinterpret_cast<float*>(take((size_t)Bq * d_ * 4));
    b.rotq = reinterpret_cast<float*>(take(std::max<size_t>(1, rotq_scratch_floats(Bq)) * 4));
    b.scores = nl > 1 ? reinterpret_cast<float*>(take(coarse_scratch_floats(Bq) * 4)) : nullptr;
    b.probes = reinterpret_cast<int32_t*>(take((size_t)Bq * np * 4));
    b.plan.cnt = reinterpret_cast<int32_t*>(take((size_t)(nl + 1) * 4));
    b.plan.bucket_off = reinterpret_cast<int32_t*>(take((size_t)(nl + 1) * 4));
    b.plan.unit_off = reinterpret_cast<int32_t*>(take((size_t)(nl + 1) * 4));
    b.plan.fill = reinterpret_cast<int32_t*>(take((size_t)nl * 4));
    b.plan.bucket = reinterpret_cast<int2*>(take((size_t)Bq * np * 8));
    b.plan.cpo = reinterpret_cast<int32_t*>(take((size_t)Bq * (np + 1) * 4));
    b.plan.qslot_off = reinterpret_cast<int64_t*>(take((size_t)(Bq + 1) * 8));
    b.plan.gthr = reinterpret_cast<uint64_t*>(take((size_t)Bq * 8));
    b.cand = reinterpret_cast<uint64_t*>(take((size_t)sh.max_slots * sh.ck * 8));
    if (pilot_lists() > 0) {
        b.pkeys = reinterpret_cast<uint64_t*>(take((size_t)Bq * PILOT_SPLIT * sh.ck * 8));
        b.pscores = reinterpret_cast<float*>(take((size_t)Bq * pilot_lists() * 4));
    }
    if (off > NOALLOC_SCRATCH_BYTES)
        fail(JHQ_EINVAL, "search_device_noalloc: batch needs " + std::to_string(off) +
                         " bytes of scratch, the fixed array holds " +
                         std::to_string(NOALLOC_SCRATCH_BYTES) + " (reduce batch_size or k)");
    if (nl == 1) JHQ_CUDA(cudaMemsetAsync(b.probes, 0, (size_t)Bq * np * 4, s));

    for (int64_t q0 = 0; q0 < nq; q0 += Bq) {
        const int nv = (int)std::min<int64_t>(Bq, nq - q0);
        enqueue_pipeline(d_q + q0 * d_, nv, nullptr, sh, b, d_dists + q0 * k, d_ids + q0 * k, s,
                         nullptr);
    }
}

}  // namespace jhq
