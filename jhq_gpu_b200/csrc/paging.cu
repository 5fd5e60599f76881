// paging.cu — out-of-core list paging for indexes larger than device memory.
//
// The reference keeps every code on one GPU; its hblock_v39-v43 builds page
// list blocks through a bounded GPU region pool in waves
// (hblock_v41/README.md, VERSIONS.md:533-555). The same idea for the JHQ IVF
// index:
//
//   * the page layout (primary codes of each list, padded to 32-vector pages),
//     the slot ids, the residual codes, corr and the kept vectors of the exact
//     rerank live in pinned host memory mapped into the device address space;
//   * a search batch runs rotation + coarse step on the device, copies its
//     probe lists back, and cuts the batch into waves of consecutive queries
//     whose probed lists fit the device page pool together;
//   * per wave, one gather kernel stages those lists' pages and slot ids from
//     host memory into the pool (each list read over the host link once per
//     wave, however many queries probe it), the list page offsets are remapped
//     to the pool, and the ordinary plan / scan / refine run on the pool; the
//     refine reads the few residual rows it needs (ck per query) straight from
//     mapped host memory.
//
// Results are identical to the resident index: same codes, same probe lists,
// and the scan's top-ck is exact whatever the page order.
#include <algorithm>
#include <cstring>
#include <vector>

#include "index.h"
#include "kernels.cuh"

namespace jhq {
namespace {

// Segment s copies seg[3s+2] bytes from host byte offset seg[3s] to pool byte
// offset seg[3s+1] (16-byte aligned, multiples of 16 bytes).
__global__ void gather_segments_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                       const int64_t* __restrict__ seg, int nseg) {
    for (int s = blockIdx.x; s < nseg; s += gridDim.x) {
        const uint4* a = reinterpret_cast<const uint4*>(src + seg[3 * s]);
        uint4* b = reinterpret_cast<uint4*>(dst + seg[3 * s + 1]);
        const int64_t n = seg[3 * s + 2] / 16;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) b[i] = a[i];
    }
}

}  // namespace

void Index::set_list_paging(int64_t pool_bytes) {
    DeviceGuard g(dev_);
    if (pool_bytes < 0) fail(JHQ_EINVAL, "list paging: pool size must be >= 0");
    if (ntotal_ > 0 || cap_ > 0)
        fail(JHQ_ESTATE, "list paging: choose it before the first add()");
    if (pool_bytes > 0 && p_.nlist <= 1)
        fail(JHQ_EINVAL, "list paging needs an IVF index (nlist > 1)");
    const int64_t page_bytes = (int64_t)Mp_ * 32 + 32 * 4;
    pool_pages_ = pool_bytes / page_bytes;
    if (pool_bytes > 0 && pool_pages_ < 1) fail(JHQ_EINVAL, "list paging: pool smaller than one page");
    destroy_graph();
    ws_.batch_cap = 0;
}

// Pages [npages][Mp/16][32][16] and slot ids in host memory (the layout
// scatter_pages_kernel builds on the device for a resident index).
void Index::build_host_pages(const std::vector<int32_t>& lpo, const std::vector<int32_t>& slots) {
    const int G = Mp_ / 16;
    const size_t npg = (size_t)npages_;
    hpages_.grow(std::max<size_t>(16, npg * Mp_ * 32), 0);
    hslot_ids_.grow(std::max<size_t>(1, slots.size()), 0);
    std::memcpy(hslot_ids_.get(), slots.data(), slots.size() * 4);
    uint8_t* pages = hpages_.get();
    const uint8_t* pc = hpcodes_.get();
    for (size_t slot = 0; slot < slots.size(); ++slot) {
        const int32_t v = slots[slot];
        const size_t page = slot / 32, lane = slot % 32;
        for (int g = 0; g < G; ++g) {
            uint8_t* dst = pages + ((page * G + g) * 32 + lane) * 16;
            for (int b = 0; b < 16; ++b) {
                const int m = g * 16 + b;
                dst[b] = (v >= 0 && m < M_) ? pc[(size_t)v * M_ + m] : 0;
            }
        }
    }
    h_lpo_ = lpo;
    int64_t maxl = 0;
    for (int c = 0; c < p_.nlist; ++c) maxl = std::max<int64_t>(maxl, lpo[c + 1] - lpo[c]);
    if (maxl * std::min(p_.nprobe, p_.nlist) > pool_pages_ && maxl > pool_pages_)
        fail(JHQ_EINVAL, "list paging: the page pool is smaller than the largest list");
    dpool_pages_.ensure((size_t)pool_pages_ * Mp_ * 32);
    dpool_slots_.ensure((size_t)pool_pages_ * 32);
    dlpo_wave_.ensure((size_t)p_.nlist + 1);
}

void Index::run_paged_batch(const float* q_in, int nq, float* out_d, int32_t* out_i,
                            cudaStream_t s) {
    const int np = p_.nprobe, nl = p_.nlist;
    BatchShape sh = batch_shape(ws_.batch_cap, ws_.k);
    rotate_queries_device(q_in, nq, ws_.q_rot.get(), ws_.rotq.get(), s);
    coarse_probes(ws_.q_rot.get(), nq, ws_.batch_cap, np, ws_.scores.get(), ws_.probes.get(), s);
    std::vector<int32_t> pr((size_t)nq * np);
    d2h(pr.data(), ws_.probes.get(), pr.size(), s);
    JHQ_CUDA(cudaStreamSynchronize(s));
    if ((coarse_tc_ || rot_tc_) && coarse_tc_error(true))
        fail(JHQ_ETIMEDOUT, "search: a tensor-core coarse wait gave up");

    std::vector<int32_t> stamp(nl, -1), wave_lists, lpo_w(nl + 1);
    std::vector<int64_t> seg;
    const int64_t page_bytes = (int64_t)Mp_ * 32;
    int q0 = 0, wave = 0;
    while (q0 < nq) {
        // the longest run of queries from q0 whose probed lists fit the pool
        wave_lists.clear();
        int64_t pages = 0;
        int q1 = q0;
        for (; q1 < nq; ++q1) {
            int64_t add = 0;
            for (int p = 0; p < np; ++p) {
                const int l = pr[(size_t)q1 * np + p];
                if (stamp[l] != wave) add += h_lpo_[l + 1] - h_lpo_[l];
            }
            if (pages + add > pool_pages_) {
                if (q1 == q0) fail(JHQ_EINVAL, "list paging: one query's lists exceed the page pool");
                break;
            }
            pages += add;
            for (int p = 0; p < np; ++p) {
                const int l = pr[(size_t)q1 * np + p];
                if (stamp[l] != wave) { stamp[l] = wave; wave_lists.push_back(l); }
            }
        }
        // remapped offsets: wave lists packed in the pool, others empty
        std::sort(wave_lists.begin(), wave_lists.end());
        seg.clear();
        int64_t at = 0;
        size_t wi = 0;
        for (int l = 0; l < nl; ++l) {
            lpo_w[l] = (int32_t)at;
            if (wi < wave_lists.size() && wave_lists[wi] == l) {
                const int64_t n = h_lpo_[l + 1] - h_lpo_[l];
                if (n > 0) {
                    seg.push_back((int64_t)h_lpo_[l] * page_bytes);
                    seg.push_back(at * page_bytes);
                    seg.push_back(n * page_bytes);
                }
                at += n;
                ++wi;
            }
        }
        lpo_w[nl] = (int32_t)at;
        const int nseg = (int)(seg.size() / 3);
        // slot ids follow the same segments (128 bytes per page)
        const size_t nseg_all = seg.size();
        for (size_t i = 0; i < nseg_all; i += 3) {
            seg.push_back(seg[i] / page_bytes * 128);
            seg.push_back(seg[i + 1] / page_bytes * 128);
            seg.push_back(seg[i + 2] / page_bytes * 128);
        }
        dseg_.ensure(std::max<size_t>(3, seg.size()));
        h2d(dseg_.get(), seg.data(), seg.size(), s);
        h2d(dlpo_wave_.get(), lpo_w.data(), lpo_w.size(), s);
        if (nseg > 0) {
            gather_segments_kernel<<<std::min(nseg, 4096), 256, 0, s>>>(
                hpages_.get(), dpool_pages_.get(), dseg_.get(), nseg);
            JHQ_LAUNCH_CHECK();
            gather_segments_kernel<<<std::min(nseg, 4096), 256, 0, s>>>(
                reinterpret_cast<const uint8_t*>(hslot_ids_.get()),
                reinterpret_cast<uint8_t*>(dpool_slots_.get()), dseg_.get() + 3 * nseg, nseg);
            JHQ_LAUNCH_CHECK();
            count_launch(2);
        }
        // plan / scan / refine of queries [q0, q1) over the pool
        const int nw = q1 - q0;
        const int32_t* probes = ws_.probes.get() + (size_t)q0 * np;
        const float* q_rot = ws_.q_rot.get() + (size_t)q0 * d_;
        PlanBufs b{ws_.cnt.get(), ws_.bucket_off.get(), ws_.unit_off.get(), ws_.fill.get(),
                   ws_.bucket.get(), ws_.cpo.get(), ws_.qslot_off.get(), ws_.gthr.get()};
        if (sh.qmajor)
            plan_build_qmajor(probes, nw, np, dlpo_wave_.get(), nullptr, sh.chunk_pages, b, s);
        else
            plan_build(probes, nw, np, nl, dlpo_wave_.get(), nullptr, sh.chunk_pages,
                       sh.mode == 0 ? 1 : sh.mode, b, s);
        ScanArgs sa;
        sa.q_rot = q_rot; sa.c1d = dc1d_.get(); sa.list_page_off = dlpo_wave_.get();
        sa.pages = dpool_pages_.get(); sa.slot_ids = dpool_slots_.get();
        sa.unit_off = b.unit_off; sa.bucket_off = b.bucket_off; sa.bucket = b.bucket;
        sa.cpo = b.cpo; sa.qslot_off = b.qslot_off; sa.gthr = b.gthr; sa.cand = ws_.cand.get();
        sa.nq = nw; sa.nlist = nl; sa.d = d_; sa.M = M_; sa.Mp = Mp_; sa.B = B_;
        sa.nprobe = np; sa.ck = sh.ck; sa.ck_pad = sh.ck_pad; sa.grid = sh.grid;
        sa.chunk_pages = sh.chunk_pages; sa.mode = sh.mode; sa.qmajor = sh.qmajor;
        sa.probes = probes;
        scan_topck(sa, s);
        RefineArgs ra;
        ra.q_rot = q_rot; ra.res_c1d = dres_.get(); ra.cand = ws_.cand.get();
        ra.res_per_sub = res_per_sub_ ? 1 : 0; ra.M = M_;
        ra.qslot_off = b.qslot_off; ra.gthr = b.gthr; ra.rcodes = hrcodes_.get();
        ra.corr = hcorr_.get(); ra.out_dists = out_d + (size_t)q0 * sh.k;
        ra.out_ids = out_i + (size_t)q0 * sh.k;
        ra.nq = nw; ra.d = d_; ra.Br = Br_; ra.bpv_pad = bpv_pad_; ra.ck = sh.ck;
        ra.ck_pad = sh.ck_pad; ra.k = sh.k; ra.kr = sh.kr;
        if (keep_raw_ && rerank_ > 0) {
            ra.q_raw = q_in + (size_t)q0 * d_;
            ra.raw = hraw_.get();
        }
        refine_topk(ra, s);
        ++paging_waves_;
        q0 = q1;
        ++wave;
        // the host-side tables are rewritten for the next wave only after this
        // wave's copies have read them
        JHQ_CUDA(cudaStreamSynchronize(s));
    }
}

}  // namespace jhq
