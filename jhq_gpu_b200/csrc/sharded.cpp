// sharded.cpp — jhq::ShardedIndex (see sharded.h).
#include "sharded.h"

#include <algorithm>
#include <climits>
#include <cstring>
#include <exception>
#include <thread>

#include "kernels.cuh"

namespace jhq {

namespace {
constexpr int64_t QCHUNK = 16384;        // queries per search chunk
constexpr int64_t ACHUNK = 1 << 20;      // rows per add chunk

// Runs f(s) for every shard on its own host thread; rethrows the first error.
template <class F>
void for_each_shard(int n, F&& f) {
    std::vector<std::exception_ptr> err(n);
    std::vector<std::thread> th;
    for (int s = 0; s < n; ++s)
        th.emplace_back([&, s] {
            try { f(s); } catch (...) { err[s] = std::current_exception(); }
        });
    for (auto& t : th) t.join();
    for (auto& e : err)
        if (e) std::rethrow_exception(e);
}
}  // namespace

ShardedIndex::ShardedIndex(int d, const Params& p, const std::vector<int>& devices)
    : d_(d), p_(p) {
    if (devices.empty()) fail(JHQ_EINVAL, "sharded index: need at least one shard");
    if (devices.size() > 64) fail(JHQ_EINVAL, "sharded index: at most 64 shards");
    int ndev = 0;
    JHQ_CUDA(cudaGetDeviceCount(&ndev));
    for (int dv : devices)
        if (dv < 0 || dv >= ndev) fail(JHQ_EINVAL, "sharded index: bad device ordinal");
    b_.resize(devices.size());
    try {
        for (size_t s = 0; s < devices.size(); ++s) {
            Params ps = p;
            ps.device = devices[s];
            sh_.emplace_back(new Index(d, ps));
            b_[s].dev = devices[s];
            DeviceGuard g(devices[s]);
            JHQ_CUDA(cudaStreamCreateWithFlags(&b_[s].st, cudaStreamNonBlocking));
            JHQ_CUDA(cudaEventCreateWithFlags(&b_[s].ev_probe, cudaEventDisableTiming));
            JHQ_CUDA(cudaEventCreateWithFlags(&b_[s].ev_done, cudaEventDisableTiming));
        }
        p_ = sh_[0]->params();
        // direct peer access where the hardware offers it (copies work without it)
        for (size_t s = 0; s < devices.size(); ++s)
            for (size_t t = 0; t < devices.size(); ++t) {
                if (devices[s] == devices[t]) continue;
                int ok = 0;
                JHQ_CUDA(cudaDeviceCanAccessPeer(&ok, devices[s], devices[t]));
                if (!ok) continue;
                DeviceGuard g(devices[s]);
                const cudaError_t e = cudaDeviceEnablePeerAccess(devices[t], 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) JHQ_CUDA(e);
                cudaGetLastError();
            }
    } catch (...) {
        for (auto& b : b_) {
            if (b.st) cudaStreamDestroy(b.st);
            if (b.ev_probe) cudaEventDestroy(b.ev_probe);
            if (b.ev_done) cudaEventDestroy(b.ev_done);
        }
        throw;
    }
}

ShardedIndex::~ShardedIndex() {
    for (auto& b : b_) {
        DeviceGuard g(b.dev);
        if (b.st) cudaStreamSynchronize(b.st);
        b.q.release(); b.D.release(); b.I.release(); b.probes.release();
        if (b.st) cudaStreamDestroy(b.st);
        if (b.ev_probe) cudaEventDestroy(b.ev_probe);
        if (b.ev_done) cudaEventDestroy(b.ev_done);
    }
    if (!b_.empty()) {
        DeviceGuard g(b_[0].dev);
        allD_.release(); allI_.release(); outD_.release(); outI_.release();
    }
}

void ShardedIndex::sync_artefacts() {
    Index& s0 = *sh_[0];
    std::vector<float> Pi((size_t)d_ * d_), c1d(s0.K1D()), res((size_t)s0.residual_floats()),
        cents((size_t)p_.nlist * d_);
    float sigma = 0.0f;
    s0.get_trained(Pi.data(), c1d.data(), res.data(), cents.data(), &sigma);
    const std::vector<float>& pc = s0.pilot_centroids();
    for_each_shard(nshards() - 1, [&](int s) {
        sh_[s + 1]->set_residual_codebooks(s0.residual_per_subspace());
        sh_[s + 1]->set_trained(Pi.data(), c1d.data(), res.data(), cents.data(), sigma);
        if (s0.pilot_lists() > 0) sh_[s + 1]->set_pilot(pc.data(), s0.pilot_lists());
    });
}

// JHQGpuIndex::train (jhq_gpu_index.cu:333-364) on the first shard; the other
// shards import its artefacts.
void ShardedIndex::train(const float* h_x, int64_t n) {
    if (ntotal_ > 0) fail(JHQ_ESTATE, "train() after add()");
    sh_[0]->train(h_x, n);
    sync_artefacts();
}

void ShardedIndex::add(const float* h_x, int64_t n) {
    if (!trained()) fail(JHQ_ESTATE, "call train() before add()");
    if (n < 0 || (n > 0 && !h_x)) fail(JHQ_EINVAL, "add: bad input");
    if (n == 0) return;
    if (ntotal_ + n > INT32_MAX) fail(JHQ_EINVAL, "add: more than 2^31-1 vectors");
    const int S = nshards();
    std::vector<std::vector<float>> part(S);
    for (int64_t r0 = 0; r0 < n; r0 += ACHUNK) {
        const int64_t nr = std::min(ACHUNK, n - r0);
        for (int s = 0; s < S; ++s) part[s].clear();
        for (int64_t r = 0; r < nr; ++r) {              // global id ntotal_ + r0 + r
            const int s = (int)((ntotal_ + r0 + r) % S);
            const float* src = h_x + (r0 + r) * d_;
            part[s].insert(part[s].end(), src, src + d_);
        }
        for_each_shard(S, [&](int s) {
            const int64_t ns = (int64_t)(part[s].size() / d_);
            if (ns > 0) sh_[s]->add(part[s].data(), ns);
        });
    }
    ntotal_ += n;
}

void ShardedIndex::set_nprobe(int nprobe) {
    for (auto& s : sh_) s->set_nprobe(nprobe);
    p_.nprobe = sh_[0]->params().nprobe;
}

void ShardedIndex::search(const float* h_q, int64_t nq, int k, float* h_dists, int32_t* h_ids) {
    if (nq < 0) fail(JHQ_EINVAL, "nq must be >= 0");
    if (k <= 0) fail(JHQ_EINVAL, "k must be positive");
    if (!trained() || ntotal_ == 0) fail(JHQ_ESTATE, "index is empty");
    if (nq == 0) return;
    if (!h_q || !h_dists || !h_ids) fail(JHQ_EINVAL, "search: null buffer");
    const int S = nshards();
    std::vector<int> act;                                  // shards holding vectors
    for (int s = 0; s < S; ++s)
        if (sh_[s]->ntotal() > 0) act.push_back(s);
    const int R = (int)act.size();
    const int np = sh_[0]->params().nprobe;
    const int64_t QC = std::min<int64_t>(QCHUNK, nq);
    for (int s : act) {
        DeviceGuard g(b_[s].dev);
        b_[s].q.ensure((size_t)QC * d_);
        b_[s].D.ensure((size_t)QC * k);
        b_[s].I.ensure((size_t)QC * k);
        b_[s].probes.ensure((size_t)QC * np);
    }
    const int dev0 = b_[act[0]].dev;
    cudaStream_t st0 = b_[act[0]].st;
    {
        DeviceGuard g(dev0);
        allD_.ensure((size_t)R * QC * k);
        allI_.ensure((size_t)R * QC * k);
        outD_.ensure((size_t)QC * k);
        outI_.ensure((size_t)QC * k);
    }
    hq_.ensure((size_t)QC * d_);
    hD_.ensure((size_t)QC * k);
    hI_.ensure((size_t)QC * k);

    for (int64_t q0 = 0; q0 < nq; q0 += QC) {
        const int64_t nc = std::min(QC, nq - q0);
        std::memcpy(hq_.get(), h_q + q0 * d_, (size_t)nc * d_ * sizeof(float));
        // 1. queries to every shard; 2. coarse step split by queries
        const int64_t per = (nc + R - 1) / R;
        for (int r = 0; r < R; ++r) {
            ShardBufs& b = b_[act[r]];
            DeviceGuard g(b.dev);
            JHQ_CUDA(cudaMemcpyAsync(b.q.get(), hq_.get(), (size_t)nc * d_ * sizeof(float),
                                     cudaMemcpyHostToDevice, b.st));
            const int64_t lo = std::min(nc, r * per), hi = std::min(nc, lo + per);
            if (hi > lo)
                sh_[act[r]]->probe_device(b.q.get() + lo * d_, hi - lo, b.probes.get() + lo * np, b.st);
            JHQ_CUDA(cudaEventRecord(b.ev_probe, b.st));
        }
        for (int t = 0; t < R; ++t) {
            ShardBufs& bt = b_[act[t]];
            DeviceGuard g(bt.dev);
            for (int r = 0; r < R; ++r) {
                if (r == t) continue;
                const int64_t lo = std::min(nc, r * per), hi = std::min(nc, lo + per);
                if (hi <= lo) continue;
                ShardBufs& br = b_[act[r]];
                JHQ_CUDA(cudaStreamWaitEvent(bt.st, br.ev_probe, 0));
                JHQ_CUDA(cudaMemcpyPeerAsync(bt.probes.get() + lo * np, bt.dev,
                                             br.probes.get() + lo * np, br.dev,
                                             (size_t)(hi - lo) * np * sizeof(int32_t), bt.st));
            }
            // 3. scan + refine with the shared lists, global ids
            sh_[act[t]]->search_device_probes(bt.q.get(), bt.probes.get(), nc, k, bt.D.get(),
                                              bt.I.get(), bt.st);
            remap_ids(bt.I.get(), nc * k, S, act[t], bt.st);
            JHQ_CUDA(cudaEventRecord(bt.ev_done, bt.st));
        }
        // 4. gather on the first shard's device, merge, copy out
        {
            DeviceGuard g(dev0);
            for (int r = 0; r < R; ++r) {
                ShardBufs& br = b_[act[r]];
                JHQ_CUDA(cudaStreamWaitEvent(st0, br.ev_done, 0));
                JHQ_CUDA(cudaMemcpyPeerAsync(allD_.get() + (size_t)r * nc * k, dev0, br.D.get(), br.dev,
                                             (size_t)nc * k * sizeof(float), st0));
                JHQ_CUDA(cudaMemcpyPeerAsync(allI_.get() + (size_t)r * nc * k, dev0, br.I.get(), br.dev,
                                             (size_t)nc * k * sizeof(int32_t), st0));
            }
            merge_shard_lists(allD_.get(), allI_.get(), R, nc, k, outD_.get(), outI_.get(), st0);
            JHQ_CUDA(cudaMemcpyAsync(hD_.get(), outD_.get(), (size_t)nc * k * sizeof(float),
                                     cudaMemcpyDeviceToHost, st0));
            JHQ_CUDA(cudaMemcpyAsync(hI_.get(), outI_.get(), (size_t)nc * k * sizeof(int32_t),
                                     cudaMemcpyDeviceToHost, st0));
        }
        // every shard's stream is idle before its buffers are reused
        for (int r = 0; r < R; ++r) {
            DeviceGuard g(b_[act[r]].dev);
            JHQ_CUDA(cudaStreamSynchronize(b_[act[r]].st));
        }
        std::memcpy(h_dists + q0 * k, hD_.get(), (size_t)nc * k * sizeof(float));
        std::memcpy(h_ids + q0 * k, hI_.get(), (size_t)nc * k * sizeof(int32_t));
    }
}

}  // namespace jhq
