// index.cu — jhq::Index: train / add / search orchestration on one GPU.
// Mirrors JHQGpuIndex (jhq_v14_streaming_add/jhq_gpu_index.cu) and
// search_gpu (jhq_v14_streaming_add/search.cu:388-445); see index.h for
// the device data layout.
#include "index.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <thread>

#include "kernels.cuh"
#include "train_cpu.h"

namespace jhq {

namespace {
constexpr int MAX_CK_PAD = 256;

}  // namespace

// ---- construction: JHQGpuIndex ctor validation (jhq_gpu_index.cu:103-131) ----
Index::Index(int d, const Params& p) : p_(p) {
    if (d <= 0) fail(JHQ_EINVAL, "d must be positive");
    if (p.M <= 0) fail(JHQ_EINVAL, "M must be positive");
    if (d % p.M != 0) fail(JHQ_EINVAL, "d must be divisible by M");
    if (p.B <= 0 || p.B % (d / p.M) != 0) fail(JHQ_EINVAL, "B must be divisible by Ds = d/M");
    if (p.B > 8) fail(JHQ_EINVAL, "B must be <= 8");
    if (p.Br != 4 && p.Br != 8) fail(JHQ_EINVAL, "Br must be 4 or 8");
    if (p.nlist <= 0) fail(JHQ_EINVAL, "nlist must be positive");
    if (p.nprobe <= 0) fail(JHQ_EINVAL, "nprobe must be positive");
    if (p.ivf_iters <= 0) fail(JHQ_EINVAL, "ivf_iters must be positive");
    if (p.batch_size <= 0) fail(JHQ_EINVAL, "batch_size must be positive");
    if (p.add_batch <= 0) fail(JHQ_EINVAL, "add_batch must be positive");
    if (!(p.alpha > 0.0f)) fail(JHQ_EINVAL, "alpha must be positive");
    d_ = d; M_ = p.M; B_ = p.B; Br_ = p.Br;
    Ds_ = d / M_; bpd_ = B_ / Ds_; K1D_ = 1 << bpd_; Kr_ = 1 << Br_;
    bpv_ = (d * Br_ + 7) / 8;
    bpv_pad_ = (int)ceil_div(bpv_, 16) * 16;
    Mp_ = (int)ceil_div(M_, 16) * 16;
    p_.nprobe = std::min(p.nprobe, p.nlist);
    if (d > 16384) fail(JHQ_EINVAL, "d must be <= 16384");
    if (scan_smem_bytes(Mp_, d_, 32, scan_mode_for(d_, M_, B_, 1.0)) > 227 * 1024)
        fail(JHQ_EINVAL, "M too large: the per-query byte LUT (M x 1 KB) must fit in shared memory");
    if (p.device < 0) JHQ_CUDA(cudaGetDevice(&dev_));
    else dev_ = p.device;
    p_.device = dev_;
    DeviceGuard g(dev_);
    JHQ_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
}

Index::~Index() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(dev_);
    if (stream_) cudaStreamSynchronize(stream_);
    destroy_graph();
    for (auto& e : prof_ev_)
        if (e) cudaEventDestroy(e);
    if (stream_) cudaStreamDestroy(stream_);
    // DevBuf / PinnedBuf members free themselves (device still current).
    dPi_.release(); dc1d_.release(); dres_.release(); dcentsT_.release(); dcents_.release(); dpilot_centsT_.release(); dpilot_cents_.release(); dpilot_norms_.release(); dpilot_off_.release(); dpilot_ids_.release(); dcents3_.release(); dassign_scratch_.release(); dnorms_.release();
    dpcodes_.release(); drcodes_.release(); dpages_.release(); dcorr_.release();
    dassign_.release(); dslot_ids_.release(); dlist_page_off_.release();
    ws_.q.release(); ws_.q_rot.release(); ws_.scores.release(); ws_.out_d.release();
    ws_.probes.release(); ws_.out_i.release(); ws_.cnt.release(); ws_.bucket_off.release();
    ws_.unit_off.release(); ws_.fill.release(); ws_.cpo.release(); ws_.bucket.release();
    ws_.qslot_off.release(); ws_.cand.release(); ws_.gthr.release(); ws_.nvalid.release();
    ws_.h_q.release(); ws_.h_d.release(); ws_.h_i.release(); ws_.h_nvalid.release();
    cudaSetDevice(prev);
}

void Index::destroy_graph() {
    if (ws_.exec) cudaGraphExecDestroy(ws_.exec);
    if (ws_.graph) cudaGraphDestroy(ws_.graph);
    ws_.exec = nullptr;
    ws_.graph = nullptr;
    ws_.graph_kernels = 0;
}

// ---- device helpers ----------------------------------------------------------
void Index::rotate_device(const float* d_x, int64_t n, float* d_y, cudaStream_t s) const {
    gemm_rows(d_x, dPi_.get(), d_y, n, d_, d_, EPI_STORE, nullptr, s);
}

bool Index::flat_tc() const {
    const char* e = std::getenv("JHQ_FLAT");
    if (e && std::string(e) == "simt") return false;
    return p_.nlist == 1 && bpd_ == 1 && ntotal_ > 0 && dpop_.size() >= (size_t)ntotal_ &&
           flat_tc_supported(d_, M_, B_, (int)std::min<int64_t>(ntotal_, INT32_MAX)) &&
           !paging();
}

// IVF, 2 bits per dimension, d padded to 128 (C3 / C4): the two-pass
// tensor-core scan (JHQ_IVF=simt keeps the query-major SIMT scan)
bool Index::ivf_tc() const {
    const char* e = std::getenv("JHQ_IVF");
    if (e && std::string(e) == "simt") return false;
    return p_.nlist > 1 && ntotal_ > 0 && ivf_tc_supported(d_, M_, B_, p_.nprobe) && !paging();
}

size_t Index::rotq_scratch_floats(int Bq) const {
    if (!rot_tc_) return 0;
    const size_t q3f = (((size_t)Bq * coarse_tc_k3(d_) + 1) / 2 + 63) & ~(size_t)63;
    return q3f + (size_t)Bq * coarse_tc_tiles(d_);
}

void Index::rotate_queries_device(const float* d_x, int64_t n, float* d_y, float* scratch,
                                  cudaStream_t s) const {
    if (!rot_tc_) {
        rotate_device(d_x, n, d_y, s);
        return;
    }
    const size_t q3f = (((size_t)n * coarse_tc_k3(d_) + 1) / 2 + 63) & ~(size_t)63;
    uint16_t* q3 = reinterpret_cast<uint16_t*>(scratch);
    float* tmin = scratch + q3f;
    split3_rows(d_x, n, d_, q3, s);
    coarse_scores_tc(q3, (int)n, dPi3_.get(), dzero_.get(), d_, d_, d_y, tmin, s);
    scale_floats(d_y, n * d_, -0.5f, s);
}

void Index::assign_device(const float* d_y, int64_t n, int32_t* d_assign, cudaStream_t s) {
    if (p_.nlist == 1) {
        JHQ_CUDA(cudaMemsetAsync(d_assign, 0, n * sizeof(int32_t), s));
        return;
    }
    if (coarse_tc_) {
        // tensor-core scores + margin selection of the single nearest list, in
        // row blocks whose score rows stay within about 256 MB
        const int64_t R = std::max<int64_t>(128, std::min<int64_t>(
            n, ((256ll << 20) / ((int64_t)p_.nlist * 4)) / 128 * 128));
        dassign_scratch_.ensure(coarse_scratch_floats((int)R));
        for (int64_t r0 = 0; r0 < n; r0 += R)
            coarse_probes(d_y + r0 * d_, (int)std::min(R, n - r0), (int)R, 1,
                          dassign_scratch_.get(), d_assign + r0, s);
        return;
    }
    // fused GEMM + running argmin, in row blocks within the grid limit
    const int64_t rows = 65535ll * 128;
    for (int64_t r0 = 0; r0 < n; r0 += rows)
        gemm_argmin(d_y + r0 * d_, dcentsT_.get(), dnorms_.get(), std::min(rows, n - r0), d_,
                    p_.nlist, d_assign + r0, s);
}

void Index::upload_trained() {
    dPi_.resize((size_t)d_ * d_);
    h2d(dPi_.get(), Pi_.data(), Pi_.size(), stream_);
    dc1d_.resize(K1D_);
    h2d(dc1d_.get(), c1d_.data(), c1d_.size(), stream_);
    dres_.resize((size_t)residual_floats());
    if (!res_c1d_.empty()) h2d(dres_.get(), res_c1d_.data(), res_c1d_.size(), stream_);
    // Query rotation on the tensor cores: y = x . Pi as the coarse kernel's
    // s~ = 0 - 2 x . Pi[:, c] over the d columns of Pi (bf16 split rows of Pi^T,
    // zero norms), scaled by -1/2 (exact). JHQ_ROTATE=simt keeps the fp32 chains.
    {
        // The tensor-core kernel tiles 128 queries x 256 outputs; batches below
        // ~1k queries leave most SMs idle there and are faster on the fp32
        // chains (C1, batch 64: 34 vs 27 us per batch), so the choice follows
        // the index's batch size (and JHQ_ROTATE=simt|tc forces it).
        const char* rm = std::getenv("JHQ_ROTATE");
        rot_tc_ = d_ <= 2048 && p_.batch_size >= 1024;
        if (rm && std::string(rm) == "simt") rot_tc_ = false;
        if (rm && std::string(rm) == "tc") rot_tc_ = d_ <= 2048;
        if (rot_tc_) {
            std::vector<float> piT((size_t)d_ * d_);
            for (int j = 0; j < d_; ++j)
                for (int c = 0; c < d_; ++c) piT[(size_t)c * d_ + j] = Pi_[(size_t)j * d_ + c];
            std::vector<uint16_t> p3((size_t)d_ * coarse_tc_k3(d_));
            split3_rows_host(piT.data(), d_, d_, 1, p3.data());
            dPi3_.resize(p3.size());
            h2d(dPi3_.get(), p3.data(), p3.size(), stream_);
            std::vector<float> z((size_t)d_, 0.0f);
            dzero_.resize(z.size());
            h2d(dzero_.get(), z.data(), z.size(), stream_);
        }
    }
    // centroids as the row-major [d][nlist] right operand, plus |c|^2 in double
    // (jhq_gpu_index.cu:243-249)
    const int nl = p_.nlist;
    std::vector<float> cT((size_t)d_ * nl), norms(nl);
    for (int c = 0; c < nl; ++c) {
        double s = 0.0;
        for (int j = 0; j < d_; ++j) {
            float v = cents_[(size_t)c * d_ + j];
            cT[(size_t)j * nl + c] = v;
            s += (double)v * v;
        }
        norms[c] = (float)s;
    }
    dcentsT_.resize(cT.size());
    dnorms_.resize(nl);
    h2d(dcentsT_.get(), cT.data(), cT.size(), stream_);
    h2d(dnorms_.get(), norms.data(), norms.size(), stream_);
    // Row-major copy for the tensor-core path (TMA operand and exact rescoring).
    const char* cm = std::getenv("JHQ_COARSE");
    coarse_tc_ = nl > 1 && coarse_tc_supported(d_, nl) && d_ <= 2048 &&
                 !(cm && std::string(cm) == "simt");
    if (coarse_tc_) {
        dcents_.resize((size_t)nl * d_);
        h2d(dcents_.get(), cents_.data(), (size_t)nl * d_, stream_);
        std::vector<uint16_t> c3((size_t)nl * coarse_tc_k3(d_));
        split3_rows_host(cents_.data(), nl, d_, 1, c3.data());
        dcents3_.resize(c3.size());
        h2d(dcents3_.get(), c3.data(), c3.size(), stream_);
        double mx = 0.0;
        for (int c = 0; c < nl; ++c) mx = std::max(mx, (double)norms[c]);
        cmax_ = (float)(std::sqrt(mx) * 1.0001);
    } else {
        dcents_.release();
        dcents3_.release();
    }
    JHQ_CUDA(cudaStreamSynchronize(stream_));
}

// Lloyd k-means of the rotated rows y [n][d] into nl centroids (host copy in
// `cents`, row-major): init rows floor(c * n / nl), `iters` rounds of
// assign (on the device, through `assign`, which returns the device
// assignment) + mean update in double, an empty cluster reseeded from the
// row LCG(c, iter) (jhq_gpu_index.cu:228-299).
// Lloyd k-means in the rotated space (jhq_gpu_index.cu:228-299): init rows
// floor(c n / nl), `assign` gives the device assignment for the current
// centroids, mean update with index-order double sums, empty lists reseeded from
// row (c * 1103515245 + iter * 12345) % n. The update runs on the device
// (train_gpu.cu, bit-identical); JHQ_TRAIN_HOST=1 runs it on the host instead.
void Index::lloyd(const float* d_y, int64_t n, int nl, int iters, std::vector<float>& cents,
                  const std::function<const int32_t*(const std::vector<float>&)>& assign) {
    cents.assign((size_t)nl * d_, 0.0f);
    DevBuf<float> dc((size_t)nl * d_);
    for (int c = 0; c < nl; ++c) {
        const int64_t src = (int64_t)c * n / nl;
        JHQ_CUDA(cudaMemcpyAsync(dc.get() + (size_t)c * d_, d_y + (size_t)src * d_, 4 * (size_t)d_,
                                 cudaMemcpyDeviceToDevice, stream_));
    }
    d2h(cents.data(), dc.get(), cents.size(), stream_);
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    const char* th = std::getenv("JHQ_TRAIN_HOST");
    if (th && std::string(th) == "1") {                 // host update (train_cpu order)
        std::vector<float> y((size_t)n * d_);
        d2h(y.data(), d_y, y.size(), stream_);
        JHQ_CUDA(cudaStreamSynchronize(stream_));
        std::vector<int32_t> as((size_t)n);
        std::vector<double> sums((size_t)nl * d_);
        std::vector<int> counts(nl);
        for (int iter = 0; iter < iters; ++iter) {
            const int32_t* da = assign(cents);
            d2h(as.data(), da, as.size(), stream_);
            JHQ_CUDA(cudaStreamSynchronize(stream_));
            std::fill(sums.begin(), sums.end(), 0.0);
            std::fill(counts.begin(), counts.end(), 0);
            for (int64_t i = 0; i < n; ++i) {
                const int c = as[i];
                counts[c]++;
                double* sc = &sums[(size_t)c * d_];
                const float* yi = &y[(size_t)i * d_];
                for (int j = 0; j < d_; ++j) sc[j] += yi[j];
            }
            for (int c = 0; c < nl; ++c) {
                float* cc = &cents[(size_t)c * d_];
                if (counts[c] == 0) {
                    const int64_t src = ((int64_t)c * 1103515245 + (int64_t)(iter * 12345)) % n;
                    std::memcpy(cc, &y[(size_t)src * d_], sizeof(float) * d_);
                    continue;
                }
                const double inv = 1.0 / (double)counts[c];
                const double* sc = &sums[(size_t)c * d_];
                for (int j = 0; j < d_; ++j) cc[j] = (float)(sc[j] * inv);
            }
        }
        return;
    }
    std::vector<int64_t> counts;
    for (int iter = 0; iter < iters; ++iter) {
        const int32_t* da = assign(cents);
        lloyd_update_device(d_y, n, d_, nl, da, dc.get(), counts, stream_);
        for (int c = 0; c < nl; ++c)
            if (counts[c] == 0) {
                const int64_t src = ((int64_t)c * 1103515245 + (int64_t)(iter * 12345)) % n;
                JHQ_CUDA(cudaMemcpyAsync(dc.get() + (size_t)c * d_, d_y + (size_t)src * d_,
                                         4 * (size_t)d_, cudaMemcpyDeviceToDevice, stream_));
            }
        d2h(cents.data(), dc.get(), cents.size(), stream_);
        JHQ_CUDA(cudaStreamSynchronize(stream_));
    }
}

// Pilot centroids to the device: transposed [d][P] (assignment GEMM),
// row-major [P][d] (nearest pilot at search) and squared norms.
void Index::upload_pilot(const std::vector<float>& c, int P) {
    std::vector<float> cT((size_t)d_ * P), norms(P);
    for (int k = 0; k < P; ++k) {
        double s2 = 0.0;
        for (int j = 0; j < d_; ++j) {
            const float v = c[(size_t)k * d_ + j];
            cT[(size_t)j * P + k] = v;
            s2 += (double)v * v;
        }
        norms[k] = (float)s2;
    }
    dpilot_centsT_.resize(cT.size());
    dpilot_cents_.resize(c.size());
    h2d(dpilot_cents_.get(), c.data(), c.size(), stream_);
    dpilot_norms_.resize(P);
    h2d(dpilot_centsT_.get(), cT.data(), cT.size(), stream_);
    h2d(dpilot_norms_.get(), norms.data(), norms.size(), stream_);
    JHQ_CUDA(cudaStreamSynchronize(stream_));
}

void Index::set_pilot(const float* cents, int P) {
    DeviceGuard g(dev_);
    if (!trained_ || ntotal_ > 0) fail(JHQ_ESTATE, "set_pilot: needs a trained, empty index");
    if (P < 0 || (P > 0 && !cents)) fail(JHQ_EINVAL, "set_pilot: bad clusters");
    pilot_cents_.assign(cents, cents + (size_t)P * d_);
    pilotP_ = P;
    if (P > 0) upload_pilot(pilot_cents_, P);
}

// ---- train: JHQGpuIndex::train (jhq_gpu_index.cu:333-364) --------------------
void Index::train(const float* h_x, int64_t n) {
    DeviceGuard g(dev_);
    if (!h_x || n <= 0) fail(JHQ_EINVAL, "train: need at least one vector");
    if (n < p_.nlist) fail(JHQ_EINVAL, "n_train must be >= nlist");
    if (n > INT32_MAX / std::max(1, d_)) fail(JHQ_EINVAL, "train: n_train * d exceeds 2^31");
    if (ntotal_ > 0) fail(JHQ_ESTATE, "train() on a non-empty index");

    sigma_ = train::estimate_sigma(h_x, n, d_);
    c1d_ = train::lloyd_max_c1d(sigma_, K1D_);
    Pi_ = train::build_rotation(d_, p_.seed);
    res_c1d_.clear();
    cents_.assign((size_t)p_.nlist * d_, 0.0f);
    upload_trained();

    // rotate + primary-encode the training rows on the device
    DevBuf<float> dx((size_t)std::min<int64_t>(n, p_.add_batch) * d_);
    DevBuf<float> dy((size_t)n * d_);
    DevBuf<uint8_t> dcodes((size_t)n * M_);
    for (int64_t r0 = 0; r0 < n; r0 += p_.add_batch) {
        int64_t nr = std::min<int64_t>(p_.add_batch, n - r0);
        h2d(dx.get(), h_x + r0 * d_, (size_t)nr * d_, stream_);
        rotate_device(dx.get(), nr, dy.get() + r0 * d_, stream_);
    }
    encode_rows(dy.get(), n, d_, M_, B_, Br_, dc1d_.get(), nullptr, false, dcodes.get(), nullptr,
                bpv_pad_, nullptr, stream_);
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    dx.release();

    // IVF centroids: Lloyd k-means in the rotated space (jhq_gpu_index.cu:228-299)
    {
        DevBuf<int32_t> dassign((size_t)n);
        lloyd(dy.get(), n, p_.nlist, p_.ivf_iters, cents_, [&](const std::vector<float>&) {
            upload_trained();
            assign_device(dy.get(), n, dassign.get(), stream_);
            return dassign.get();
        });
    }
    // pilot clusters of a flat index (search-time bound, see pilot.cu)
    pilot_cents_.clear();
    pilotP_ = 0;
    const char* pe = std::getenv("JHQ_PILOT");
    if (p_.nlist == 1 && !(pe && std::string(pe) == "0") && n >= 64 * PILOT_MIN_MEMBERS) {
        const char* pl = std::getenv("JHQ_PILOT_LISTS");
        const int P = std::max(2, std::min<int>(pl ? std::atoi(pl) : PILOT_LISTS,
                                                (int)(n / PILOT_MIN_MEMBERS)));
        DevBuf<int32_t> dassign((size_t)n);
        lloyd(dy.get(), n, P, 6, pilot_cents_, [&](const std::vector<float>& c) {
            upload_pilot(c, P);
            gemm_argmin(dy.get(), dpilot_centsT_.get(), dpilot_norms_.get(), n, d_, P,
                        dassign.get(), stream_);
            return dassign.get();
        });
        pilotP_ = P;
        upload_pilot(pilot_cents_, P);
    }

    // residual codebook: 1-D k-means of y - yhat (jhq_gpu_index.cu:302-330), on
    // the device (train_gpu.cu) or, with JHQ_TRAIN_HOST=1, on the host. Per
    // subspace: one k-means per subspace m over its residuals in (row, dim) order.
    residuals_device(dy.get(), dcodes.get(), n, d_, M_, B_, dc1d_.get(), stream_);
    const char* th = std::getenv("JHQ_TRAIN_HOST");
    const bool host = th && std::string(th) == "1";
    auto fit = [&](const float* dv, int64_t cnt) {
        std::vector<float> c;
        if (host) {
            std::vector<float> r((size_t)cnt);
            d2h(r.data(), dv, r.size(), stream_);
            JHQ_CUDA(cudaStreamSynchronize(stream_));
            c = train::kmeans_1d(r.data(), cnt, Kr_);
        } else {
            c = kmeans_1d_device(dv, cnt, Kr_, 25, stream_);
        }
        c.resize(Kr_, c.empty() ? 0.0f : c.back());
        return c;
    };
    if (!res_per_sub_) {
        res_c1d_ = fit(dy.get(), n * d_);
    } else {
        DevBuf<float> seg((size_t)n * Ds_);
        res_c1d_.clear();
        for (int m = 0; m < M_; ++m) {
            JHQ_CUDA(cudaMemcpy2DAsync(seg.get(), (size_t)Ds_ * 4, dy.get() + (size_t)m * Ds_,
                                       (size_t)d_ * 4, (size_t)Ds_ * 4, (size_t)n,
                                       cudaMemcpyDeviceToDevice, stream_));
            const std::vector<float> c = fit(seg.get(), n * Ds_);
            res_c1d_.insert(res_c1d_.end(), c.begin(), c.end());
        }
    }
    dy.release();
    upload_trained();
    trained_ = true;
    layout_dirty_ = true;
}

void Index::set_trained(const float* Pi, const float* c1d, const float* res_c1d,
                        const float* cents, float sigma) {
    DeviceGuard g(dev_);
    if (ntotal_ > 0) fail(JHQ_ESTATE, "set_trained() on a non-empty index");
    if (!Pi || !c1d || !res_c1d || !cents) fail(JHQ_EINVAL, "set_trained: null artefact");
    pilotP_ = 0;                       // pilot clusters come from train() (or a saved index)
    pilot_cents_.clear();
    Pi_.assign(Pi, Pi + (size_t)d_ * d_);
    c1d_.assign(c1d, c1d + K1D_);
    res_c1d_.assign(res_c1d, res_c1d + residual_floats());
    cents_.assign(cents, cents + (size_t)p_.nlist * d_);
    sigma_ = sigma;
    upload_trained();
    trained_ = true;
    layout_dirty_ = true;
    destroy_graph();
}

void Index::get_trained(float* Pi, float* c1d, float* res_c1d, float* cents, float* sigma) const {
    if (!trained_) fail(JHQ_ESTATE, "index is not trained");
    if (Pi) std::memcpy(Pi, Pi_.data(), Pi_.size() * sizeof(float));
    if (c1d) std::memcpy(c1d, c1d_.data(), c1d_.size() * sizeof(float));
    if (res_c1d) std::memcpy(res_c1d, res_c1d_.data(), res_c1d_.size() * sizeof(float));
    if (cents) std::memcpy(cents, cents_.data(), cents_.size() * sizeof(float));
    if (sigma) *sigma = sigma_;
}

// ---- add: JHQGpuIndex::add (jhq_gpu_index.cu:417-532), repeatable ------------
void Index::grow_master(int64_t need) {
    if (need <= cap_) return;
    if (paging()) {                    // host-resident codes (paging.cu)
        const int64_t nc = std::max<int64_t>(need, cap_ + cap_ / 2);
        hpcodes_.grow((size_t)nc * M_, (size_t)ntotal_ * M_);
        hrcodes_.grow((size_t)nc * bpv_pad_, (size_t)ntotal_ * bpv_pad_);
        hcorr_.grow((size_t)nc, (size_t)ntotal_);
        if (keep_raw_) hraw_.grow((size_t)nc * d_, (size_t)ntotal_ * d_);
        dassign_.resize(1);
        cap_ = nc;
        return;
    }
    int64_t nc = std::max<int64_t>(need, cap_ + cap_ / 2);
    DevBuf<uint8_t> pc((size_t)nc * M_), rc((size_t)nc * bpv_pad_);
    DevBuf<float> co((size_t)nc);
    DevBuf<int32_t> as((size_t)nc);
    DevBuf<float> rw;
    if (keep_raw_) rw.resize((size_t)nc * d_);
    if (ntotal_ > 0) {
        if (keep_raw_)
            JHQ_CUDA(cudaMemcpyAsync(rw.get(), draw_.get(), (size_t)ntotal_ * d_ * 4,
                                     cudaMemcpyDeviceToDevice, stream_));
        JHQ_CUDA(cudaMemcpyAsync(pc.get(), dpcodes_.get(), (size_t)ntotal_ * M_, cudaMemcpyDeviceToDevice, stream_));
        JHQ_CUDA(cudaMemcpyAsync(rc.get(), drcodes_.get(), (size_t)ntotal_ * bpv_pad_, cudaMemcpyDeviceToDevice, stream_));
        JHQ_CUDA(cudaMemcpyAsync(co.get(), dcorr_.get(), (size_t)ntotal_ * 4, cudaMemcpyDeviceToDevice, stream_));
        JHQ_CUDA(cudaMemcpyAsync(as.get(), dassign_.get(), (size_t)ntotal_ * 4, cudaMemcpyDeviceToDevice, stream_));
        JHQ_CUDA(cudaStreamSynchronize(stream_));
    }
    dpcodes_ = std::move(pc);
    drcodes_ = std::move(rc);
    dcorr_ = std::move(co);
    dassign_ = std::move(as);
    if (keep_raw_) draw_ = std::move(rw);
    cap_ = nc;
}

void Index::add(const float* h_x, int64_t n) {
    DeviceGuard g(dev_);
    if (!trained_) fail(JHQ_ESTATE, "call train() before add()");
    if (n < 0 || (n > 0 && !h_x)) fail(JHQ_EINVAL, "add: bad input");
    if (n == 0) return;
    if (ntotal_ + n > INT32_MAX) fail(JHQ_EINVAL, "add: more than 2^31-1 vectors");
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    grow_master(ntotal_ + n);
    const int64_t AB = std::min<int64_t>(p_.add_batch, n);
    DevBuf<float> dx((size_t)AB * d_), dy((size_t)AB * d_);
    DevBuf<int32_t> dpa;
    DevBuf<uint8_t> tp, tr;            // paging: per-batch codes before the host copy
    DevBuf<float> tc;
    DevBuf<int32_t> ta;
    if (pilotP_ > 0) h_pilot_assign_.resize((size_t)(ntotal_ + n));
    for (int64_t r0 = 0; r0 < n; r0 += AB) {
        const int64_t nr = std::min(AB, n - r0);
        const int64_t at = ntotal_ + r0;
        h2d(dx.get(), h_x + r0 * d_, (size_t)nr * d_, stream_);
        if (paging()) {                // encode into batch temporaries, append to host
            if (keep_raw_) std::memcpy(hraw_.get() + at * d_, h_x + r0 * d_, (size_t)nr * d_ * 4);
            rotate_device(dx.get(), nr, dy.get(), stream_);
            tp.ensure((size_t)AB * M_);
            tr.ensure((size_t)AB * bpv_pad_);
            tc.ensure((size_t)AB);
            ta.ensure((size_t)AB);
            assign_device(dy.get(), nr, ta.get(), stream_);
            encode_rows(dy.get(), nr, d_, M_, B_, Br_, dc1d_.get(), dres_.get(), res_per_sub_,
                        tp.get(), tr.get(), bpv_pad_, tc.get(), stream_);
            h_assign_.resize((size_t)(at + nr));
            d2h(h_assign_.data() + at, ta.get(), (size_t)nr, stream_);
            d2h(hpcodes_.get() + at * M_, tp.get(), (size_t)nr * M_, stream_);
            d2h(hrcodes_.get() + at * bpv_pad_, tr.get(), (size_t)nr * bpv_pad_, stream_);
            d2h(hcorr_.get() + at, tc.get(), (size_t)nr, stream_);
            JHQ_CUDA(cudaStreamSynchronize(stream_));
            continue;
        }
        if (keep_raw_)
            JHQ_CUDA(cudaMemcpyAsync(draw_.get() + at * d_, dx.get(), (size_t)nr * d_ * 4,
                                     cudaMemcpyDeviceToDevice, stream_));
        rotate_device(dx.get(), nr, dy.get(), stream_);
        assign_device(dy.get(), nr, dassign_.get() + at, stream_);
        if (pilotP_ > 0) {
            dpa.ensure((size_t)AB);
            gemm_argmin(dy.get(), dpilot_centsT_.get(), dpilot_norms_.get(), nr, d_, pilotP_,
                        dpa.get(), stream_);
            d2h(h_pilot_assign_.data() + at, dpa.get(), (size_t)nr, stream_);
        }
        encode_rows(dy.get(), nr, d_, M_, B_, Br_, dc1d_.get(), dres_.get(), res_per_sub_,
                    dpcodes_.get() + at * M_, drcodes_.get() + at * bpv_pad_, bpv_pad_,
                    dcorr_.get() + at, stream_);
    }
    if (!paging()) {
        h_assign_.resize((size_t)(ntotal_ + n));
        d2h(h_assign_.data() + ntotal_, dassign_.get() + ntotal_, (size_t)n, stream_);
    }
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    ntotal_ += n;
    rebuild_layout();
}

// Group vectors by list (stable in id order), pad lists to 32-vector pages and
// scatter the primary codes into the page layout. Replaces thrust::sort_by_key
// + gather_list_storage_kernel + transpose_uint8_kernel (jhq_gpu_index.cu:468-522).
void Index::rebuild_layout() {
    const int nl = p_.nlist;
    std::vector<int64_t> cnt(nl, 0);
    for (int64_t i = 0; i < ntotal_; ++i) {
        int a = h_assign_[(size_t)i];
        if (a < 0 || a >= nl) fail(JHQ_EDEVICE, "invalid IVF assignment");
        cnt[a]++;
    }
    std::vector<int32_t> lpo(nl + 1, 0);
    int64_t pages = 0;
    for (int c = 0; c < nl; ++c) {
        lpo[c] = (int32_t)pages;
        pages += ceil_div(cnt[c], 32);
        if (pages > INT32_MAX) fail(JHQ_EINVAL, "too many pages");
    }
    lpo[nl] = (int32_t)pages;
    std::vector<int32_t> slots((size_t)pages * 32, -1);
    std::vector<int64_t> cur(nl);
    for (int c = 0; c < nl; ++c) cur[c] = (int64_t)lpo[c] * 32;
    for (int64_t i = 0; i < ntotal_; ++i) slots[(size_t)cur[h_assign_[(size_t)i]]++] = (int32_t)i;
    npages_ = pages;
    h_list_pages_sorted_.resize(nl);
    for (int c = 0; c < nl; ++c) h_list_pages_sorted_[c] = lpo[c + 1] - lpo[c];
    std::sort(h_list_pages_sorted_.begin(), h_list_pages_sorted_.end(), std::greater<int32_t>());
    if (paging()) {                    // pages and slot ids built in host memory
        build_host_pages(lpo, slots);
        layout_dirty_ = false;
        destroy_graph();
        return;
    }
    dlist_page_off_.resize(nl + 1);
    dslot_ids_.resize(std::max<size_t>(1, slots.size()));
    dpages_.resize(std::max<size_t>(16, (size_t)pages * Mp_ * 32));
    h2d(dlist_page_off_.get(), lpo.data(), lpo.size(), stream_);
    h2d(dslot_ids_.get(), slots.data(), slots.size(), stream_);
    scatter_pages(dslot_ids_.get(), (int64_t)slots.size(), dpcodes_.get(), M_, Mp_, dpages_.get(),
                  stream_);
    if (p_.nlist == 1 && bpd_ == 1) {  // bit counts for the tensor-core flat scan
        dpop_.resize((size_t)std::max<int64_t>(1, ntotal_));
        popcount_rows(dpcodes_.get(), ntotal_, M_, dpop_.get(), stream_);
    }
    if (pilotP_ > 0) {                 // pilot members, grouped by cluster in id order
        std::vector<int32_t> off(pilotP_ + 1, 0), ids((size_t)std::max<int64_t>(1, ntotal_));
        for (int64_t i = 0; i < ntotal_; ++i) off[h_pilot_assign_[(size_t)i] + 1]++;
        for (int c = 0; c < pilotP_; ++c) off[c + 1] += off[c];
        std::vector<int32_t> pos(off.begin(), off.end() - 1);
        for (int64_t i = 0; i < ntotal_; ++i) ids[(size_t)pos[h_pilot_assign_[(size_t)i]]++] = (int32_t)i;
        dpilot_off_.resize(off.size());
        dpilot_ids_.resize(ids.size());
        h2d(dpilot_off_.get(), off.data(), off.size(), stream_);
        h2d(dpilot_ids_.get(), ids.data(), ids.size(), stream_);
    }
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    layout_dirty_ = false;
    destroy_graph();          // captured pointers changed
}

// ---- search: search_gpu (search.cu:388-445) ----------------------------------
void Index::check_search_args(int64_t nq, int k) const {
    if (nq < 0) fail(JHQ_EINVAL, "nq must be >= 0");
    if (k <= 0) fail(JHQ_EINVAL, "k must be positive");
    if (!trained_ || ntotal_ == 0) fail(JHQ_ESTATE, "index is empty");
    const int kj = stage_k(k);
    int ck = std::max(kj, (int)std::ceil(p_.alpha * (float)kj));
    if (next_pow2(ck) > MAX_CK_PAD)
        fail(JHQ_EINVAL, rerank_ > 0 ? "max(R, ceil(alpha*R)) must be <= 256 (R = rerank depth)"
                                     : "max(k, ceil(alpha*k)) must be <= 256");
    if (scan_smem_bytes(Mp_, d_, std::max(32, next_pow2(ck)), scan_mode_for(d_, M_, B_, 1.0)) > 227 * 1024)
        fail(JHQ_EINVAL, "max(k, ceil(alpha*k)) too large for this M: the LUT and the top-ck "
                         "lists must fit in shared memory together");
}

Index::BatchShape Index::batch_shape(int Bq, int k) const {
    BatchShape sh;
    sh.Bq = Bq;
    sh.k = k;
    sh.kr = stage_k(k);
    sh.ck = std::max(sh.kr, (int)std::ceil(p_.alpha * (float)sh.kr));
    sh.ck_pad = std::max(32, next_pow2(sh.ck));
    // queries per list decide the query-group size; shrink it while the tables
    // and top-ck lists do not fit in shared memory
    const double qpl = (double)Bq * p_.nprobe / p_.nlist;
    sh.mode = scan_mode_for(d_, M_, B_, qpl);
    // tuning override: JHQ_SCAN_MODE=1|2|4 forces the query-group width
    if (const char* e = std::getenv("JHQ_SCAN_MODE"))
        if (sh.mode != 0 && (!std::strcmp(e, "1") || !std::strcmp(e, "2") || !std::strcmp(e, "4")))
            sh.mode = std::atoi(e);
    while (sh.mode > 1 && scan_smem_bytes(Mp_, d_, sh.ck_pad, sh.mode) > 227 * 1024) sh.mode /= 2;
    sh.grid = scan_grid_for(Mp_, d_, sh.ck_pad, sh.mode);
    // chunk size: about four units per CTA for the expected page visits
    const int qg = sh.mode == 0 ? 1 : sh.mode;
    const double avg_pages = (double)npages_ / p_.nlist;
    const double visits = std::max(1.0, (double)Bq * p_.nprobe * avg_pages / qg);
    sh.chunk_pages = (int)std::min(256.0, std::max(16.0, visits / (4.0 * sh.grid)));
    int64_t top_pages = 0;
    for (int i = 0; i < p_.nprobe && i < (int)h_list_pages_sorted_.size(); ++i)
        top_pages += h_list_pages_sorted_[i];
    // IVF with small per-query tables (Mp <= 64): query-major warp items. On
    // C3 (M=32, nlist 65,536) they beat list-major units for small lists
    // (12.5M-vector shard: 2.1 vs 38 ms per 10k queries at 4M rows) and large
    // ones (100M rows, 48 pages per list: 39.5 vs 78.4 ms).
    sh.qmajor = 0;
    if (p_.nlist > 1 && sh.mode == 1 && Mp_ <= 64 &&
        scan_qmajor_smem_bytes(Mp_, sh.ck_pad) <= 227 * 1024)
        sh.qmajor = 1;
    if (const char* e = std::getenv("JHQ_SCAN_ORDER")) {     // tuning / test override
        if (!std::strcmp(e, "list")) sh.qmajor = 0;
        if (!std::strcmp(e, "query") && sh.mode == 1 && Mp_ <= 128 &&
            scan_qmajor_smem_bytes(Mp_, sh.ck_pad) <= 227 * 1024)
            sh.qmajor = 1;
    }
    if (sh.qmajor) {
        sh.grid = scan_qmajor_grid_for(Mp_, sh.ck_pad);
        const double pages = std::max(1.0, (double)Bq * p_.nprobe * avg_pages);
        sh.chunk_pages = (int)std::min(256.0, std::max(16.0, pages / (8.0 * sh.grid * 8)));
        sh.max_slots = (int64_t)Bq * (1 + ceil_div(top_pages, sh.chunk_pages));
        return sh;
    }
    // slots: per query, one per chunk of each probed list; bounded by nprobe
    // plus the chunks of the nprobe largest lists
    sh.max_slots = (int64_t)Bq * (p_.nprobe + ceil_div(top_pages, sh.chunk_pages));
    return sh;
}

void Index::prepare_workspace(int k) {
    const int Bq = p_.batch_size;
    if (ws_.batch_cap == Bq && ws_.k == k && (ws_.exec || paging()) &&
        ws_.coarse_floats == coarse_scratch_floats(Bq))
        return;
    destroy_graph();
    scan_configure();
    refine_configure();
    const BatchShape sh = batch_shape(Bq, k);
    const int nl = p_.nlist, np = p_.nprobe;
    ws_.q.ensure((size_t)Bq * d_);
    ws_.q_rot.ensure((size_t)Bq * d_);
    ws_.rotq.ensure(std::max<size_t>(1, rotq_scratch_floats(Bq)));
    ws_.coarse_floats = coarse_scratch_floats(Bq);
    if (nl > 1) ws_.scores.ensure(ws_.coarse_floats);
    ws_.probes.ensure((size_t)Bq * np);
    ws_.cnt.ensure((size_t)nl + 1);
    ws_.bucket_off.ensure((size_t)nl + 1);
    ws_.unit_off.ensure((size_t)nl + 1);
    ws_.fill.ensure((size_t)nl);
    ws_.bucket.ensure((size_t)Bq * np);
    ws_.cpo.ensure((size_t)Bq * (np + 1));
    ws_.qslot_off.ensure((size_t)Bq + 1);
    ws_.gthr.ensure((size_t)Bq);
    ws_.cand.ensure((size_t)sh.max_slots * sh.ck);
    if (flat_tc()) ws_.flat.ensure(flat_tc_scratch_bytes(Bq, d_, (int)ntotal_));
    ws_.ivf_tiles = 0;
    if (ivf_tc()) {
        // per query at most nprobe partial tiles plus the tiles of the nprobe largest lists
        int64_t top_pages = 0;
        for (int i = 0; i < np && i < (int)h_list_pages_sorted_.size(); ++i)
            top_pages += h_list_pages_sorted_[i];
        ws_.ivf_tiles = (int64_t)Bq * (np + ceil_div(top_pages, 4));
        ws_.ivf.ensure(ivf_tc_scratch_bytes(Bq, ws_.ivf_tiles));
    }
    if (pilotP_ > 0) {
        ws_.pkeys.ensure((size_t)Bq * PILOT_SPLIT * sh.ck);
        ws_.pscores.ensure((size_t)Bq * pilotP_);
    }
    ws_.out_d.ensure((size_t)Bq * k);
    ws_.out_i.ensure((size_t)Bq * k);
    ws_.nvalid.ensure(1);
    ws_.h_q.ensure((size_t)2 * Bq * d_);
    ws_.h_d.ensure((size_t)2 * Bq * k);
    ws_.h_i.ensure((size_t)2 * Bq * k);
    if (nl == 1) JHQ_CUDA(cudaMemsetAsync(ws_.probes.get(), 0, (size_t)Bq * np * 4, stream_));
    ws_.batch_cap = Bq;
    ws_.k = k;
    ws_.ck = sh.ck;
    ws_.ck_pad = sh.ck_pad;
    ws_.grid = sh.grid;
    ws_.mode = sh.mode;
    ws_.chunk_pages = sh.chunk_pages;
    ws_.max_slots = sh.max_slots;
    ws_.qmajor = sh.qmajor;
    if (paging()) {                    // paged batches are host-orchestrated (paging.cu)
        JHQ_CUDA(cudaStreamSynchronize(stream_));
        return;
    }
    // capture the per-batch pipeline once (capture_graph, search.cu:315-386)
    const int64_t before = g_kernel_launches.load();
    JHQ_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
        enqueue_batch(stream_);
    } catch (...) {
        cudaGraph_t gph = nullptr;
        cudaStreamEndCapture(stream_, &gph);
        if (gph) cudaGraphDestroy(gph);
        throw;
    }
    JHQ_CUDA(cudaStreamEndCapture(stream_, &ws_.graph));
    JHQ_CUDA(cudaGraphInstantiate(&ws_.exec, ws_.graph, 0));
    ws_.graph_kernels = g_kernel_launches.load() - before;
    g_kernel_launches.fetch_sub(ws_.graph_kernels);     // counted when launched instead
    JHQ_CUDA(cudaStreamSynchronize(stream_));
}

size_t Index::coarse_scratch_floats(int Bq) const {
    if (p_.nlist <= 1) return 0;
    const size_t sc = ((size_t)Bq * p_.nlist + 63) & ~(size_t)63;   // split rows 256-byte aligned
    // then the bf16 split queries (Bq x K3, rounded to 64 floats), then tile minima
    const size_t q3f = (((size_t)Bq * coarse_tc_k3(d_) + 1) / 2 + 63) & ~(size_t)63;
    return sc + (coarse_tc_ ? q3f + (size_t)Bq * coarse_tc_tiles(p_.nlist) : 0);
}

void Index::coarse_probes(const float* q_rot, int nq, int Bq, int nprobe, float* scores,
                          int32_t* probes, cudaStream_t s) {
    if (coarse_tc_) {
        float* q3f = scores + (((size_t)Bq * p_.nlist + 63) & ~(size_t)63);
        uint16_t* q3 = reinterpret_cast<uint16_t*>(q3f);
        float* tmin = q3f + ((((size_t)Bq * coarse_tc_k3(d_) + 1) / 2 + 63) & ~(size_t)63);
        const int nt = coarse_tc_tiles(p_.nlist);
        split3_rows(q_rot, nq, d_, q3, s);
        coarse_scores_tc(q3, nq, dcents3_.get(), dnorms_.get(), p_.nlist, d_, scores, tmin, s);
        select_probes_margin(scores, q_rot, dcents_.get(), dnorms_.get(), tmin, nt, nq, p_.nlist,
                             d_, nprobe, cmax_, probes, s);
    } else {
        gemm_rows(q_rot, dcentsT_.get(), scores, nq, d_, p_.nlist, EPI_COARSE, dnorms_.get(), s);
        select_probes(scores, nq, p_.nlist, nprobe, probes, s);
    }
}

// Kernel sequence of one query batch: rotate -> coarse scores + probes ->
// plan -> scan -> refine, with optional events between the stages.
void Index::enqueue_pipeline(const float* q_in, int nq, const int* d_nvalid,
                             const BatchShape& sh, const BatchBufs& b, float* out_d,
                             int32_t* out_i, cudaStream_t s, cudaEvent_t* ev,
                             const int32_t* probes_in) {
    auto mark = [&](int i) { if (ev) JHQ_CUDA(cudaEventRecord(ev[i], s)); };
    mark(0);
    rotate_queries_device(q_in, nq, b.q_rot, b.rotq, s);
    mark(1);
    const int32_t* probes = probes_in ? probes_in : b.probes;
    if (p_.nlist > 1 && !probes_in) {
        coarse_probes(b.q_rot, nq, sh.Bq, p_.nprobe, b.scores, b.probes, s);
    }
    mark(2);
    // the refine of a scan that leaves one candidate slot per query
    auto refine_single = [&]() {
        RefineArgs ra;
        ra.q_rot = b.q_rot; ra.res_c1d = dres_.get(); ra.cand = b.cand;
        ra.res_per_sub = res_per_sub_ ? 1 : 0; ra.M = M_;
        ra.qslot_off = b.plan.qslot_off; ra.gthr = b.plan.gthr; ra.rcodes = drcodes_.get();
        ra.corr = dcorr_.get(); ra.out_dists = out_d; ra.out_ids = out_i;
        ra.nq = nq; ra.d = d_; ra.Br = Br_; ra.bpv_pad = bpv_pad_; ra.ck = sh.ck;
        ra.ck_pad = sh.ck_pad; ra.k = sh.k; ra.kr = sh.kr;
        if (keep_raw_ && rerank_ > 0) {
            ra.q_raw = q_in;
            ra.raw = draw_.get();
        }
        refine_topk(ra, s);
    };
    if (p_.nlist == 1 && b.flat && !probes_in) {     // flat, 1-bit codes: tensor-core ADC
        FlatTcArgs fa;
        fa.q_rot = b.q_rot; fa.c1d = dc1d_.get(); fa.c1d_host = c1d_.data();
        fa.codes = dpcodes_.get(); fa.pop = dpop_.get();
        fa.nvec = (int)ntotal_; fa.M = M_; fa.nq = nq; fa.ck = sh.ck; fa.ck_pad = sh.ck_pad;
        fa.scratch = b.flat; fa.cand = b.cand; fa.gthr = b.plan.gthr;
        fa.qslot_off = b.plan.qslot_off; fa.d_nvalid = d_nvalid;
        mark(3);                       // no plan: the "scan" stage is the GEMM + selection
        flat_search_tc(fa, s);
        mark(4);
        refine_single();
        mark(5);
        return;
    }
    if (p_.nlist > 1 && b.ivf) {      // IVF, 2 bits per dimension: two-pass tensor-core scan
        IvfTcArgs ia;
        ia.q_rot = b.q_rot; ia.c1d = dc1d_.get(); ia.c1d_host = c1d_.data();
        ia.probes = probes; ia.list_page_off = dlist_page_off_.get();
        ia.pages = dpages_.get(); ia.slot_ids = dslot_ids_.get();
        ia.plan = b.plan; ia.scratch = b.ivf; ia.max_tiles = b.ivf_tiles;
        ia.nq = nq; ia.nprobe = p_.nprobe; ia.nlist = p_.nlist; ia.d = d_; ia.M = M_;
        ia.ck = sh.ck; ia.ck_pad = sh.ck_pad;
        ia.cand = b.cand; ia.gthr = b.plan.gthr; ia.qslot_out = b.plan.qslot_off;
        ia.d_nvalid = d_nvalid;
        mark(3);                       // the plan is built inside: the "scan" stage is all of it
        ivf_search_tc(ia, s);
        mark(4);
        refine_single();
        mark(5);
        return;
    }
    const int qg = sh.mode == 0 ? 1 : sh.mode;
    if (sh.qmajor)
        plan_build_qmajor(probes, nq, p_.nprobe, dlist_page_off_.get(), d_nvalid,
                          sh.chunk_pages, b.plan, s);
    else
        plan_build(probes, nq, p_.nprobe, p_.nlist, dlist_page_off_.get(), d_nvalid,
                   sh.chunk_pages, qg, b.plan, s);
    ScanArgs sa;
    sa.q_rot = b.q_rot; sa.c1d = dc1d_.get(); sa.list_page_off = dlist_page_off_.get();
    sa.pages = dpages_.get(); sa.slot_ids = dslot_ids_.get();
    sa.unit_off = b.plan.unit_off; sa.bucket_off = b.plan.bucket_off; sa.bucket = b.plan.bucket;
    sa.cpo = b.plan.cpo; sa.qslot_off = b.plan.qslot_off; sa.gthr = b.plan.gthr; sa.cand = b.cand;
    sa.nq = nq; sa.nlist = p_.nlist; sa.d = d_; sa.M = M_; sa.Mp = Mp_; sa.B = B_;
    sa.nprobe = p_.nprobe; sa.ck = sh.ck; sa.ck_pad = sh.ck_pad; sa.grid = sh.grid;
    sa.chunk_pages = sh.chunk_pages; sa.mode = sh.mode; sa.qmajor = sh.qmajor;
    sa.probes = probes;
    if (pilotP_ > 0 && p_.nlist == 1 && sh.mode == 1 && !sh.qmajor && ntotal_ > 0 && b.pkeys) {
        PilotArgs pa;
        pa.q_rot = b.q_rot; pa.c1d = dc1d_.get(); pa.pcents = dpilot_cents_.get();
        pa.pnorms = dpilot_norms_.get(); pa.pilot_off = dpilot_off_.get();
        pa.pilot_ids = dpilot_ids_.get(); pa.pcodes = dpcodes_.get(); pa.gthr = b.plan.gthr;
        pa.pkeys = b.pkeys; pa.pscores = b.pscores;
        pa.d_nvalid = d_nvalid; pa.nq = nq; pa.d = d_; pa.M = M_; pa.B = B_; pa.P = pilotP_;
        pa.ck = sh.ck;
        pilot_bound(pa, s);
        sa.prune = 1;
    }
    mark(3);
    scan_topck(sa, s);
    mark(4);
    RefineArgs ra;
    ra.q_rot = b.q_rot; ra.res_c1d = dres_.get(); ra.cand = b.cand;
    ra.res_per_sub = res_per_sub_ ? 1 : 0; ra.M = M_;
    ra.qslot_off = b.plan.qslot_off; ra.gthr = b.plan.gthr; ra.rcodes = drcodes_.get();
    ra.corr = dcorr_.get(); ra.out_dists = out_d; ra.out_ids = out_i;
    ra.nq = nq; ra.d = d_; ra.Br = Br_; ra.bpv_pad = bpv_pad_; ra.ck = sh.ck;
    ra.ck_pad = sh.ck_pad; ra.k = sh.k; ra.kr = sh.kr;
    if (keep_raw_ && rerank_ > 0) {
        ra.q_raw = q_in;
        ra.raw = draw_.get();
    }
    refine_topk(ra, s);
    mark(5);
}

void Index::enqueue_batch(cudaStream_t s, cudaEvent_t* ev) {
    BatchShape sh;
    sh.Bq = ws_.batch_cap; sh.k = ws_.k; sh.kr = stage_k(ws_.k); sh.ck = ws_.ck;
    sh.ck_pad = ws_.ck_pad;
    sh.grid = ws_.grid; sh.mode = ws_.mode; sh.chunk_pages = ws_.chunk_pages;
    sh.max_slots = ws_.max_slots;
    sh.qmajor = ws_.qmajor;
    BatchBufs b;
    b.q_rot = ws_.q_rot.get(); b.scores = ws_.scores.get(); b.probes = ws_.probes.get();
    b.rotq = ws_.rotq.get();
    b.flat = flat_tc() ? ws_.flat.get() : nullptr;
    b.ivf = ws_.ivf_tiles > 0 ? ws_.ivf.get() : nullptr;
    b.ivf_tiles = ws_.ivf_tiles;
    b.plan = PlanBufs{ws_.cnt.get(), ws_.bucket_off.get(), ws_.unit_off.get(), ws_.fill.get(),
                      ws_.bucket.get(), ws_.cpo.get(), ws_.qslot_off.get(), ws_.gthr.get()};
    b.cand = ws_.cand.get();
    b.pkeys = ws_.pkeys.get(); b.pscores = ws_.pscores.get();
    enqueue_pipeline(ws_.q.get(), ws_.batch_cap, ws_.nvalid.get(), sh, b, ws_.out_d.get(),
                     ws_.out_i.get(), s, ev);
}

void Index::run_batch(cudaStream_t s, int nvalid) {
    set_int(ws_.nvalid.get(), nvalid, s);
    if (!profiling_) {
        JHQ_CUDA(cudaGraphLaunch(ws_.exec, s));
        count_launch((int)ws_.graph_kernels);
        return;
    }
    // profiled batch: direct launches with events between the stages
    for (auto& e : prof_ev_)
        if (!e) JHQ_CUDA(cudaEventCreate(&e));
    enqueue_batch(s, prof_ev_);
    JHQ_CUDA(cudaEventSynchronize(prof_ev_[5]));
    for (int i = 0; i < 5; ++i) {
        float ms = 0.0f;
        JHQ_CUDA(cudaEventElapsedTime(&ms, prof_ev_[i], prof_ev_[i + 1]));
        stage_ms_[i] += ms;
    }
    ++stage_batches_;
}

void Index::set_residual_codebooks(bool per_subspace) {
    if (per_subspace == res_per_sub_) return;
    if (trained_) fail(JHQ_ESTATE, "residual codebooks: choose them before train()/set_trained()");
    if (per_subspace && (size_t)M_ * Kr_ > 16384)
        fail(JHQ_EINVAL, "per-subspace residual codebooks: M * 2^Br must be <= 16384");
    res_per_sub_ = per_subspace;
}

void Index::set_rerank(int R) {
    if (R < 0 || R > MAX_CK_PAD) fail(JHQ_EINVAL, "rerank: R must be in [0, 256]");
    if (R > 0 && !keep_raw_) {
        if (ntotal_ > 0)
            fail(JHQ_ESTATE, "rerank: enable it before the first add() (the vectors are kept "
                             "from then on)");
        if (d_ % 4 != 0) fail(JHQ_EINVAL, "rerank: d must be a multiple of 4");
        keep_raw_ = true;
        if (cap_ > 0) draw_.resize((size_t)cap_ * d_);
    }
    if (R != rerank_) {
        DeviceGuard g(dev_);
        JHQ_CUDA(cudaStreamSynchronize(stream_));
        rerank_ = R;
        destroy_graph();
        ws_.batch_cap = 0;             // workspace and graph are rebuilt
    }
}

void Index::set_profiling(bool on) {
    profiling_ = on;
    for (double& v : stage_ms_) v = 0.0;
    stage_batches_ = 0;
}

void Index::stage_times(double* ms, int64_t* batches, int n) const {
    for (int i = 0; i < n && i < 5; ++i) {
        if (ms) ms[i] = stage_ms_[i];
    }
    if (batches) *batches = stage_batches_;
}

void Index::search(const float* h_q, int64_t nq, int k, float* h_dists, int32_t* h_ids) {
    DeviceGuard g(dev_);
    check_search_args(nq, k);
    if (nq == 0) return;
    if (!h_q || !h_dists || !h_ids) fail(JHQ_EINVAL, "search: null buffer");
    prepare_workspace(k);
    const int Bq = ws_.batch_cap;
    const int64_t nb = ceil_div(nq, Bq);
    cudaEvent_t ev[2];
    JHQ_CUDA(cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming));
    JHQ_CUDA(cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming));
    int64_t pending[2] = {-1, -1};
    auto drain = [&](int slot) {
        if (pending[slot] < 0) return;
        JHQ_CUDA(cudaEventSynchronize(ev[slot]));
        const int64_t b = pending[slot];
        const int64_t q0 = b * Bq, nv = std::min<int64_t>(Bq, nq - q0);
        std::memcpy(h_dists + q0 * k, ws_.h_d.get() + (size_t)slot * Bq * k, (size_t)nv * k * 4);
        std::memcpy(h_ids + q0 * k, ws_.h_i.get() + (size_t)slot * Bq * k, (size_t)nv * k * 4);
        pending[slot] = -1;
    };
    try {
        for (int64_t b = 0; b < nb; ++b) {
            const int slot = (int)(b & 1);
            drain(slot);
            const int64_t q0 = b * Bq, nv = std::min<int64_t>(Bq, nq - q0);
            float* hq = ws_.h_q.get() + (size_t)slot * Bq * d_;
            std::memcpy(hq, h_q + q0 * d_, (size_t)nv * d_ * 4);
            if (nv < Bq) std::memset(hq + nv * d_, 0, (size_t)(Bq - nv) * d_ * 4);
            h2d(ws_.q.get(), hq, (size_t)Bq * d_, stream_);
            if (paging()) run_paged_batch(ws_.q.get(), (int)nv, ws_.out_d.get(), ws_.out_i.get(), stream_);
            else run_batch(stream_, (int)nv);
            d2h(ws_.h_d.get() + (size_t)slot * Bq * k, ws_.out_d.get(), (size_t)Bq * k, stream_);
            d2h(ws_.h_i.get() + (size_t)slot * Bq * k, ws_.out_i.get(), (size_t)Bq * k, stream_);
            JHQ_CUDA(cudaEventRecord(ev[slot], stream_));
            pending[slot] = b;
        }
        drain((int)(nb & 1));
        drain((int)((nb + 1) & 1));
    } catch (...) {
        cudaStreamSynchronize(stream_);
        cudaEventDestroy(ev[0]);
        cudaEventDestroy(ev[1]);
        throw;
    }
    cudaEventDestroy(ev[0]);
    cudaEventDestroy(ev[1]);
    if ((coarse_tc_ || rot_tc_) && coarse_tc_error(true))
        fail(JHQ_ETIMEDOUT, "search: a tensor-core coarse wait gave up");
}

void Index::search_device(const float* d_q, int64_t nq, int k, float* d_dists, int32_t* d_ids,
                          cudaStream_t stream) {
    DeviceGuard g(dev_);
    check_search_args(nq, k);
    if (nq == 0) return;
    if (!d_q || !d_dists || !d_ids) fail(JHQ_EINVAL, "search_device: null buffer");
    prepare_workspace(k);
    cudaStream_t s = stream ? stream : stream_;
    const int Bq = ws_.batch_cap;
    for (int64_t q0 = 0; q0 < nq; q0 += Bq) {
        const int64_t nv = std::min<int64_t>(Bq, nq - q0);
        JHQ_CUDA(cudaMemcpyAsync(ws_.q.get(), d_q + q0 * d_, (size_t)nv * d_ * 4,
                                 cudaMemcpyDeviceToDevice, s));
        if (paging()) run_paged_batch(ws_.q.get(), (int)nv, ws_.out_d.get(), ws_.out_i.get(), s);
        else run_batch(s, (int)nv);
        JHQ_CUDA(cudaMemcpyAsync(d_dists + q0 * k, ws_.out_d.get(), (size_t)nv * k * 4,
                                 cudaMemcpyDeviceToDevice, s));
        JHQ_CUDA(cudaMemcpyAsync(d_ids + q0 * k, ws_.out_i.get(), (size_t)nv * k * 4,
                                 cudaMemcpyDeviceToDevice, s));
    }
}

void Index::probe_device(const float* d_q, int64_t nq, int32_t* d_probes, cudaStream_t stream) {
    DeviceGuard g(dev_);
    check_search_args(nq, ws_.k ? ws_.k : 10);
    if (nq == 0) return;
    if (!d_q || !d_probes) fail(JHQ_EINVAL, "probe_device: null buffer");
    if (paging()) fail(JHQ_ESTATE, "probe_device: not available with list paging");
    prepare_workspace(ws_.k ? ws_.k : 10);
    cudaStream_t s = stream ? stream : stream_;
    const int Bq = ws_.batch_cap, np = p_.nprobe;
    for (int64_t q0 = 0; q0 < nq; q0 += Bq) {
        const int nv = (int)std::min<int64_t>(Bq, nq - q0);
        rotate_queries_device(d_q + q0 * d_, nv, ws_.q_rot.get(), ws_.rotq.get(), s);
        if (p_.nlist > 1) {
            coarse_probes(ws_.q_rot.get(), nv, Bq, np, ws_.scores.get(), d_probes + q0 * np, s);
        } else {
            JHQ_CUDA(cudaMemsetAsync(d_probes + q0 * np, 0, (size_t)nv * np * 4, s));
        }
    }
}

void Index::search_device_probes(const float* d_q, const int32_t* d_probes, int64_t nq, int k,
                                 float* d_dists, int32_t* d_ids, cudaStream_t stream) {
    DeviceGuard g(dev_);
    check_search_args(nq, k);
    if (nq == 0) return;
    if (!d_q || !d_probes || !d_dists || !d_ids) fail(JHQ_EINVAL, "search_device_probes: null buffer");
    if (paging()) fail(JHQ_ESTATE, "search_device_probes: not available with list paging");
    prepare_workspace(k);
    cudaStream_t s = stream ? stream : stream_;
    BatchShape sh;
    sh.Bq = ws_.batch_cap; sh.k = ws_.k; sh.kr = stage_k(ws_.k); sh.ck = ws_.ck;
    sh.ck_pad = ws_.ck_pad;
    sh.grid = ws_.grid; sh.mode = ws_.mode; sh.chunk_pages = ws_.chunk_pages;
    sh.max_slots = ws_.max_slots; sh.qmajor = ws_.qmajor;
    BatchBufs b;
    b.q_rot = ws_.q_rot.get(); b.scores = ws_.scores.get(); b.probes = ws_.probes.get();
    b.rotq = ws_.rotq.get();
    b.flat = flat_tc() ? ws_.flat.get() : nullptr;
    b.ivf = ws_.ivf_tiles > 0 ? ws_.ivf.get() : nullptr;
    b.ivf_tiles = ws_.ivf_tiles;
    b.plan = PlanBufs{ws_.cnt.get(), ws_.bucket_off.get(), ws_.unit_off.get(), ws_.fill.get(),
                      ws_.bucket.get(), ws_.cpo.get(), ws_.qslot_off.get(), ws_.gthr.get()};
    b.cand = ws_.cand.get();
    b.pkeys = ws_.pkeys.get(); b.pscores = ws_.pscores.get();
    const int Bq = ws_.batch_cap;
    for (int64_t q0 = 0; q0 < nq; q0 += Bq) {
        const int nv = (int)std::min<int64_t>(Bq, nq - q0);
        enqueue_pipeline(d_q + q0 * d_, nv, nullptr, sh, b, d_dists + q0 * k, d_ids + q0 * k, s,
                         nullptr, d_probes + q0 * p_.nprobe);
    }
}

void Index::set_nprobe(int nprobe) {
    DeviceGuard g(dev_);
    if (nprobe <= 0) fail(JHQ_EINVAL, "nprobe must be positive");
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    p_.nprobe = std::min(nprobe, p_.nlist);
    destroy_graph();
    ws_.batch_cap = 0;                         // workspace and graph are rebuilt
}

void Index::list_sizes(int64_t* sizes) const {
    std::fill(sizes, sizes + p_.nlist, (int64_t)0);
    for (int64_t i = 0; i < ntotal_; ++i) sizes[h_assign_[(size_t)i]]++;
}

void Index::set_alpha(float alpha) {
    DeviceGuard g(dev_);
    if (!(alpha > 0.0f)) fail(JHQ_EINVAL, "alpha must be positive");
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    p_.alpha = alpha;
    destroy_graph();
    ws_.batch_cap = 0;
}

bool Index::flat_tc_scores(const float* h_q, int nq, float* h_scores) {
    DeviceGuard g(dev_);
    if (!flat_tc() || nq <= 0 || nq > 128) return false;
    DevBuf<float> dq((size_t)nq * d_), dr((size_t)nq * d_);
    DevBuf<float> sc(std::max<size_t>(1, rotq_scratch_floats(nq)));
    DevBuf<unsigned char> fl(flat_tc_scratch_bytes(nq, d_, (int)ntotal_));
    DevBuf<uint64_t> cand((size_t)nq * 256), gth((size_t)nq);
    DevBuf<int64_t> qs((size_t)nq + 1);
    h2d(dq.get(), h_q, (size_t)nq * d_, stream_);
    rotate_queries_device(dq.get(), nq, dr.get(), sc.get(), stream_);
    FlatTcArgs fa;
    fa.q_rot = dr.get(); fa.c1d = dc1d_.get(); fa.c1d_host = c1d_.data();
    fa.codes = dpcodes_.get(); fa.pop = dpop_.get();
    fa.nvec = (int)ntotal_; fa.M = M_; fa.nq = nq; fa.ck = 10; fa.ck_pad = 32;
    fa.scratch = fl.get(); fa.cand = cand.get(); fa.gthr = gth.get(); fa.qslot_off = qs.get();
    fa.scores_only = true;
    flat_search_tc(fa, stream_);
    d2h(h_scores, flat_tc_scores_of(fl.get(), nq, d_, (int)ntotal_), (size_t)nq * ntotal_, stream_);
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    return true;
}

void Index::check_device_status() {
    DeviceGuard g(dev_);
    if ((coarse_tc_ || rot_tc_) && coarse_tc_error(true))
        fail(JHQ_ETIMEDOUT, "a tensor-core coarse wait gave up: the probe lists of that search "
                            "are not valid");
}

void Index::synchronize(double timeout_s) {
    DeviceGuard g(dev_);
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t e = cudaStreamQuery(stream_);
        if (e == cudaSuccess) {
            if ((coarse_tc_ || rot_tc_) && coarse_tc_error(true))
                fail(JHQ_ETIMEDOUT, "synchronize: a tensor-core coarse wait gave up");
            return;
        }
        if (e != cudaErrorNotReady) JHQ_CUDA(e);
        double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > timeout_s) fail(JHQ_ETIMEDOUT, "synchronize: stream still busy at the deadline");
        std::this_thread::yield();
    }
}

// ---- inspection ---------------------------------------------------------------
void Index::get_codes(uint8_t* primary, uint8_t* residual, float* corr, int32_t* assign) const {
    DeviceGuard g(dev_);
    const int64_t n = ntotal_;
    if (n == 0) return;
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    const uint8_t* pc = paging() ? hpcodes_.get() : dpcodes_.get();
    const uint8_t* rc = paging() ? hrcodes_.get() : drcodes_.get();
    const float* co = paging() ? hcorr_.get() : dcorr_.get();
    if (primary) JHQ_CUDA(cudaMemcpy(primary, pc, (size_t)n * M_, cudaMemcpyDefault));
    if (residual)
        JHQ_CUDA(cudaMemcpy2D(residual, bpv_, rc, bpv_pad_, bpv_, (size_t)n, cudaMemcpyDefault));
    if (corr) JHQ_CUDA(cudaMemcpy(corr, co, (size_t)n * 4, cudaMemcpyDefault));
    if (assign) std::memcpy(assign, h_assign_.data(), (size_t)n * 4);
}

void Index::rotate_queries(const float* h_x, int64_t n, float* h_y) {
    DeviceGuard g(dev_);
    if (!trained_) fail(JHQ_ESTATE, "index is not trained");
    if (n <= 0) return;
    DevBuf<float> dx((size_t)n * d_), dy((size_t)n * d_), sc(std::max<size_t>(1, rotq_scratch_floats((int)n)));
    h2d(dx.get(), h_x, (size_t)n * d_, stream_);
    rotate_queries_device(dx.get(), n, dy.get(), sc.get(), stream_);
    d2h(h_y, dy.get(), (size_t)n * d_, stream_);
    JHQ_CUDA(cudaStreamSynchronize(stream_));
}

void Index::rotate(const float* h_x, int64_t n, float* h_y) {
    DeviceGuard g(dev_);
    if (!trained_) fail(JHQ_ESTATE, "index is not trained");
    if (n <= 0) return;
    DevBuf<float> dx((size_t)n * d_), dy((size_t)n * d_);
    h2d(dx.get(), h_x, (size_t)n * d_, stream_);
    rotate_device(dx.get(), n, dy.get(), stream_);
    d2h(h_y, dy.get(), (size_t)n * d_, stream_);
    JHQ_CUDA(cudaStreamSynchronize(stream_));
}

void Index::encode(const float* h_y, int64_t n, uint8_t* primary, uint8_t* residual, float* corr) {
    DeviceGuard g(dev_);
    if (!trained_) fail(JHQ_ESTATE, "index is not trained");
    if (n <= 0) return;
    DevBuf<float> dy((size_t)n * d_);
    DevBuf<uint8_t> pc((size_t)n * M_), rc((size_t)n * bpv_pad_);
    DevBuf<float> co((size_t)n);
    h2d(dy.get(), h_y, (size_t)n * d_, stream_);
    encode_rows(dy.get(), n, d_, M_, B_, Br_, dc1d_.get(), dres_.get(), res_per_sub_, pc.get(), rc.get(),
                bpv_pad_, co.get(), stream_);
    JHQ_CUDA(cudaStreamSynchronize(stream_));
    if (primary) JHQ_CUDA(cudaMemcpy(primary, pc.get(), (size_t)n * M_, cudaMemcpyDeviceToHost));
    if (residual)
        JHQ_CUDA(cudaMemcpy2D(residual, bpv_, rc.get(), bpv_pad_, bpv_, (size_t)n,
                              cudaMemcpyDeviceToHost));
    if (corr) JHQ_CUDA(cudaMemcpy(corr, co.get(), (size_t)n * 4, cudaMemcpyDeviceToHost));
}

// ---- persistence ----------------------------------------------------------------
namespace {
constexpr char MAGIC[8] = {'J', 'H', 'Q', 'B', '2', '0', '0', '\0'};
constexpr uint32_t FORMAT_VERSION = 1;
}

void Index::save(const std::string& path) const {
    DeviceGuard g(dev_);
    if (!trained_) fail(JHQ_ESTATE, "save: index is not trained");
    std::ofstream f(path, std::ios::binary);
    if (!f) fail(JHQ_EIO, "save: cannot open " + path);
    auto put = [&](const void* p, size_t n) { f.write(static_cast<const char*>(p), (std::streamsize)n); };
    put(MAGIC, 8);
    put(&FORMAT_VERSION, 4);
    int32_t hdr[12] = {d_, p_.M, p_.B, p_.Br, p_.nlist, p_.nprobe, p_.ivf_iters,
                       p_.batch_size, p_.seed, p_.add_batch, pilotP_,
                       (keep_raw_ ? 1 : 0) | (res_per_sub_ ? 2 : 0) | (rerank_ << 8)};
                       // flags: kept vectors, per-subspace residual codebooks, rerank R
    put(hdr, sizeof hdr);
    put(&p_.alpha, 4);
    put(&sigma_, 4);
    put(&ntotal_, 8);
    put(Pi_.data(), Pi_.size() * 4);
    put(c1d_.data(), c1d_.size() * 4);
    put(res_c1d_.data(), res_c1d_.size() * 4);
    put(cents_.data(), cents_.size() * 4);
    if (pilotP_ > 0) put(pilot_cents_.data(), pilot_cents_.size() * 4);
    if (ntotal_ > 0) {
        std::vector<uint8_t> pc((size_t)ntotal_ * M_), rc((size_t)ntotal_ * bpv_);
        std::vector<float> co((size_t)ntotal_);
        std::vector<int32_t> as((size_t)ntotal_);
        get_codes(pc.data(), rc.data(), co.data(), as.data());
        put(pc.data(), pc.size());
        put(rc.data(), rc.size());
        put(co.data(), co.size() * 4);
        put(as.data(), as.size() * 4);
        if (pilotP_ > 0) put(h_pilot_assign_.data(), (size_t)ntotal_ * 4);
        if (keep_raw_) {
            std::vector<float> rw((size_t)ntotal_ * d_);
            JHQ_CUDA(cudaMemcpy(rw.data(), paging() ? hraw_.get() : draw_.get(), rw.size() * 4,
                                cudaMemcpyDefault));
            put(rw.data(), rw.size() * 4);
        }
    }
    if (!f) fail(JHQ_EIO, "save: write failed for " + path);
}

Index* Index::load(const std::string& path, int device) {
    std::ifstream f(path, std::ios::binary);
    if (!f) fail(JHQ_EIO, "load: cannot open " + path);
    auto get = [&](void* p, size_t n) {
        f.read(static_cast<char*>(p), (std::streamsize)n);
        if (!f) fail(JHQ_EIO, "load: truncated file " + path);
    };
    char magic[8];
    uint32_t ver = 0;
    get(magic, 8);
    get(&ver, 4);
    if (std::memcmp(magic, MAGIC, 8) != 0 || ver != FORMAT_VERSION) fail(JHQ_EIO, "load: not a JHQ-B200 index file");
    int32_t hdr[12];
    get(hdr, sizeof hdr);
    Params p;
    p.M = hdr[1]; p.B = hdr[2]; p.Br = hdr[3]; p.nlist = hdr[4]; p.nprobe = hdr[5];
    p.ivf_iters = hdr[6]; p.batch_size = hdr[7]; p.seed = hdr[8]; p.add_batch = hdr[9];
    p.device = device;
    get(&p.alpha, 4);
    float sigma;
    int64_t n;
    get(&sigma, 4);
    get(&n, 8);
    if (n < 0 || n > INT32_MAX) fail(JHQ_EIO, "load: bad vector count");
    Index* idx = new Index(hdr[0], p);
    try {
        const int d = idx->d_;
        idx->res_per_sub_ = (hdr[11] & 2) != 0;
        if (idx->res_per_sub_ && (size_t)idx->M_ * idx->Kr_ > 16384) fail(JHQ_EIO, "load: bad flags");
        std::vector<float> Pi((size_t)d * d), c1d(idx->K1D_), res((size_t)idx->residual_floats()),
            cents((size_t)p.nlist * d);
        get(Pi.data(), Pi.size() * 4);
        get(c1d.data(), c1d.size() * 4);
        get(res.data(), res.size() * 4);
        get(cents.data(), cents.size() * 4);
        idx->set_trained(Pi.data(), c1d.data(), res.data(), cents.data(), sigma);
        const int P = hdr[10];                       // pilot clusters (0 = none)
        if (P < 0 || P > (1 << 20)) fail(JHQ_EIO, "load: bad pilot cluster count");
        if (P > 0) {
            std::vector<float> pc((size_t)P * d);
            get(pc.data(), pc.size() * 4);
            DeviceGuard g(idx->dev_);
            idx->pilot_cents_ = pc;
            idx->upload_pilot(pc, P);
            idx->pilotP_ = P;
        }
        const int flags = hdr[11];
        if ((flags & 1) && idx->d_ % 4 != 0) fail(JHQ_EIO, "load: bad flags");
        idx->keep_raw_ = (flags & 1) != 0;
        idx->rerank_ = idx->keep_raw_ ? (flags >> 8) : 0;
        if (idx->rerank_ < 0 || idx->rerank_ > MAX_CK_PAD) fail(JHQ_EIO, "load: bad rerank depth");
        if (n > 0) {
            DeviceGuard g(idx->dev_);
            std::vector<uint8_t> pc((size_t)n * idx->M_), rc((size_t)n * idx->bpv_);
            std::vector<float> co((size_t)n);
            std::vector<int32_t> as((size_t)n);
            get(pc.data(), pc.size());
            get(rc.data(), rc.size());
            get(co.data(), co.size() * 4);
            get(as.data(), as.size() * 4);
            for (int32_t a : as)
                if (a < 0 || a >= p.nlist) fail(JHQ_EIO, "load: bad list id");
            if (P > 0) {
                idx->h_pilot_assign_.resize((size_t)n);
                get(idx->h_pilot_assign_.data(), (size_t)n * 4);
                for (int32_t a : idx->h_pilot_assign_)
                    if (a < 0 || a >= P) fail(JHQ_EIO, "load: bad pilot cluster id");
            }
            idx->grow_master(n);
            JHQ_CUDA(cudaMemcpy(idx->dpcodes_.get(), pc.data(), pc.size(), cudaMemcpyHostToDevice));
            JHQ_CUDA(cudaMemcpy2D(idx->drcodes_.get(), idx->bpv_pad_, rc.data(), idx->bpv_, idx->bpv_,
                                  (size_t)n, cudaMemcpyHostToDevice));
            JHQ_CUDA(cudaMemset2D(idx->drcodes_.get() + idx->bpv_, idx->bpv_pad_, 0,
                                  idx->bpv_pad_ - idx->bpv_, (size_t)n));
            JHQ_CUDA(cudaMemcpy(idx->dcorr_.get(), co.data(), co.size() * 4, cudaMemcpyHostToDevice));
            JHQ_CUDA(cudaMemcpy(idx->dassign_.get(), as.data(), as.size() * 4, cudaMemcpyHostToDevice));
            if (idx->keep_raw_) {
                std::vector<float> rw((size_t)n * d);
                get(rw.data(), rw.size() * 4);
                JHQ_CUDA(cudaMemcpy(idx->draw_.get(), rw.data(), rw.size() * 4, cudaMemcpyHostToDevice));
            }
            idx->h_assign_ = std::move(as);
            idx->ntotal_ = n;
            idx->rebuild_layout();
        }
    } catch (...) {
        delete idx;
        throw;
    }
    return idx;
}

}  // namespace jhq
