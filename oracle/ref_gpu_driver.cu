// Test/baseline infrastructure (oracle/_ref only): a C-ABI shim that runs the
// reference's own CUDA index (jhq_gpu::JHQGpuIndex of the version directory
// this file is compiled against, e.g. jhq_v14_streaming_add or jhq_v1_plain)
// through its public API — train, add, one warm-up search, then timed
// searches — exactly as the reference's demo mains do
// (examples/demo_jhq_v14_streaming_add.cu:78-106). Built by oracle/Makefile
// from the reference tree; the product never links it.
#include <chrono>
#include <memory>
#include <stdexcept>
#include <cstring>
#include <exception>
#include <vector>

// The nprobe sweep below lowers the reference index's private nprobe_ member
// between searches (the reference fixes it at construction and sizes its probe
// buffers for it, so the index is built with the largest value of the sweep),
// and ref_gpu_pin writes trained artefacts into, and reads the encoded lists
// out of, its private members.
#define private public
#include REF_INDEX_HEADER
#undef private

extern "C" int ref_gpu_run(const float* x, int n, int n_train, const float* q, int nq, int d,
                           int M, int B, int Br, float alpha, int k, int nlist, int nprobe,
                           int batch, int reps, float* out_d, int* out_i,
                           double* train_ms, double* add_ms, double* search_ms) {
    using Clock = std::chrono::high_resolution_clock;
    using Ms = std::chrono::duration<double, std::milli>;
    try {
        jhq_gpu::JHQGpuIndex::Params p;
        p.M = M; p.B = B; p.Br = Br; p.alpha = alpha;
#ifdef REF_HAS_IVF
        p.nlist = nlist; p.nprobe = nprobe; p.batch_size = batch;
#else
        (void)nlist; (void)nprobe; (void)batch;
#endif
        jhq_gpu::JHQGpuIndex idx(d, p);
        auto t0 = Clock::now();
        idx.train(x, n_train);
        *train_ms = Ms(Clock::now() - t0).count();
        t0 = Clock::now();
        idx.add(x, n);
        *add_ms = Ms(Clock::now() - t0).count();
        idx.search(q, nq, k, out_d, out_i);               // warm-up (graph capture)
        t0 = Clock::now();
        for (int r = 0; r < reps; ++r) idx.search(q, nq, k, out_d, out_i);
        *search_ms = Ms(Clock::now() - t0).count() / reps;
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

#ifdef REF_HAS_IVF
// Train once with nprobe = max(nprobes), add, then for each nprobe value: one
// warm-up search and `reps` timed searches; ids of each sweep point go to
// out_i + s*nq*k, mean search wall time to search_ms[s].
extern "C" int ref_gpu_sweep(const float* x, int n, int n_train, const float* q, int nq, int d,
                             int M, int B, int Br, float alpha, int k, int nlist,
                             const int* nprobes, int nsweep, int batch, int reps, int* out_i,
                             double* train_ms, double* add_ms, double* search_ms) {
    using Clock = std::chrono::high_resolution_clock;
    using Ms = std::chrono::duration<double, std::milli>;
    try {
        int npmax = 1;
        for (int s = 0; s < nsweep; ++s) npmax = nprobes[s] > npmax ? nprobes[s] : npmax;
        jhq_gpu::JHQGpuIndex::Params p;
        p.M = M; p.B = B; p.Br = Br; p.alpha = alpha;
        p.nlist = nlist; p.nprobe = npmax; p.batch_size = batch;
        jhq_gpu::JHQGpuIndex idx(d, p);
        auto t0 = Clock::now();
        idx.train(x, n_train);
        *train_ms = Ms(Clock::now() - t0).count();
        t0 = Clock::now();
        idx.add(x, n);
        *add_ms = Ms(Clock::now() - t0).count();
        std::vector<float> dist((size_t)nq * k);
        for (int s = 0; s < nsweep; ++s) {
            idx.nprobe_ = nprobes[s] < nlist ? nprobes[s] : nlist;
            int* ids = out_i + (size_t)s * nq * k;
            idx.search(q, nq, k, dist.data(), ids);
            t0 = Clock::now();
            for (int r = 0; r < reps; ++r) idx.search(q, nq, k, dist.data(), ids);
            search_ms[s] = Ms(Clock::now() - t0).count() / reps;
        }
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}
#endif

// ---------------------------------------------------------------------------
// Parity pin: run the reference's own add() encode and search() on artefacts
// given by the caller instead of its train(): the rotation is the identity and
// the caller passes already-rotated rows y and queries q_rot (I*x is exact in
// fp32 whatever the GEMM's summation order, so both builds see the same y),
// c1d / res_c1d / IVF centroids are the caller's. The centroid norms follow the
// reference's own rule (double sum, jhq_gpu_index.cu:241-247).
// Outputs, all in id order: primary codes [n][M], residual codes [n][bpv],
// corrections [n] (read back from the reference's device buffers and, for v14,
// un-permuted through its list_ids), and the search result [nq][k].
namespace {
template <class T>
static void up(T** dst, const T* src, size_t n) {
    cudaFree(*dst);
    *dst = nullptr;
    if (cudaMalloc((void**)dst, n * sizeof(T)) != cudaSuccess) throw std::bad_alloc();
    cudaMemcpy(*dst, src, n * sizeof(T), cudaMemcpyHostToDevice);
}
template <class T>
static void down(T* dst, const T* src, size_t n) {
    cudaMemcpy(dst, src, n * sizeof(T), cudaMemcpyDeviceToHost);
}
}  // namespace

// Builds the reference index on the caller's artefacts and adds y (see above).
static std::unique_ptr<jhq_gpu::JHQGpuIndex> pinned_index(
    const float* y, int n, int d, int M, int B, int Br, float alpha, int nlist, int nprobe,
    int batch, const float* c1d, int K1D, const float* res_c1d, int Kr, const float* cents,
    float sigma) {
    jhq_gpu::JHQGpuIndex::Params p;
    p.M = M; p.B = B; p.Br = Br; p.alpha = alpha;
#ifdef REF_HAS_IVF
    p.nlist = nlist; p.nprobe = nprobe; p.batch_size = batch;
#else
    (void)nlist; (void)nprobe; (void)batch; (void)cents;
#endif
    auto idx = std::make_unique<jhq_gpu::JHQGpuIndex>(d, p);
    if (K1D != idx->K1D_ || Kr != idx->Kr_) throw std::invalid_argument("codebook sizes");
    idx->cb_ = std::make_unique<LloydMaxCodebook>(d, M, B, sigma);
    std::vector<float> eye((size_t)d * d, 0.0f);
    for (int i = 0; i < d; ++i) eye[(size_t)i * d + i] = 1.0f;
    up(&idx->d_Pi_, eye.data(), eye.size());
    up(&idx->d_c1d_, c1d, (size_t)K1D);
    idx->res_c1d_.assign(res_c1d, res_c1d + Kr);
    up(&idx->d_res_c1d_, res_c1d, (size_t)Kr);
#ifdef REF_HAS_IVF
    idx->centroids_.assign(cents, cents + (size_t)nlist * d);
    std::vector<float> norms(nlist);
    for (int c = 0; c < nlist; ++c) {
        double s = 0.0;
        for (int j = 0; j < d; ++j) s += (double)cents[(size_t)c * d + j] * cents[(size_t)c * d + j];
        norms[c] = (float)s;
    }
    up(&idx->d_centroids_, cents, (size_t)nlist * d);
    up(&idx->d_cent_norms_, norms.data(), (size_t)nlist);
#endif
    idx->add(y, n);
    return idx;
}

extern "C" int ref_gpu_pin(const float* y, int n, const float* q_rot, int nq, int d, int M,
                           int B, int Br, float alpha, int k, int nlist, int nprobe, int batch,
                           const float* c1d, int K1D, const float* res_c1d, int Kr,
                           const float* cents, float sigma, uint8_t* out_pc, uint8_t* out_rc,
                           float* out_corr, float* out_d, int* out_i) {
    try {
        auto ip = pinned_index(y, n, d, M, B, Br, alpha, nlist, nprobe, batch, c1d, K1D, res_c1d,
                               Kr, cents, sigma);
        jhq_gpu::JHQGpuIndex& idx = *ip;
        const int bpv = idx.bpv_;
#ifdef REF_HAS_IVF
        std::vector<int> ids(n);
        std::vector<uint8_t> pt((size_t)M * n), rc((size_t)n * bpv);
        std::vector<float> co(n);
        down(ids.data(), idx.d_list_ids_, (size_t)n);
        down(pt.data(), idx.d_list_primary_t_, pt.size());
        down(rc.data(), idx.d_list_res_, rc.size());
        down(co.data(), idx.d_list_corr_, (size_t)n);
        for (int pos = 0; pos < n; ++pos) {
            const int v = ids[pos];
            if (v < 0 || v >= n) return 3;
            for (int m = 0; m < M; ++m) out_pc[(size_t)v * M + m] = pt[(size_t)m * n + pos];
            std::memcpy(out_rc + (size_t)v * bpv, rc.data() + (size_t)pos * bpv, bpv);
            out_corr[v] = co[pos];
        }
#else
        down(out_pc, idx.d_primary_codes_, (size_t)n * M);
        down(out_rc, idx.d_res_codes_, (size_t)n * bpv);
        down(out_corr, idx.d_corrections_, (size_t)n);
#endif
        idx.search(q_rot, nq, k, out_d, out_i);
        return cudaDeviceSynchronize() == cudaSuccess ? 0 : 4;
    } catch (const std::exception&) {
        return 1;
    }
}

// Timing on the caller's artefacts: for each alpha of the sweep (written into
// the index's private alpha_, which the reference fixes at construction), one
// warm-up search() and `reps` timed ones with host buffers (the demo's method,
// examples/demo_jhq_v14_streaming_add.cu:92-99). Ids of sweep point s go to
// out_i + s*nq*k, the mean search wall time to search_ms[s].
extern "C" int ref_gpu_pin_sweep(const float* y, int n, const float* q_rot, int nq, int d,
                                 int M, int B, int Br, int k, int nlist, int nprobe, int batch,
                                 const float* c1d, int K1D, const float* res_c1d, int Kr,
                                 const float* cents, float sigma, const float* alphas, int nalpha,
                                 int reps, int* out_i, double* add_ms, double* search_ms) {
    using Clock = std::chrono::high_resolution_clock;
    using Ms = std::chrono::duration<double, std::milli>;
    try {
        auto t0 = Clock::now();
        auto ip = pinned_index(y, n, d, M, B, Br, alphas[0], nlist, nprobe, batch, c1d, K1D,
                               res_c1d, Kr, cents, sigma);
        *add_ms = Ms(Clock::now() - t0).count();
        std::vector<float> dist((size_t)nq * k);
        for (int s = 0; s < nalpha; ++s) {
            ip->alpha_ = alphas[s];
            int* ids = out_i + (size_t)s * nq * k;
            ip->search(q_rot, nq, k, dist.data(), ids);
            t0 = Clock::now();
            for (int r = 0; r < reps; ++r) ip->search(q_rot, nq, k, dist.data(), ids);
            search_ms[s] = Ms(Clock::now() - t0).count() / reps;
        }
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}
