// Test/baseline infrastructure (oracle/_ref only): a C-ABI shim that runs the
// reference's own CUDA index (jhq_gpu::JHQGpuIndex of the version directory
// this file is compiled against, e.g. jhq_v14_streaming_add or jhq_v1_plain)
// through its public API — train, add, one warm-up search, then timed
// searches — exactly as the reference's demo mains do
// (examples/demo_jhq_v14_streaming_add.cu:78-106). Built by oracle/Makefile
// from the reference tree; the product never links it.
#include <chrono>
#include <cstring>
#include <exception>
#include <vector>

// The nprobe sweep below lowers the reference index's private nprobe_ member
// between searches (the reference fixes it at construction and sizes its probe
// buffers for it, so the index is built with the largest value of the sweep).
#ifdef REF_HAS_IVF
#define private public
#endif
#include REF_INDEX_HEADER
#ifdef REF_HAS_IVF
#undef private
#endif

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
