// Test/baseline infrastructure (oracle/_ref only): a C-ABI shim that runs one of
// the reference's own hblock graph indexes (hblock_v34/v35/v36, chosen by
// HB_NS / HB_HEADER at compile time) through its public API exactly as its demo
// main does (examples/demo_hblock_v34.cu:62-110): train on min(n, 200k) rows,
// add all rows, one warm-up search at the largest ef, then for every ef of the
// sweep `reps` timed searches with host buffers. Built by oracle/Makefile from
// the reference tree; the product never links it.
#include <algorithm>
#include <chrono>
#include <exception>
#include HB_HEADER

extern "C" int ref_hblock_run(const float* x, int n, const float* q, int nq, int d, int k,
                              int max_ef, int batch, const int* efs, int nef, int reps,
                              int* out_i, double* train_ms, double* add_ms, double* search_ms) {
    using Clock = std::chrono::high_resolution_clock;
    using Ms = std::chrono::duration<double, std::milli>;
    try {
        HB_NS::HBlockIndex::Params p;          // the demo's defaults otherwise
        p.max_ef = max_ef;
        p.batch_size = batch;
        HB_NS::HBlockIndex idx(d, p);
        auto t0 = Clock::now();
        idx.train(x, std::min(n, 200000));
        *train_ms = Ms(Clock::now() - t0).count();
        t0 = Clock::now();
        idx.add(x, n);
        *add_ms = Ms(Clock::now() - t0).count();
        std::vector<float> dist((size_t)nq * k);
        std::vector<int> ids((size_t)nq * k);
        idx.search(q, nq, k, dist.data(), ids.data(), max_ef);      // warm-up
        for (int s = 0; s < nef; ++s) {
            int* o = out_i + (size_t)s * nq * k;
            t0 = Clock::now();
            for (int r = 0; r < reps; ++r) idx.search(q, nq, k, dist.data(), o, efs[s]);
            search_ms[s] = Ms(Clock::now() - t0).count() / reps;
        }
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}
