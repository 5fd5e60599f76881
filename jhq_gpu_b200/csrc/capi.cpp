// capi.cpp — the extern "C" boundary of include/jhq.h over jhq::Index.
// Every entry point catches all exceptions and turns them into a JHQ_*
// status plus a thread-local message (jhq_last_error); nothing exits.
#include <cuda_runtime.h>

#include <cstring>
#include <exception>
#include <new>
#include <string>
#include <vector>
#include <climits>

#include "../../include/jhq.h"
#include "index.h"
#include "sharded.h"
#include "kernels.cuh"
#include "train_cpu.h"

struct jhq_index {
    jhq::Index* impl;
};

struct jhq_sharded {
    jhq::ShardedIndex* impl;
};

namespace {
thread_local std::string g_last_error;

template <class F>
int guarded(F&& f) {
    try {
        f();
        g_last_error.clear();
        return JHQ_OK;
    } catch (const jhq::Error& e) {
        g_last_error = e.what();
        return e.code();
    } catch (const std::bad_alloc&) {
        g_last_error = "host allocation failed";
        return JHQ_ENOMEM;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return JHQ_EDEVICE;
    } catch (...) {
        g_last_error = "unknown error";
        return JHQ_EDEVICE;
    }
}

jhq::Params to_params(const jhq_params* p) {
    jhq::Params q;
    q.M = p->M; q.B = p->B; q.Br = p->Br; q.alpha = p->alpha; q.nlist = p->nlist;
    q.nprobe = p->nprobe; q.ivf_iters = p->ivf_iters; q.batch_size = p->batch_size;
    q.seed = p->seed; q.add_batch = p->add_batch; q.device = p->device;
    return q;
}

jhq::Index* need(const jhq_index* idx) {
    if (!idx || !idx->impl) jhq::fail(JHQ_EINVAL, "null index");
    return idx->impl;
}
}  // namespace

extern "C" {

int jhq_params_default(jhq_params* p) {
    if (!p) { g_last_error = "null params"; return JHQ_EINVAL; }
    jhq::Params d;
    p->M = d.M; p->B = d.B; p->Br = d.Br; p->alpha = d.alpha; p->nlist = d.nlist;
    p->nprobe = d.nprobe; p->ivf_iters = d.ivf_iters; p->batch_size = d.batch_size;
    p->seed = d.seed; p->add_batch = d.add_batch; p->device = -1;
    return JHQ_OK;
}

int jhq_index_create(int d, const jhq_params* p, jhq_index** out) {
    return guarded([&] {
        if (!out) jhq::fail(JHQ_EINVAL, "null output pointer");
        *out = nullptr;
        jhq_params def;
        if (!p) { jhq_params_default(&def); p = &def; }
        auto* h = new jhq_index{nullptr};
        try { h->impl = new jhq::Index(d, to_params(p)); } catch (...) { delete h; throw; }
        *out = h;
    });
}

int jhq_index_destroy(jhq_index* idx) {
    return guarded([&] {
        if (!idx) return;
        delete idx->impl;
        delete idx;
    });
}

int jhq_train(jhq_index* idx, const float* x, int64_t n) {
    return guarded([&] { need(idx)->train(x, n); });
}

int jhq_add(jhq_index* idx, const float* x, int64_t n) {
    return guarded([&] { need(idx)->add(x, n); });
}

int jhq_search(jhq_index* idx, const float* q, int64_t nq, int k, float* dists, int32_t* ids) {
    return guarded([&] { need(idx)->search(q, nq, k, dists, ids); });
}

int jhq_search_device(jhq_index* idx, const float* d_q, int64_t nq, int k, float* d_dists,
                      int32_t* d_ids, void* stream) {
    return guarded([&] {
        need(idx)->search_device(d_q, nq, k, d_dists, d_ids, static_cast<cudaStream_t>(stream));
    });
}

int jhq_search_device_noalloc(jhq_index* idx, const float* d_q, int64_t nq, int k,
                              float* d_dists, int32_t* d_ids, void* stream) {
    return guarded([&] {
        need(idx)->search_device_noalloc(d_q, nq, k, d_dists, d_ids,
                                         static_cast<cudaStream_t>(stream));
    });
}

int jhq_synchronize(jhq_index* idx, double timeout_s) {
    return guarded([&] { need(idx)->synchronize(timeout_s); });
}

int jhq_probe_device(jhq_index* idx, const float* d_q, int64_t nq, int32_t* d_probes,
                     void* stream) {
    return guarded([&] {
        need(idx)->probe_device(d_q, nq, d_probes, static_cast<cudaStream_t>(stream));
    });
}

int jhq_search_device_probes(jhq_index* idx, const float* d_q, const int32_t* d_probes,
                             int64_t nq, int k, float* d_dists, int32_t* d_ids, void* stream) {
    return guarded([&] {
        need(idx)->search_device_probes(d_q, d_probes, nq, k, d_dists, d_ids,
                                        static_cast<cudaStream_t>(stream));
    });
}

int jhq_set_nprobe(jhq_index* idx, int nprobe) {
    return guarded([&] { need(idx)->set_nprobe(nprobe); });
}

int jhq_set_residual_codebooks(jhq_index* idx, int per_subspace) {
    return guarded([&] { need(idx)->set_residual_codebooks(per_subspace != 0); });
}

int jhq_get_residual_codebooks(const jhq_index* idx, int* per_subspace) {
    return guarded([&] {
        if (!per_subspace) jhq::fail(JHQ_EINVAL, "null output");
        *per_subspace = need(idx)->residual_per_subspace() ? 1 : 0;
    });
}

int jhq_set_list_paging(jhq_index* idx, int64_t pool_bytes) {
    return guarded([&] { need(idx)->set_list_paging(pool_bytes); });
}

int jhq_paging_waves(const jhq_index* idx, int64_t* waves) {
    return guarded([&] {
        if (!waves) jhq::fail(JHQ_EINVAL, "null output");
        *waves = need(idx)->paging_waves();
    });
}

int jhq_debug_flat_scores(jhq_index* idx, const float* q, int nq, float* scores) {
    return guarded([&] {
        if (!q || !scores) jhq::fail(JHQ_EINVAL, "null buffer");
        if (!need(idx)->flat_tc_scores(q, nq, scores))
            jhq::fail(JHQ_ESTATE, "this index does not use the tensor-core flat scan (or nq > 128)");
    });
}

int jhq_device_status(jhq_index* idx) {
    return guarded([&] { need(idx)->check_device_status(); });
}

int jhq_list_sizes(const jhq_index* idx, int64_t* sizes) {
    return guarded([&] {
        if (!sizes) jhq::fail(JHQ_EINVAL, "null output");
        need(idx)->list_sizes(sizes);
    });
}

int jhq_set_alpha(jhq_index* idx, float alpha) {
    return guarded([&] { need(idx)->set_alpha(alpha); });
}

int jhq_set_rerank(jhq_index* idx, int R) {
    return guarded([&] { need(idx)->set_rerank(R); });
}

int jhq_get_rerank(const jhq_index* idx, int* R) {
    return guarded([&] {
        if (!R) jhq::fail(JHQ_EINVAL, "null output");
        *R = need(idx)->rerank();
    });
}

int jhq_ntotal(const jhq_index* idx, int64_t* n) {
    return guarded([&] {
        if (!n) jhq::fail(JHQ_EINVAL, "null output");
        *n = need(idx)->ntotal();
    });
}

int jhq_dim(const jhq_index* idx, int* d) {
    return guarded([&] {
        if (!d) jhq::fail(JHQ_EINVAL, "null output");
        *d = need(idx)->dim();
    });
}

int jhq_is_trained(const jhq_index* idx, int* t) {
    return guarded([&] {
        if (!t) jhq::fail(JHQ_EINVAL, "null output");
        *t = need(idx)->trained() ? 1 : 0;
    });
}

int jhq_get_trained(const jhq_index* idx, float* Pi, float* c1d, float* res_c1d, float* cents,
                    float* sigma) {
    return guarded([&] { need(idx)->get_trained(Pi, c1d, res_c1d, cents, sigma); });
}

int jhq_set_trained(jhq_index* idx, const float* Pi, const float* c1d, const float* res_c1d,
                    const float* cents, float sigma) {
    return guarded([&] { need(idx)->set_trained(Pi, c1d, res_c1d, cents, sigma); });
}

int jhq_get_codes(const jhq_index* idx, uint8_t* primary, uint8_t* residual, float* corr,
                  int32_t* assign) {
    return guarded([&] { need(idx)->get_codes(primary, residual, corr, assign); });
}

int jhq_rotate_queries(jhq_index* idx, const float* x, int64_t n, float* y) {
    return guarded([&] {
        if (n < 0 || (n > 0 && (!x || !y))) jhq::fail(JHQ_EINVAL, "rotate_queries: bad buffers");
        need(idx)->rotate_queries(x, n, y);
    });
}

int jhq_rotate(jhq_index* idx, const float* x, int64_t n, float* y) {
    return guarded([&] {
        if (n > 0 && (!x || !y)) jhq::fail(JHQ_EINVAL, "null buffer");
        need(idx)->rotate(x, n, y);
    });
}

int jhq_encode(jhq_index* idx, const float* y, int64_t n, uint8_t* primary, uint8_t* residual,
               float* corr) {
    return guarded([&] {
        if (n > 0 && !y) jhq::fail(JHQ_EINVAL, "null buffer");
        need(idx)->encode(y, n, primary, residual, corr);
    });
}

int jhq_save(const jhq_index* idx, const char* path) {
    return guarded([&] {
        if (!path) jhq::fail(JHQ_EINVAL, "null path");
        need(idx)->save(path);
    });
}

int jhq_load(const char* path, int device, jhq_index** out) {
    return guarded([&] {
        if (!path || !out) jhq::fail(JHQ_EINVAL, "null argument");
        *out = nullptr;
        auto* h = new jhq_index{nullptr};
        try { h->impl = jhq::Index::load(path, device); } catch (...) { delete h; throw; }
        *out = h;
    });
}

int jhq_merge_shards(const float* d_in_dists, const int32_t* d_in_ids, int nshards, int64_t nq,
                     int k, float* d_out_dists, int32_t* d_out_ids, void* stream) {
    return guarded([&] {
        if (nshards <= 0 || k <= 0 || nq < 0) jhq::fail(JHQ_EINVAL, "merge_shards: bad sizes");
        if (nq > 0 && (!d_in_dists || !d_in_ids || !d_out_dists || !d_out_ids))
            jhq::fail(JHQ_EINVAL, "merge_shards: null buffer");
        jhq::merge_shard_lists(d_in_dists, d_in_ids, nshards, nq, k, d_out_dists, d_out_ids,
                               static_cast<cudaStream_t>(stream));
    });
}

int jhq_sharded_create(int d, const jhq_params* p, int nshards, const int* devices,
                       jhq_sharded** out) {
    return guarded([&] {
        if (!out) jhq::fail(JHQ_EINVAL, "null output pointer");
        *out = nullptr;
        if (nshards <= 0 || nshards > 64) jhq::fail(JHQ_EINVAL, "nshards must be in 1..64");
        jhq_params def;
        if (!p) { jhq_params_default(&def); p = &def; }
        std::vector<int> devs(nshards);
        for (int s = 0; s < nshards; ++s) devs[s] = devices ? devices[s] : s;
        auto* h = new jhq_sharded{nullptr};
        try { h->impl = new jhq::ShardedIndex(d, to_params(p), devs); } catch (...) { delete h; throw; }
        *out = h;
    });
}

int jhq_sharded_destroy(jhq_sharded* idx) {
    return guarded([&] {
        if (!idx) return;
        delete idx->impl;
        delete idx;
    });
}

namespace {
jhq::ShardedIndex* need_sharded(const jhq_sharded* idx) {
    if (!idx || !idx->impl) jhq::fail(JHQ_EINVAL, "null sharded index");
    return idx->impl;
}
}  // namespace

int jhq_sharded_train(jhq_sharded* idx, const float* x, int64_t n_train) {
    return guarded([&] {
        if (!x || n_train <= 0) jhq::fail(JHQ_EINVAL, "train: need at least one vector");
        need_sharded(idx)->train(x, n_train);
    });
}

int jhq_sharded_add(jhq_sharded* idx, const float* x, int64_t n) {
    return guarded([&] { need_sharded(idx)->add(x, n); });
}

int jhq_sharded_search(jhq_sharded* idx, const float* q, int64_t nq, int k, float* dists,
                       int32_t* ids) {
    return guarded([&] { need_sharded(idx)->search(q, nq, k, dists, ids); });
}

int jhq_sharded_set_nprobe(jhq_sharded* idx, int nprobe) {
    return guarded([&] { need_sharded(idx)->set_nprobe(nprobe); });
}

int64_t jhq_sharded_ntotal(const jhq_sharded* idx) {
    if (!idx || !idx->impl) return -1;
    return idx->impl->ntotal();
}

int jhq_set_profiling(jhq_index* idx, int on) {
    return guarded([&] { need(idx)->set_profiling(on != 0); });
}

int jhq_stage_times(const jhq_index* idx, double* ms, int64_t* batches, int n) {
    return guarded([&] { need(idx)->stage_times(ms, batches, n); });
}

int jhq_jl_rotation(int d, int seed, float* Pi) {
    return guarded([&] {
        if (d <= 0 || !Pi) jhq::fail(JHQ_EINVAL, "jl_rotation: bad argument");
        std::vector<float> P = jhq::train::build_rotation(d, seed);
        std::memcpy(Pi, P.data(), P.size() * sizeof(float));
    });
}

int jhq_estimate_sigma(const float* x, int64_t n, int d, float* sigma) {
    return guarded([&] {
        if (!x || n <= 0 || d <= 0 || !sigma) jhq::fail(JHQ_EINVAL, "estimate_sigma: bad argument");
        *sigma = jhq::train::estimate_sigma(x, n, d);
    });
}

int jhq_lloyd_max_c1d(float sigma, int K1D, float* c1d) {
    return guarded([&] {
        if (K1D <= 0 || K1D > 256 || !c1d) jhq::fail(JHQ_EINVAL, "lloyd_max_c1d: bad argument");
        std::vector<float> c = jhq::train::lloyd_max_c1d(sigma, K1D);
        std::memcpy(c1d, c.data(), c.size() * sizeof(float));
    });
}

int jhq_kmeans_1d(const float* vals, int64_t n, int Kr, int max_iter, float* out, int* nout) {
    return guarded([&] {
        if ((n > 0 && !vals) || !out || Kr <= 0 || n > INT32_MAX) jhq::fail(JHQ_EINVAL, "kmeans_1d: bad argument");
        std::vector<float> c = jhq::train::kmeans_1d(vals, n, Kr, max_iter);
        std::memcpy(out, c.data(), c.size() * sizeof(float));
        if (nout) *nout = (int)c.size();
    });
}

int64_t jhq_kernel_launches(void) { return jhq::g_kernel_launches.load(); }

const char* jhq_last_error(void) { return g_last_error.c_str(); }

const char* jhq_version(void) { return "jhq-b200 0.1 (sm_100a)"; }

}  // extern "C"
