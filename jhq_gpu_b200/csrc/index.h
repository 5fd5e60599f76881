// index.h — jhq::Index, the B200 counterpart of the reference's
// jhq_gpu::JHQGpuIndex (jhq_v14_streaming_add/jhq_gpu_index.cuh:14-83) with
// its SearchWorkspace (search.cuh:24-46).
//
// Device data held per index (HBM):
//   Pi [d][d] fp32 (the reference's column-major array, used as the row-major
//   right operand of y = x . Pi), c1d [K1D], res_c1d [Kr], centroids
//   transposed [d][nlist] and their norms [nlist];
//   id-ordered "master" codes: primary [N][M], residual [N][bpv_pad]
//   (bpv_pad = ceil(d*Br/8) rounded up to 16), corr [N], list [N];
//   the scan layout: pages [npages][Mp/16][32][16] of primary codes grouped
//   by list (each list padded to whole 32-vector pages), slot_ids
//   [npages*32] (-1 = empty slot) and list_page_off [nlist+1].
// The master arrays grow geometrically, so add() may be called repeatedly;
// the page layout is rebuilt from them after every add().
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <algorithm>
#include <functional>
#include <string>
#include <vector>

#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {

struct Params {
    int M = 96, B = 8, Br = 4;
    float alpha = 4.0f;
    int nlist = 1024, nprobe = 8, ivf_iters = 8, batch_size = 256, seed = 42;
    int add_batch = 65536;
    int device = -1;
};

class Index {
public:
    Index(int d, const Params& p);
    ~Index();
    Index(const Index&) = delete;
    Index& operator=(const Index&) = delete;

    void train(const float* h_x, int64_t n);
    void add(const float* h_x, int64_t n);
    void search(const float* h_q, int64_t nq, int k, float* h_dists, int32_t* h_ids);
    void search_device(const float* d_q, int64_t nq, int k, float* d_dists, int32_t* d_ids,
                       cudaStream_t stream);
    // Same search as search_device, but every temporary lives in a fixed
    // device array compiled into the library (noalloc.cu); nothing is allocated.
    void search_device_noalloc(const float* d_q, int64_t nq, int k, float* d_dists,
                               int32_t* d_ids, cudaStream_t stream);
    void synchronize(double timeout_s);
    // Raises JHQ_ETIMEDOUT (and clears the flag) when a bounded device wait of a
    // search enqueued on any stream gave up; call after that stream has drained.
    void check_device_status();
    // Diagnostics of the tensor-core flat scan: the approximate ADC scores
    // s~[q][v] of host queries (same rotation and GEMM as search), or false when
    // this index does not use the tensor-core flat scan.
    bool flat_tc_scores(const float* h_q, int nq, float* h_scores);
    void set_nprobe(int nprobe);
    void set_alpha(float alpha);
    void probe_device(const float* d_q, int64_t nq, int32_t* d_probes, cudaStream_t stream);
    void search_device_probes(const float* d_q, const int32_t* d_probes, int64_t nq, int k,
                              float* d_dists, int32_t* d_ids, cudaStream_t stream);

    int64_t ntotal() const { return ntotal_; }
    int dim() const { return d_; }
    bool trained() const { return trained_; }
    const Params& params() const { return p_; }
    int device() const { return dev_; }

    void get_trained(float* Pi, float* c1d, float* res_c1d, float* cents, float* sigma) const;
    void set_trained(const float* Pi, const float* c1d, const float* res_c1d, const float* cents,
                     float sigma);
    void get_codes(uint8_t* primary, uint8_t* residual, float* corr, int32_t* assign) const;
    void rotate(const float* h_x, int64_t n, float* h_y);
    void rotate_queries(const float* h_x, int64_t n, float* h_y);
    void encode(const float* h_y, int64_t n, uint8_t* primary, uint8_t* residual, float* corr);
    void save(const std::string& path) const;
    static Index* load(const std::string& path, int device);

    void set_profiling(bool on);
    void stage_times(double* ms, int64_t* batches, int n) const;

    int K1D() const { return K1D_; }
    int pilot_lists() const { return pilotP_; }
    // Pilot clusters (flat index): copy out [P][d]; install on a trained, empty index.
    const std::vector<float>& pilot_centroids() const { return pilot_cents_; }
    void set_pilot(const float* cents, int P);
    int Kr() const { return Kr_; }
    int bpv() const { return bpv_; }
    // Exact rerank: the index keeps its vectors as given (fp32, [N][d]) from the
    // first add() on; a search for k then takes the best max(R, k) JHQ
    // candidates and returns the k nearest of them by exact L2. R = 0 turns the
    // rerank off (the reference's JHQ search); the stored vectors stay.
    void set_rerank(int R);
    // Residual codebooks: one global Kr-entry codebook (the reference's format,
    // default) or M per-subspace codebooks, res_c1d [M][Kr] (dim j uses codebook
    // j / Ds). Chosen before train() / set_trained(); fixed afterwards.
    void set_residual_codebooks(bool per_subspace);
    // Out-of-core list paging: the codes (page layout, slot ids, residual codes,
    // corr, kept vectors) live in mapped pinned host memory, and every search
    // batch stages the pages of the lists it probes into a device pool of
    // `pool_bytes` (waves of queries when the union does not fit). IVF only
    // (nlist > 1); enable before the first add(). 0 = off (all resident).
    void set_list_paging(int64_t pool_bytes);
    bool paging() const { return pool_pages_ > 0; }
    int64_t pool_pages() const { return pool_pages_; }
    int64_t paging_waves() const { return paging_waves_; }
    bool residual_per_subspace() const { return res_per_sub_; }
    int residual_floats() const { return res_per_sub_ ? M_ * Kr_ : Kr_; }
    int rerank() const { return rerank_; }
    // vectors per IVF list [nlist] (host copy of the assignment; no device work)
    void list_sizes(int64_t* sizes) const;
    bool keeps_vectors() const { return keep_raw_; }

private:
    struct Workspace {                 // SearchWorkspace (search.cuh:24-46)
        int batch_cap = 0, k = 0, ck = 0, ck_pad = 0, grid = 0;
        int mode = 0, chunk_pages = 64, qmajor = 0;
        int64_t max_slots = 0;         // candidate slots a batch can need
        PinnedBuf<float> h_q;          // [batch][d] staged queries
        PinnedBuf<float> h_d;          // [batch][k]
        PinnedBuf<int32_t> h_i;
        PinnedBuf<int> h_nvalid;
        DevBuf<float> q, q_rot, scores, out_d, rotq;
        DevBuf<unsigned char> flat;    // flat_search_tc scratch
        DevBuf<unsigned char> ivf;     // ivf_search_tc scratch
        int64_t ivf_tiles = 0;         // (query, probed tile) pairs it holds
        DevBuf<int32_t> probes, out_i, cnt, bucket_off, unit_off, fill, cpo;
        DevBuf<int2> bucket;
        DevBuf<int64_t> qslot_off;
        DevBuf<uint64_t> cand, gthr, pkeys;
        DevBuf<float> pscores;
        DevBuf<int> nvalid;
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        int64_t graph_kernels = 0;
        size_t coarse_floats = 0;
    };

    void upload_trained();
    void lloyd(const float* d_y, int64_t n, int nl, int iters, std::vector<float>& cents,
               const std::function<const int32_t*(const std::vector<float>&)>& assign);
    void upload_pilot(const std::vector<float>& c, int P);
    void rotate_device(const float* d_x, int64_t n, float* d_y, cudaStream_t s) const;
    // Search-side query rotation: tensor cores (rot_tc_, bf16 split, error below
    // 2^-16 |x||Pi|) or the exact fp32 chains; scratch holds rotq_scratch_floats(n).
    void rotate_queries_device(const float* d_x, int64_t n, float* d_y, float* scratch,
                               cudaStream_t s) const;
    size_t rotq_scratch_floats(int Bq) const;
    // q_rot [nq][d] -> probes [nq][nprobe] through scores [nq][nlist] (scratch):
    // tensor-core scores + margin selection, or the fp32 SIMT GEMM + exact
    // selection (JHQ_COARSE=simt); both give the same lists.
    // `scores` holds coarse_scratch_floats(Bq) floats (scores, then the split queries).
    void coarse_probes(const float* q_rot, int nq, int Bq, int nprobe, float* scores,
                       int32_t* probes, cudaStream_t s);
    size_t coarse_scratch_floats(int Bq) const;
    void assign_device(const float* d_y, int64_t n, int32_t* d_assign, cudaStream_t s);
    void grow_master(int64_t need);
    void rebuild_layout();
    void prepare_workspace(int k);
    void destroy_graph();
    // Shapes of one search batch: ck, scan mode / grid / chunking, slot bound.
    struct BatchShape {
        int Bq, k, kr, ck, ck_pad, grid, mode, chunk_pages, qmajor;
        int64_t max_slots;
    };
    // Device temporaries of one batch (workspace or fixed scratch array).
    struct BatchBufs {
        float* q_rot;
        float* scores;
        int32_t* probes;
        PlanBufs plan;
        uint64_t* cand;
        uint64_t* pkeys = nullptr;     // pilot scratch (flat index with pilot clusters)
        float* pscores = nullptr;
        float* rotq = nullptr;         // tensor-core query rotation scratch
        void* flat = nullptr;          // tensor-core flat scan scratch (nullptr: SIMT scan)
        void* ivf = nullptr;           // tensor-core IVF scan scratch (nullptr: SIMT scan)
        int64_t ivf_tiles = 0;
    };
    BatchShape batch_shape(int Bq, int k) const;
    void enqueue_pipeline(const float* q_in, int nq, const int* d_nvalid, const BatchShape& sh,
                          const BatchBufs& b, float* out_d, int32_t* out_i, cudaStream_t s,
                          cudaEvent_t* ev, const int32_t* probes_in = nullptr);
    void enqueue_batch(cudaStream_t s, cudaEvent_t* ev = nullptr);
    // paged search of one batch (paging.cu): q_in [nq][d] on the device
    void run_paged_batch(const float* q_in, int nq, float* out_d, int32_t* out_i, cudaStream_t s);
    void build_host_pages(const std::vector<int32_t>& lpo, const std::vector<int32_t>& slots);
    void run_batch(cudaStream_t s, int nvalid);
    void check_search_args(int64_t nq, int k) const;
    // candidates the JHQ stage returns for a search of k: k, or max(R, k) with rerank
    int stage_k(int k) const { return rerank_ > 0 ? std::max(rerank_, k) : k; }
    // flat index with 1-bit codes: the ADC scan runs as a tensor-core GEMM of
    // the code bits with the queries (coarse_tc.cu: flat_search_tc)
    bool flat_tc() const;
    bool ivf_tc() const;

    int d_, M_, B_, Br_, Ds_, bpd_, K1D_, Kr_, bpv_, bpv_pad_, Mp_;
    Params p_;
    int dev_ = 0;
    cudaStream_t stream_ = nullptr;
    bool trained_ = false;
    int64_t ntotal_ = 0, cap_ = 0, npages_ = 0;
    std::vector<int32_t> h_list_pages_sorted_;   // list page counts, descending
    float sigma_ = 1.0f;
    std::vector<float> Pi_, c1d_, res_c1d_, cents_;
    std::vector<int32_t> h_assign_;
    bool layout_dirty_ = true;
    bool profiling_ = false;
    double stage_ms_[5] = {0, 0, 0, 0, 0};
    int64_t stage_batches_ = 0;
    cudaEvent_t prof_ev_[6] = {};

    DevBuf<float> dPi_, dc1d_, dres_, dcentsT_, dcents_, dnorms_;
    DevBuf<uint16_t> dcents3_;         // bf16 split centroids [nlist][K3]
    bool rot_tc_ = false;              // query rotation on the tensor cores
    DevBuf<uint16_t> dPi3_;            // bf16 split rows of Pi^T [d][K3]
    DevBuf<float> dzero_;              // d zeros (the rotation's "norms")
    // Pilot clusters of a flat index: per query, the ADC keys of the nearest
    // cluster's members seed its pruning bound (pilot.cu).
    static constexpr int PILOT_LISTS = 64, PILOT_MIN_MEMBERS = 16;
    int pilotP_ = 0;
    std::vector<float> pilot_cents_;   // [P][d]
    std::vector<int32_t> h_pilot_assign_;
    DevBuf<float> dpilot_centsT_, dpilot_cents_, dpilot_norms_;
    DevBuf<int32_t> dpilot_off_, dpilot_ids_;
    DevBuf<float> dassign_scratch_;    // tensor-core assignment: scores of a row block
    float cmax_ = 0.0f;                // >= max |centroid| (coarse margin)
    bool coarse_tc_ = false;
    DevBuf<uint8_t> dpcodes_, drcodes_, dpages_;
    DevBuf<float> dcorr_;
    DevBuf<int32_t> dpop_;             // popcount of each primary code row (flat tensor-core scan)
    bool res_per_sub_ = false;         // M per-subspace residual codebooks
    // list paging (paging.cu): host-resident codes + device page pool
    int64_t pool_pages_ = 0, paging_waves_ = 0;
    MappedBuf<uint8_t> hpcodes_, hrcodes_, hpages_;
    MappedBuf<float> hcorr_, hraw_;
    MappedBuf<int32_t> hslot_ids_;
    std::vector<int32_t> h_lpo_;               // list page offsets (host copy)
    DevBuf<uint8_t> dpool_pages_;
    DevBuf<int32_t> dpool_slots_, dlpo_wave_;
    DevBuf<int64_t> dseg_;
    bool keep_raw_ = false;            // stored vectors for the exact rerank
    int rerank_ = 0;
    DevBuf<float> draw_;               // [cap][d] vectors as given (keep_raw_)
    DevBuf<int32_t> dassign_, dslot_ids_, dlist_page_off_;
    Workspace ws_;
};

}  // namespace jhq
