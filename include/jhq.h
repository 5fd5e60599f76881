/*
 * jhq.h — C-ABI of the B200 JHQ search engine (libjhq_b200.so).
 *
 * Drop-in boundary for the reference's jhq_gpu::JHQGpuIndex
 * (jhq_v14_streaming_add/jhq_gpu_index.cuh:14-47) and its search_gpu /
 * SearchWorkspace pair (jhq_v14_streaming_add/search.cuh:24-69). Each entry
 * point names the reference member it replaces. Plain pointers and sizes only;
 * every function returns a JHQ_* status (0 = success) and never exits or
 * throws; jhq_last_error() gives the message of the calling thread's last
 * failure. Host pointers are caller-owned; the index owns every device buffer.
 *
 * Threading: like the reference (whose search() is const but mutates a
 * mutable workspace, search.cuh:24-46 / jhq_gpu_index.cuh:73-74), one index
 * serves one caller at a time.
 */
#ifndef JHQ_B200_H
#define JHQ_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
#define JHQ_OK        0
#define JHQ_EINVAL    1   /* bad argument (reference: std::invalid_argument)      */
#define JHQ_ENOMEM    2   /* device or pinned allocation failed                    */
#define JHQ_ETIMEDOUT 3   /* a bounded wait on the device ran out                  */
#define JHQ_EDEVICE   4   /* CUDA error (reference: CUDA_CHECK -> exit(1))         */
#define JHQ_ESTATE    5   /* call order (reference: std::runtime_error, e.g.
                             "call train() before add()", "index is empty")      */
#define JHQ_EIO       6   /* save/load file error or bad format                    */

/* ---- parameters: JHQGpuIndex::Params (jhq_gpu_index.cuh:16-36) ------- */
typedef struct jhq_params {
    int   M;           /* subspaces                      (default 96)    */
    int   B;           /* primary bits per subspace      (default 8)     */
    int   Br;          /* residual bits per dim, 4 or 8  (default 4)     */
    float alpha;       /* ck = max(k, ceil(alpha k))     (default 4.0)   */
    int   nlist;       /* IVF lists, 1 = flat            (default 1024)  */
    int   nprobe;      /* lists probed per query         (default 8)     */
    int   ivf_iters;   /* k-means iterations             (default 8)     */
    int   batch_size;  /* queries per search batch       (default 256)   */
    int   seed;        /* JL rotation seed               (default 42)    */
    int   add_batch;   /* rows rotated+encoded at once   (default 65536) */
    int   device;      /* CUDA device ordinal; -1 = current device at create */
} jhq_params;

typedef struct jhq_index jhq_index;

/* Fills the reference's defaults (jhq_gpu_index.cuh:17-35), device = -1. */
int jhq_params_default(jhq_params* p);

/* JHQGpuIndex(int d, Params p) — validation as jhq_gpu_index.cu:103-131. */
int jhq_index_create(int d, const jhq_params* p, jhq_index** out);
/* ~JHQGpuIndex() — jhq_gpu_index.cu:133-163. NULL is accepted. */
int jhq_index_destroy(jhq_index* idx);

/* JHQGpuIndex::train(h_x, n_train) — jhq_gpu_index.cu:333-364.
 * Estimates sigma, builds the Lloyd-Max codebook and the QR rotation on the
 * host, rotates/encodes on the device, trains IVF centroids (k-means, nlist>1)
 * and the Br-bit residual codebook (1-D k-means). x: host [n][d] float32. */
int jhq_train(jhq_index* idx, const float* x, int64_t n);

/* JHQGpuIndex::add(h_x, n) — jhq_gpu_index.cu:417-532. Unlike the reference
 * (single call only, :419-420) add may be called repeatedly (streaming add);
 * ids continue from the current ntotal. x: host [n][d] float32. */
int jhq_add(jhq_index* idx, const float* x, int64_t n);

/* JHQGpuIndex::search(h_q, nq, k, h_dists, h_labels) — jhq_gpu_index.cu:535-552
 * and search_gpu (search.cu:388-445). Host buffers; [nq][k] row-major outputs.
 * Distances carry the reference's +|q_rot|^2 offset (residual_encode corr,
 * encode.cu:85). Missing results are id -1, distance +inf (search.cu:285-286). */
int jhq_search(jhq_index* idx, const float* q, int64_t nq, int k,
               float* dists, int32_t* ids);

/* Same as jhq_search with DEVICE buffers on `stream` (cudaStream_t, NULL =
 * the index's stream); no host copies, asynchronous w.r.t. the host. */
int jhq_search_device(jhq_index* idx, const float* d_q, int64_t nq, int k,
                      float* d_dists, int32_t* d_ids, void* stream);

/* Same as jhq_search_device, but allocates nothing: every temporary of a
 * batch (rotated queries, coarse scores, probe lists, candidate lists) lives in
 * one fixed 16 MiB device array built into the library, which each GPU that
 * loads the library keeps until exit. For callers that may not allocate device
 * memory while serving (a host that owns a fixed pool, real-time paths, a
 * framework that reserved the whole GPU). No counterpart in the reference.
 * The first call on a device looks up that array (cudaGetSymbolAddress, once
 * per device for the life of the process); make it before any stream capture,
 * and do not use the library on that device after cudaDeviceReset. A batch
 * needing more than 16 MiB of temporaries returns JHQ_EINVAL. All calls on a device share the array, so
 * calls that overlap on the GPU race: serialise them. */
int jhq_search_device_noalloc(jhq_index* idx, const float* d_q, int64_t nq, int k,
                              float* d_dists, int32_t* d_ids, void* stream);

/* Device-side failure report for searches on the CALLER's stream
 * (jhq_search_device, jhq_search_device_noalloc, jhq_search_device_probes):
 * after that stream has drained, returns JHQ_ETIMEDOUT (and clears the flag)
 * if a bounded device wait of such a search gave up — its results are then
 * not valid — else JHQ_OK. jhq_search and jhq_synchronize check the same flag
 * themselves. No counterpart in the reference (its device errors exit). */
int jhq_device_status(jhq_index* idx);

/* Diagnostics (no counterpart in the reference): the approximate ADC scores
 * s~[q][v] the tensor-core flat scan computes for nq <= 128 host queries
 * (scores: [nq][ntotal] floats), so a checker can measure them against the
 * exact keys and the selection's error bound. JHQ_ESTATE when the index does
 * not use that scan (IVF, bits per dimension != 1, JHQ_FLAT=simt). */
int jhq_debug_flat_scores(jhq_index* idx, const float* q, int nq, float* scores);

/* Waits for the index's stream with a deadline (replaces the unbounded
 * cudaStreamQuery spin of search.cu:442-444). JHQ_ETIMEDOUT on expiry. */
int jhq_synchronize(jhq_index* idx, double timeout_s);

/* Split search for query-partitioned sharding: jhq_probe_device writes the
 * nprobe list ids of each query (rotation + coarse scores + exact top-nprobe,
 * search.cu:338-346 + select_probes_kernel) to d_probes [nq][nprobe];
 * jhq_search_device_probes then searches with those lists (so ranks can share
 * one rank's coarse work). No reference counterpart (single-GPU only). */
int jhq_probe_device(jhq_index* idx, const float* d_q, int64_t nq, int32_t* d_probes,
                     void* stream);
int jhq_search_device_probes(jhq_index* idx, const float* d_q, const int32_t* d_probes,
                             int64_t nq, int k, float* d_dists, int32_t* d_ids, void* stream);

/* Changes the number of probed lists of later searches (clamped to nlist,
 * like the constructor, jhq_gpu_index.cu:128). The reference fixes nprobe at
 * construction; this allows an nprobe sweep on one trained index. */
int jhq_set_nprobe(jhq_index* idx, int nprobe);

/* Candidate oversampling alpha (Params::alpha, ck = max(k, ceil(alpha k)),
 * search.cu:408) on a built index; alpha <= 0 -> JHQ_EINVAL. The reference
 * fixes alpha at construction; this allows an alpha sweep on one index. */
int jhq_set_alpha(jhq_index* idx, float alpha);

/* Exact rerank over stored vectors. The reference's JHQ indexes return the k
 * best refined JHQ distances; its hblock graph indexes keep the vectors and
 * rerank candidates by exact L2 (hblock_v34/jhq_gpu_index.cu:628-629,
 * hblock_v34/search.cu:531-690). With R > 0 this index keeps every added
 * vector (fp32, d*4 bytes each, from the next add() on, so enable it before
 * the first add), a search for k takes the best max(R, k) JHQ candidates
 * (ck = max(R', ceil(alpha R'))) and returns the k nearest of them by exact L2,
 * with the distance ||q - x||^2 (no offset). R = 0 restores the reference's
 * JHQ search. Errors: R outside [0, 256] or d % 4 != 0 -> JHQ_EINVAL; enabling
 * it on a non-empty index that keeps no vectors -> JHQ_ESTATE. */
int jhq_set_rerank(jhq_index* idx, int R);

/* Residual codebooks: per_subspace = 0 keeps the reference's single global
 * Kr-entry codebook (default); 1 trains M per-subspace codebooks (res_c1d
 * [M][Kr], dimension j coded against codebook j / Ds) — the ablation the
 * reference lists as its next step (README.md:66, "M per-subspace codebooks"),
 * not built there. Choose before jhq_train / jhq_set_trained; afterwards
 * JHQ_ESTATE. M * 2^Br must be <= 16384 (JHQ_EINVAL). With it, the res_c1d
 * buffers of jhq_get_trained / jhq_set_trained hold M * Kr floats. */
int jhq_set_residual_codebooks(jhq_index* idx, int per_subspace);
int jhq_get_residual_codebooks(const jhq_index* idx, int* per_subspace);

/* Out-of-core list paging (IVF only): pool_bytes > 0 keeps the index's codes
 * (pages, slot ids, residual codes, corr, and the kept vectors of the exact
 * rerank) in pinned host memory mapped into the device, and gives the device a
 * page pool of pool_bytes. Every search batch stages the pages of the lists it
 * probes into the pool (in waves of consecutive queries when they do not fit
 * together) and scans them there; results equal the resident index's. The
 * reference's counterpart is the bounded GPU region pool of its hblock_v39-v43
 * builds (hblock_v41/README.md). Enable before the first jhq_add (JHQ_ESTATE
 * otherwise); nlist = 1 or a pool smaller than one page -> JHQ_EINVAL; a search
 * whose single query's lists exceed the pool -> JHQ_EINVAL. Not combined with
 * jhq_search_device_noalloc / jhq_probe_device / jhq_search_device_probes
 * (JHQ_ESTATE). Saved files hold the codes; a loaded index is resident. */
int jhq_set_list_paging(jhq_index* idx, int64_t pool_bytes);
/* Waves the paged searches of this index have run so far (diagnostics). */
int jhq_paging_waves(const jhq_index* idx, int64_t* waves);
int jhq_get_rerank(const jhq_index* idx, int* R);

/* Accessors: JHQGpuIndex::ntotal() / dim() (jhq_gpu_index.cuh:44-45). */
int jhq_ntotal(const jhq_index* idx, int64_t* n);
int jhq_dim(const jhq_index* idx, int* d);
int jhq_is_trained(const jhq_index* idx, int* trained);
/* Vectors per IVF list, sizes[nlist] (the reference's list_offsets differences,
 * jhq_gpu_index.cu:475-495). */
int jhq_list_sizes(const jhq_index* idx, int64_t* sizes);

/* ---- trained artefacts (Pi, c1d, res_c1d, IVF centroids) -------------
 * The reference keeps these private (jhq_gpu_index.cuh:56-61). They are
 * exported/imported here so that two builds can run on identical training
 * (parity), and for persistence. Sizes: Pi d*d (column-major, as
 * cpu/jl_transform.h:24), c1d K1D = 2^(B/(d/M)), res_c1d 2^Br, cents nlist*d.
 * jhq_get_trained copies out (NULL pointers skipped); jhq_set_trained replaces
 * the index's training and requires an empty index. */
int jhq_get_trained(const jhq_index* idx, float* Pi, float* c1d, float* res_c1d,
                    float* cents, float* sigma);
int jhq_set_trained(jhq_index* idx, const float* Pi, const float* c1d,
                    const float* res_c1d, const float* cents, float sigma);

/* Codes of the stored vectors in id order: primary [n][M], residual
 * [n][ceil(d*Br/8)], corr [n], list assignment [n] (encode.cu:20-86,
 * jhq_gpu_index.cu:458-473). Any pointer may be NULL. */
int jhq_get_codes(const jhq_index* idx, uint8_t* primary, uint8_t* residual,
                  float* corr, int32_t* assign);

/* JL rotation y = Pi x of host rows (jhq_gpu_index.cu:209-225). */
int jhq_rotate(jhq_index* idx, const float* x, int64_t n, float* y);

/* The rotation search() applies to queries (search.cu:338-339). For indexes
 * whose batch_size is >= 1024 it is a tcgen05 GEMM on a bf16 three-term split
 * (x = hi + lo + r, |r| <= 2^-18 |x|; the products hi.hi, hi.lo, lo.hi
 * accumulated in fp32, so |error| <= 2^-16 |x| |Pi col| per output); smaller
 * batches use the exact fp32 chains of jhq_rotate (JHQ_ROTATE=simt|tc forces
 * either). Database rows (add/train) always use jhq_rotate's path. Exposed so
 * that a checker can search with the very same rotated queries. */
int jhq_rotate_queries(jhq_index* idx, const float* x, int64_t n, float* y);

/* Encode already-rotated host rows with the index's codebooks without adding
 * them (primary_encode_kernel + residual_encode_kernel, encode.cu:20-86). */
int jhq_encode(jhq_index* idx, const float* y, int64_t n, uint8_t* primary,
               uint8_t* residual, float* corr);

/* Serialise / restore trained artefacts and stored codes (versioned binary).
 * The reference has no persistence; every demo retrains (demo :78-86). */
int jhq_save(const jhq_index* idx, const char* path);
int jhq_load(const char* path, int device, jhq_index** out);

/* ---- sharded search (one process per GPU) ----------------------------
 * k-way merge of per-shard top-k lists on the device: in_dists/in_ids are
 * [nshards][nq][k] (device), out [nq][k] (device), order (distance, id),
 * missing entries (+inf, -1). Used after an all-gather of every shard's
 * jhq_search_device output. No reference counterpart (single-GPU only). */
int jhq_merge_shards(const float* d_in_dists, const int32_t* d_in_ids,
                     int nshards, int64_t nq, int k,
                     float* d_out_dists, int32_t* d_out_ids, void* stream);

/* ---- single-process sharded index ------------------------------------
 * The JHQGpuIndex call shape (jhq_gpu_index.cuh:38-47) over nshards shards
 * driven by one process: devices[s] is the GPU of shard s (NULL = 0..nshards-1;
 * ordinals may repeat to put several shards on one GPU). Global id g lives on
 * shard g % nshards. train() trains shard 0 and copies its artefacts to the
 * others; add() may be called repeatedly; search() splits the coarse step by
 * queries, scans every shard with the shared probe lists, and merges the
 * shards' top-k on the first shard's GPU (order (distance, id), missing
 * (+inf, -1)). Results equal searching each shard and merging with
 * jhq_merge_shards. No reference counterpart (the reference is single-GPU). */
typedef struct jhq_sharded jhq_sharded;
int jhq_sharded_create(int d, const jhq_params* p, int nshards, const int* devices,
                       jhq_sharded** out);
int jhq_sharded_destroy(jhq_sharded* idx);
int jhq_sharded_train(jhq_sharded* idx, const float* x, int64_t n_train);
int jhq_sharded_add(jhq_sharded* idx, const float* x, int64_t n);
int jhq_sharded_search(jhq_sharded* idx, const float* q, int64_t nq, int k, float* dists,
                       int32_t* ids);
int jhq_sharded_set_nprobe(jhq_sharded* idx, int nprobe);
int64_t jhq_sharded_ntotal(const jhq_sharded* idx);

/* ---- per-stage timing (the reference's jhq_v9_step_timing / v13 step
 * events, jhq_v13_step_timing/search.cu:456-491) -------------------------
 * With profiling on, search runs each batch as direct launches (no CUDA
 * graph) with CUDA events between the stages and accumulates per-stage device
 * time. Stages: 0 rotate, 1 coarse scores + probe selection, 2 scan plan,
 * 3 LUT + ADC scan + top-ck, 4 refine + final top-k. jhq_set_profiling resets
 * the totals; jhq_stage_times copies min(n, 5) totals (ms) and batch counts. */
#define JHQ_NUM_STAGES 5
int jhq_set_profiling(jhq_index* idx, int on);
int jhq_stage_times(const jhq_index* idx, double* ms, int64_t* batches, int n);

/* ---- host-side training primitives (no GPU needed) --------------------
 * The CPU steps of train(), exported so callers can reproduce or inspect them:
 *  jhq_jl_rotation      JLTransform(d, seed) -> Pi (cpu/jl_transform.cpp:21-56);
 *                       Householder QR in double, LAPACK sign convention.
 *  jhq_estimate_sigma   JLTransform::estimate_sigma (cpu/jl_transform.cpp:73-83).
 *  jhq_lloyd_max_c1d    LloydMaxCodebook codewords (cpu/codebook.cpp:60-80).
 *  jhq_kmeans_1d        train_1d_kmeans (cpu/codebook.cpp:8-58); *nout = count. */
int jhq_jl_rotation(int d, int seed, float* Pi);
int jhq_estimate_sigma(const float* x, int64_t n, int d, float* sigma);
int jhq_lloyd_max_c1d(float sigma, int K1D, float* c1d);
int jhq_kmeans_1d(const float* vals, int64_t n, int Kr, int max_iter, float* out, int* nout);

/* Per-call kernel launch counter of the calling process (all indexes), for
 * reporting how many engine kernels ran in a timed region. */
int64_t jhq_kernel_launches(void);

const char* jhq_last_error(void);
const char* jhq_version(void);

#ifdef __cplusplus
}
#endif
#endif /* JHQ_B200_H */
