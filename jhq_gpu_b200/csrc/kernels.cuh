// kernels.cuh — launch wrappers of the JHQ B200 engine's CUDA kernels.
// All wrappers are asynchronous on `stream`, count their launches (for the
// jhq_kernel_launches() report) and throw jhq::Error on a launch failure.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <vector>

namespace jhq {

extern std::atomic<int64_t> g_kernel_launches;
inline void count_launch(int n = 1) { g_kernel_launches.fetch_add(n, std::memory_order_relaxed); }

// ---- dense fp32 products (gemm.cu) --------------------------------------
// C[r][n] = epi( sum_{k=0..K-1} A[r*K + k] * B[k*N + n] ), each output an
// in-order fma chain over k. epi = identity, or norms[n] - 2*x (coarse).
enum GemmEpi { EPI_STORE = 0, EPI_COARSE = 1 };
void gemm_rows(const float* A, const float* B, float* C, int64_t R, int K, int N,
               GemmEpi epi, const float* norms, cudaStream_t s);

// out[r] = argmin_n (norms[n] - 2 * sum_k A[r*K+k] B[k*N+n]), first minimum,
// each dot an in-order fma chain; the scores are never stored.
void gemm_argmin(const float* A, const float* B, const float* norms, int64_t R, int K, int N,
                 int32_t* out, cudaStream_t s);

// ---- encode / IVF build (encode.cu) --------------------------------------
// Primary + residual codes and corr of rotated rows y [n][d]
// (encode.cu:20-86 of the reference). res rows are bpv_pad bytes apart.
void encode_rows(const float* y, int64_t n, int d, int M, int B, int Br,
                 const float* c1d, const float* res_c1d, bool res_per_sub, uint8_t* pcodes,
                 uint8_t* rcodes, int bpv_pad, float* corr, cudaStream_t s);
// pop[v] = number of set bits of code row v ([n][M] bytes)
void popcount_rows(const uint8_t* codes, int64_t n, int M, int32_t* pop, cudaStream_t s);
// v[i] *= f (f a power of two here, so exact)
void scale_floats(float* v, int64_t n, float f, cudaStream_t s);
// dst[0] = value (stream-ordered scalar upload, no host buffer involved).
void set_int(int* dst, int value, cudaStream_t s);
// Scatter codes into the page layout: slot_ids [npages*32] (-1 = empty slot),
// pcodes [N][M] id-ordered -> pages [npages][Mp/16][32][16].
void scatter_pages(const int32_t* slot_ids, int64_t nslots, const uint8_t* pcodes,
                   int M, int Mp, uint8_t* pages, cudaStream_t s);

// ---- probe selection + scan partition (ivf.cu) ----------------------------
// Per query: the nprobe lists of smallest (s, list id) from s [nq][nlist],
// written ascending into probes [nq][nprobe].
void select_probes(const float* s, int nq, int nlist, int nprobe, int32_t* probes,
                   cudaStream_t st);
// Same lists from APPROXIMATE scores s~ (coarse_scores_tc): the lists within
// a proven error margin of the nprobe-th s~ are rescored with the exact fp32
// chain (cents [nlist][d] row-major, q_rot [nq][d]); cmax >= max |c|. The row
// of s may be overwritten. d <= 2048.
// tile_min (optional, [nq][ntiles]): minima of s~ over disjoint groups of lists.
void select_probes_margin(float* s, const float* q_rot, const float* cents, const float* norms,
                          const float* tile_min, int ntiles, int nq, int nlist, int d, int nprobe,
                          float cmax, int32_t* probes, cudaStream_t st);

// ---- tensor-core coarse scores (coarse_tc.cu) ------------------------------
// s~[q][c] = norms[c] - 2 * (q3[q] . c3[c]) with tcgen05 kind::f16 (bf16
// operands, fp32 accumulation) over K3 = coarse_tc_k3(d) >= 3d, where
// q3 = [q_hi | q_hi | q_lo] (split3_rows, order 0) and c3 = [c_hi | c_lo | c_hi]
// (order 1); hi = bf16(x), lo = bf16(x - hi), round to nearest even, zero pad.
// Approximate: see select_probes_margin.
bool coarse_tc_supported(int d, int nlist);
int coarse_tc_k3(int d);
void split3_rows(const float* x, int64_t n, int d, uint16_t* out, cudaStream_t s);   // order 0
void split3_rows_host(const float* x, int64_t n, int d, int order, uint16_t* out);
// Also tile_min[q][t] = min over lists [128t, 128t+128) of s~[q][.], t < coarse_tc_tiles.
constexpr int COARSE_TILE_LISTS = 128;
int coarse_tc_tiles(int nlist);
void coarse_scores_tc(const uint16_t* q3, int nq, const uint16_t* c3, const float* norms,
                      int nlist, int d, float* scores, float* tile_min, cudaStream_t s);
// Nonzero once a bounded wait inside the kernel gave up (cleared if `clear`).
int coarse_tc_error(bool clear);

// ---- scan plan (ivf.cu): list-major work units over query groups ----------
// The (query, probe) pairs of a batch are inverted into per-list buckets; the
// queries of list l are taken QG at a time and each list is cut into chunks of
// at most chunk_pages pages. A unit = (list, query group, chunk); units are
// numbered list-major then group-major then chunk. Every (query, probe, chunk)
// gets its own candidate slot: slot = qslot_off[q] + cpo[q][p] + chunk.
struct PlanBufs {
    int32_t* cnt;          // [nlist + 1]  pairs per list (zeroed by plan_build)
    int32_t* bucket_off;   // [nlist + 1]
    int32_t* unit_off;     // [nlist + 1]
    int32_t* fill;         // [nlist]
    int2* bucket;          // [nq * nprobe]  (query, probe index)
    int32_t* cpo;          // [nq][nprobe + 1]  chunk prefix over a query's probes
    int64_t* qslot_off;    // [nq + 1]
    uint64_t* gthr;        // [nq]  global pruning bound per query
};
// Queries >= *d_nvalid (when given) take part in nothing.
// Query-major variant (small lists): a work item = (query, up to item_pages
// consecutive pages of its probe sequence); cpo[q][p] = pages before probe p,
// qslot_off = item offsets (one slot per item). cnt/bucket/unit/fill unused.
void plan_build_qmajor(const int32_t* probes, int nq, int nprobe, const int32_t* list_page_off,
                       const int* d_nvalid, int item_pages, const PlanBufs& b, cudaStream_t st);
void plan_build(const int32_t* probes, int nq, int nprobe, int nlist,
                const int32_t* list_page_off, const int* d_nvalid, int chunk_pages, int qg,
                const PlanBufs& b, cudaStream_t st);

// ---- pilot bound of a flat index (pilot.cu) --------------------------------
// Per query q < *d_nvalid: gthr[q] = min(gthr[q], ck-th smallest ADC key of
// the members of the nearest pilot cluster + 1), keys computed exactly as the
// scan computes them (nibble tables; bits_per_dim in {1, 2, 4}).
constexpr int PILOT_SPLIT = 8;             // CTAs per query scoring members
constexpr int PILOT_CHUNK = 512;           // members per CTA (the rest are left out)
struct PilotArgs {
    const float* q_rot;            // [nq][d]
    const float* c1d;              // [K1D]
    const float* pcents;           // [P][d]
    const float* pnorms;           // [P]
    const int32_t* pilot_off;      // [P+1]
    const int32_t* pilot_ids;      // members grouped by cluster
    const uint8_t* pcodes;         // [N][M] primary codes, id order
    float* pscores;                // scratch [nq][P]
    uint64_t* pkeys;               // scratch [nq][PILOT_SPLIT][ck]
    uint64_t* gthr;                // [nq]
    const int* d_nvalid;
    int nq, d, M, B, P, ck;
};
size_t pilot_smem_bytes(int M, int d);
void pilot_bound(const PilotArgs& a, cudaStream_t st);

// ---- LUT + ADC scan + exact top-ck (scan.cu) -------------------------------
struct ScanArgs {
    const float* q_rot;            // [nq][d]
    const float* c1d;              // [K1D]
    const int32_t* list_page_off;  // [nlist+1]
    const uint8_t* pages;          // [npages][Mp/16][32][16]
    const int32_t* slot_ids;       // [npages*32]
    const int32_t* unit_off;       // plan
    const int32_t* bucket_off;
    const int2* bucket;
    const int32_t* cpo;
    const int64_t* qslot_off;
    uint64_t* gthr;                // [nq] lowered by the scan
    uint64_t* cand;                // [slots][ck] output candidate keys
    const int32_t* probes;         // [nq][nprobe] (query-major order)
    int nq, nlist, d, M, Mp, B, nprobe, ck, ck_pad, grid, chunk_pages, mode;
    int qmajor;                    // 1: query-major warp items (chunk_pages = item pages)
    int prune = 0;                 // 1: exit a page early once every slot is above its bound
};
// mode 0: byte LUT, one query per unit; 1/2/4: nibble tables, 1/2/4 queries.
int scan_mode_for(int d, int M, int B, double queries_per_list);
size_t scan_smem_bytes(int Mp, int d, int ck_pad, int mode);  // dynamic shared memory per CTA
int scan_grid_for(int Mp, int d, int ck_pad, int mode);       // persistent CTAs: SMs x resident
int scan_qmajor_grid_for(int Mp, int ck_pad);
size_t scan_qmajor_smem_bytes(int Mp, int ck_pad);
void scan_topck(const ScanArgs& a, cudaStream_t st);
void scan_configure();                               // opt-in shared memory, current device

// ---- IVF ADC scan on the tensor cores, 2 bits per dimension (coarse_tc.cu) -
struct IvfTcArgs {
    const float* q_rot;            // [nq][d]
    const float* c1d;              // [4] on the device
    const float* c1d_host;         // [4] on the host
    const int32_t* probes;         // [nq][nprobe]
    const int32_t* list_page_off;  // [nlist+1]
    const uint8_t* pages;          // [npages][Mp/16][32][16]
    const int32_t* slot_ids;       // [npages*32]
    PlanBufs plan;                 // list-major plan buffers (rebuilt here; qslot_off unused)
    void* scratch;                 // ivf_tc_scratch_bytes(nq, max_tiles)
    int64_t max_tiles;             // bound on the batch's (query, probed tile) pairs
    int nq, nprobe, nlist, d, M, ck, ck_pad;
    uint64_t* cand;                // [nq][ck] out: the exact top-ck, one slot per query
    uint64_t* gthr;                // [nq] out: the ck-th key
    int64_t* qslot_out;            // [nq+1] out: q
    const int* d_nvalid = nullptr; // device count of valid rows (rest: no candidates)
};
bool ivf_tc_supported(int d, int M, int B, int nprobe);
size_t ivf_tc_scratch_bytes(int Bq, int64_t max_tiles);
void ivf_search_tc(const IvfTcArgs& a, cudaStream_t s);

// ---- merge + residual refine + final top-k (refine.cu) --------------------
struct RefineArgs {
    const float* q_rot;        // [nq][d]
    const float* res_c1d;      // [Kr]
    const uint64_t* cand;      // scan output
    const int64_t* qslot_off;  // [nq+1] slots of each query
    const uint64_t* gthr;      // [nq] final pruning bound per query
    const uint8_t* rcodes;     // [N][bpv_pad] id order
    const float* corr;         // [N]
    float* out_dists;          // [nq][k]
    int32_t* out_ids;          // [nq][k]
    // exact rerank (optional): the kr best composite candidates are re-scored
    // by exact L2 against the stored vectors raw [N][d] and the k best returned
    const float* q_raw = nullptr;   // [nq][d] the queries as given
    const float* raw = nullptr;     // [N][d] stored vectors, nullptr = no rerank
    int nq, d, Br, bpv_pad, ck, ck_pad, k;
    int kr = 0;                     // candidates re-scored (k <= kr <= ck)
    int res_per_sub = 0;            // res_c1d is [M][Kr] (dim j: codebook j / (d / M))
    int M = 1;
};
void refine_topk(const RefineArgs& a, cudaStream_t st);
void refine_configure();

// ids[i] >= 0 -> ids[i] * mul + add (local -> global ids of a round-robin shard).
void remap_ids(int32_t* ids, int64_t n, int mul, int add, cudaStream_t st);

// k-way merge of per-shard top-k lists (jhq_merge_shards).
void merge_shard_lists(const float* in_d, const int32_t* in_i, int nshards, int64_t nq,
                       int k, float* out_d, int32_t* out_i, cudaStream_t st);

// ---- flat ADC scan on the tensor cores, 1-bit codes (coarse_tc.cu) ----------
struct FlatTcArgs {
    const float* q_rot;          // [nq][d]
    const float* c1d;            // [2] on the device
    const float* c1d_host;       // [2] on the host
    const uint8_t* codes;        // [nvec][M] primary codes, id order
    const int32_t* pop;          // [nvec] popcount of each code row
    int nvec, M, nq, ck, ck_pad;
    void* scratch;               // flat_tc_scratch_bytes(nq, d, nvec)
    uint64_t* cand;              // [nq][ck] out: the exact top-ck, one slot per query
    uint64_t* gthr;              // [nq] out: the ck-th key
    int64_t* qslot_off;          // [nq+1] out: q
    const int* d_nvalid = nullptr;   // device count of valid rows (rest: no candidates)
    bool scores_only = false;    // stop after the GEMM (diagnostics)
};
// the approximate scores [nq][nvec] inside a flat_search_tc scratch block
float* flat_tc_scores_of(void* scratch, int Bq, int d, int nvec);
bool flat_tc_supported(int d, int M, int B, int nvec);
size_t flat_tc_scratch_bytes(int Bq, int d, int nvec);
void flat_search_tc(const FlatTcArgs& a, cudaStream_t s);

// ---- training on the device (train_gpu.cu), bit-identical to train_cpu.cpp ----
// y <- y - c1d[bits of the primary code], in place ([n][d])
void residuals_device(float* d_y, const uint8_t* d_codes, int64_t n, int d, int M, int B,
                      const float* d_c1d, cudaStream_t s);
// 1-D k-means of n device values (train::kmeans_1d on the device)
std::vector<float> kmeans_1d_device(const float* d_vals, int64_t n, int Kr, int max_iter,
                                    cudaStream_t s);
// one Lloyd mean update: d_cents [nl][d] <- means of the rows of d_y assigned to
// each list (index-order double sums); lists with no rows keep their value and
// are reported with count 0
void lloyd_update_device(const float* d_y, int64_t n, int d, int nl, const int32_t* d_assign,
                         float* d_cents, std::vector<int64_t>& counts, cudaStream_t s);

}  // namespace jhq
