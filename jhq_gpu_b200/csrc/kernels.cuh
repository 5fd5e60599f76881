// kernels.cuh — launch wrappers of the JHQ B200 engine's CUDA kernels.
// All wrappers are asynchronous on `stream`, count their launches (for the
// jhq_kernel_launches() report) and throw jhq::Error on a launch failure.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace jhq {

extern std::atomic<int64_t> g_kernel_launches;
inline void count_launch(int n = 1) { g_kernel_launches.fetch_add(n, std::memory_order_relaxed); }

// ---- dense fp32 products (gemm.cu) --------------------------------------
// C[r][n] = epi( sum_{k=0..K-1} A[r*K + k] * B[k*N + n] ), each output an
// in-order fma chain over k. epi = identity, or norms[n] - 2*x (coarse).
enum GemmEpi { EPI_STORE = 0, EPI_COARSE = 1 };
void gemm_rows(const float* A, const float* B, float* C, int64_t R, int K, int N,
               GemmEpi epi, const float* norms, cudaStream_t s);

// ---- encode / IVF build (encode.cu) --------------------------------------
// Primary + residual codes and corr of rotated rows y [n][d]
// (encode.cu:20-86 of the reference). res rows are bpv_pad bytes apart.
void encode_rows(const float* y, int64_t n, int d, int M, int B, int Br,
                 const float* c1d, const float* res_c1d, uint8_t* pcodes,
                 uint8_t* rcodes, int bpv_pad, float* corr, cudaStream_t s);
// dst[0] = value (stream-ordered scalar upload, no host buffer involved).
void set_int(int* dst, int value, cudaStream_t s);
// argmin over each row of s [n][nlist] (first minimum) -> assign [n].
void argmin_rows(const float* s, int64_t n, int nlist, int32_t* assign, cudaStream_t st);
// Scatter codes into the page layout: slot_ids [npages*32] (-1 = empty slot),
// pcodes [N][M] id-ordered -> pages [npages][Mp/16][32][16].
void scatter_pages(const int32_t* slot_ids, int64_t nslots, const uint8_t* pcodes,
                   int M, int Mp, uint8_t* pages, cudaStream_t s);

// ---- probe selection + scan partition (ivf.cu) ----------------------------
// Per query: the nprobe lists of smallest (s, list id) from s [nq][nlist],
// written ascending into probes [nq][nprobe].
void select_probes(const float* s, int nq, int nlist, int nprobe, int32_t* probes,
                   cudaStream_t st);
// Page counts per (query, probe) -> qpage_off [nq+1] (exclusive scan over
// queries) and probe_page_off [nq][nprobe+1]; queries >= *d_nvalid get 0 pages.
void scan_prepare(const int32_t* probes, int nq, int nprobe, const int32_t* list_page_off,
                  const int* d_nvalid, int32_t* probe_page_off, int64_t* qpage_off,
                  cudaStream_t st);

// ---- LUT + ADC scan + exact top-ck (scan.cu) -------------------------------
struct ScanArgs {
    const float* q_rot;            // [nq][d]
    const float* c1d;              // [K1D]
    const int32_t* probes;         // [nq][nprobe]
    const int32_t* probe_page_off; // [nq][nprobe+1]
    const int64_t* qpage_off;      // [nq+1]
    const int32_t* list_page_off;  // [nlist+1]
    const uint8_t* pages;          // [npages][Mp/16][32][16]
    const int32_t* slot_ids;       // [npages*32]
    uint64_t* cand;                // [(grid + nq) * ck] output candidate keys
    int nq, d, M, Mp, B, nprobe, ck, ck_pad, grid;
};
bool scan_uses_nibbles(int d, int M, int B);        // nibble tables instead of the byte LUT
size_t scan_smem_bytes(int Mp, int d, int ck_pad, bool nib);  // dynamic shared memory per CTA
int scan_grid_for(int Mp, int d, int ck_pad, bool nib);       // persistent CTAs: SMs x resident CTAs
void scan_topck(const ScanArgs& a, cudaStream_t st);
void scan_configure();                               // opt-in shared memory, current device

// ---- merge + residual refine + final top-k (refine.cu) --------------------
struct RefineArgs {
    const float* q_rot;        // [nq][d]
    const float* res_c1d;      // [Kr]
    const uint64_t* cand;      // scan output
    const int64_t* qpage_off;  // [nq+1]
    const uint8_t* rcodes;     // [N][bpv_pad] id order
    const float* corr;         // [N]
    float* out_dists;          // [nq][k]
    int32_t* out_ids;          // [nq][k]
    int nq, d, Br, bpv_pad, ck, ck_pad, k, grid;
};
void refine_topk(const RefineArgs& a, cudaStream_t st);
void refine_configure();

// k-way merge of per-shard top-k lists (jhq_merge_shards).
void merge_shard_lists(const float* in_d, const int32_t* in_i, int nshards, int64_t nq,
                       int k, float* out_d, int32_t* out_i, cudaStream_t st);

}  // namespace jhq
