/*
 * jhq_oracle.h — scalar CPU restatement of the JHQ search path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA product
 * (jhq_gpu_b200/csrc): only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs load it. The product never links it.
 *
 * Every function restates one step of the reference (lrlorry/JHQ_GPU) and
 * cites the file:line it follows. Where the reference leaves the floating-point
 * evaluation order to a library or a compiler (cuBLAS SGEMM, FMA contraction),
 * this file fixes one order; the CUDA kernels implement exactly the same order,
 * so the product is compared with this oracle bit for bit, and with the
 * reference's own cpu/ code (oracle/_ref) within a stated tolerance.
 *
 * Fixed arithmetic (the "spec" both sides follow):
 *  - rotation  y_j = fma-chain over c = 0..d-1 of P[c*d + j] * x_c, from 0;
 *    P is the reference's column-major Pi array (cpu/jl_transform.h:24).
 *  - byte LUT  LUT[m][b] = lo + hi, where lo/hi are fma-chains of
 *    (q_k - c1d[j_k])^2 over the dims whose bits sit in the low/high nibble of b
 *    (when bits_per_dim divides 4), otherwise one fma-chain over all Ds dims.
 *  - primary   dist = sequential float sum over m = 0..M-1 of LUT[m][code_m].
 *  - residual  32 "lanes": lane l owns 16-byte chunks c = l, l+32, ... of the
 *    residual code; within a chunk, dims in ascending order; lane partial =
 *    fma-chain of (q_j - r_hat)^2; then butterfly reduction p[l] += p[l ^ o]
 *    for o = 16, 8, 4, 2, 1.
 *  - composite comp = (primary + residual) + corr    (search.cu:240)
 *  - coarse    s_c = |c|^2 - 2 * (fma-chain dot(q_rot, c))  (search.cu:32)
 *  - ordering  top-nprobe by (s, list id); top-ck by (primary, id);
 *              top-k by (comp, id); missing results are (+inf, -1).
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- training restatements (cpu/) ------------------------------------ */
float oracle_sigma(const float* x, int64_t n, int d);                 /* cpu/jl_transform.cpp:73-83 */
float oracle_erfinv(float x);                                         /* cpu/erfinv.h:7-27 */
int   oracle_c1d(float sigma, int K1D, float* out);                   /* cpu/codebook.cpp:60-80 */
int   oracle_kmeans1d(const float* vals, int64_t n, int Kr, int max_iter, float* out); /* cpu/codebook.cpp:8-58 */
void  oracle_reconstruct(const uint8_t* codes, int64_t n, int d, int M, int B,
                         const float* c1d, float* out);               /* cpu/codebook.cpp:161-171 */

/* ---- encode (jhq_v14_streaming_add/encode.cu) ------------------------ */
void  oracle_rotate(const float* P, int d, const float* x, int64_t n, float* y);
void  oracle_encode_primary(const float* y, int64_t n, int d, int M, int B,
                            const float* c1d, uint8_t* codes);        /* encode.cu:20-41 */
void  oracle_encode_residual(const float* y, const uint8_t* codes, int64_t n,
                             int d, int M, int B, const float* c1d,
                             const float* res_c1d, int Br,
                             uint8_t* res_codes, float* corr);        /* encode.cu:43-86 */

/* ---- IVF (jhq_v14_streaming_add/jhq_gpu_index.cu) -------------------- */
void  oracle_cent_norms(const float* cents, int nlist, int d, float* norms); /* jhq_gpu_index.cu:243-249 */
void  oracle_assign(const float* y, int64_t n, int d, const float* cents,
                    const float* norms, int nlist, int32_t* assign);  /* jhq_gpu_index.cu:23-39 */
void  oracle_train_ivf(const float* y, int64_t n, int d, int nlist, int iters,
                       float* cents);                                 /* jhq_gpu_index.cu:228-299 */

/* ---- search (jhq_v14_streaming_add/search.cu, jhq_v3_ivf/search.cu) --- */
void  oracle_byte_lut(const float* q_rot, int d, int M, int B, const float* c1d, float* lut);
float oracle_adc(const float* lut, int M, const uint8_t* code);
float oracle_residual(const float* q_rot, int d, int Br, const float* res_c1d,
                      const uint8_t* res_code);
int   oracle_ck(int k, float alpha);                                  /* search.cu:408 */

/* Full search over an index held in id order.
 * codes [n][M], res [n][bpv], corr [n], assign [n] (list id per vector).
 * q_rot are ALREADY rotated queries [nq][d]. Outputs [nq][k].
 * Returns 0, or nonzero on a bad argument. */
int   oracle_search(const float* q_rot, int64_t nq, int d, int M, int B, int Br,
                    const float* c1d, const float* res_c1d,
                    const uint8_t* codes, const uint8_t* res, const float* corr,
                    const int32_t* assign, int64_t n,
                    const float* cents, const float* norms, int nlist, int nprobe,
                    int k, float alpha, int nthreads,
                    float* out_dists, int32_t* out_ids);

/* Per-subspace residual codebooks (per_sub != 0): res_c1d is [M][Kr] and dim j
 * uses codebook j / Ds; per_sub = 0 is the functions above (one codebook). */
void  oracle_encode_residual_ps(const float* y, const uint8_t* codes, int64_t n, int d, int M,
                                int B, const float* c1d, const float* res_c1d, int Br,
                                int per_sub, uint8_t* res_codes, float* corr);
float oracle_residual_ps(const float* q_rot, int d, int Ds, int Br, const float* res_c1d,
                         int per_sub, const uint8_t* res_code);
int   oracle_search_ps(const float* q_rot, int64_t nq, int d, int M, int B, int Br,
                       const float* c1d, const float* res_c1d, int per_sub,
                       const uint8_t* codes, const uint8_t* res, const float* corr,
                       const int32_t* assign, int64_t n,
                       const float* cents, const float* norms, int nlist, int nprobe,
                       int k, float alpha, int nthreads,
                       float* out_dists, int32_t* out_ids);

/* Exact rerank (stored vectors): q [nq][d] and x [n][d] as given, cand [nq][kr]
 * JHQ candidate ids (-1 = none). Outputs [nq][k]. Returns nonzero on bad args. */
int   oracle_rerank(const float* q, int64_t nq, int d, const float* x, int64_t n,
                    const int32_t* cand, int kr, int k, float* out_dists, int32_t* out_ids);

#ifdef __cplusplus
}
#endif
