/*
 * jhq_oracle.c — scalar CPU restatement of the JHQ path (test infrastructure).
 * See jhq_oracle.h for the fixed arithmetic both this file and the CUDA
 * product follow. Built by oracle/Makefile with -ffp-contract=off so that
 * every fused multiply-add here is an explicit fmaf() and nothing else fuses.
 */
#include "jhq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------------- */
/* training restatements                                                   */
/* ---------------------------------------------------------------------- */

/* cpu/jl_transform.cpp:73-83 — sigma = sqrt(sum x^2 / (n d)), double accumulate. */
float oracle_sigma(const float* x, int64_t n, int d) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const float* xi = x + i * d;
        for (int j = 0; j < d; ++j) s += (double)xi[j] * xi[j];
    }
    return (float)sqrt(s / ((double)n * d));
}

/* cpu/erfinv.h:7-27 — Winitzki (2008) approximation (a = 0.147) followed by
 * one Newton step on erf(z) - x, all in float. */
float oracle_erfinv(float x) {
    if (x >= 1.0f) return INFINITY;
    if (x <= -1.0f) return -INFINITY;
    if (x == 0.0f) return 0.0f;
    const float sign = (x > 0.0f) ? 1.0f : -1.0f;
    const float a = fabsf(x);
    const float kC = 0.147f;
    const float k2Pi = 2.0f / 3.14159265358979f;
    const float ln1 = logf(1.0f - a * a);
    const float t = k2Pi / kC + 0.5f * ln1;
    float z = sign * sqrtf(sqrtf(t * t - ln1 / kC) - t);
    const float err = erff(z) - x;
    const float der = (2.0f / sqrtf((float)M_PI)) * expf(-z * z);
    z -= err / der;
    return z;
}

/* cpu/codebook.cpp:72-78 — c_i = sigma * sqrt(2) * erfinv(2 (i + .5)/K1D - 1). */
int oracle_c1d(float sigma, int K1D, float* out) {
    for (int i = 0; i < K1D; ++i) {
        float q = ((float)i + 0.5f) / (float)K1D;
        out[i] = sigma * (float)M_SQRT2 * oracle_erfinv(2.0f * q - 1.0f);
    }
    return K1D;
}

static int cmp_float(const void* a, const void* b) {
    float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

/* midpoint binary search shared by 1-D k-means and nearest_1d
 * (cpu/codebook.cpp:31-37, :82-94; encode.cu:6-18): ties go up. */
static inline int nearest_sorted(const float* c, int n, float v) {
    if (n == 1) return 0;
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = (lo + hi) / 2;
        if (v < 0.5f * (c[mid] + c[mid + 1])) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

/* cpu/codebook.cpp:8-58 — quantile init, <= max_iter Lloyd rounds. */
int oracle_kmeans1d(const float* vals, int64_t n64, int Kr, int max_iter, float* out) {
    int n = (int)n64;
    if (n <= 0 || Kr <= 0) return 0;
    if (n < Kr) Kr = n;
    float* sorted = (float*)malloc(sizeof(float) * (size_t)n);
    memcpy(sorted, vals, sizeof(float) * (size_t)n);
    qsort(sorted, (size_t)n, sizeof(float), cmp_float);
    float* c = out;
    for (int i = 0; i < Kr; ++i) {
        int idx = (int)(((float)i + 0.5f) / (float)Kr * (float)n);
        if (idx > n - 1) idx = n - 1;
        c[i] = sorted[idx];
    }
    double* sum = (double*)malloc(sizeof(double) * Kr);
    int* cnt = (int*)malloc(sizeof(int) * Kr);
    for (int iter = 0; iter < max_iter; ++iter) {
        for (int i = 0; i < Kr; ++i) { sum[i] = 0.0; cnt[i] = 0; }
        for (int i = 0; i < n; ++i) {
            int lo = nearest_sorted(c, Kr, vals[i]);
            sum[lo] += vals[i];
            cnt[lo]++;
        }
        int changed = 0;
        for (int i = 0; i < Kr; ++i) {
            float nc;
            if (cnt[i] == 0) {
                int idx = (int)(((float)i + 0.5f) / (float)Kr * (float)n);
                if (idx > n - 1) idx = n - 1;
                nc = sorted[idx];
            } else {
                nc = (float)(sum[i] / cnt[i]);
            }
            if (nc != c[i]) { c[i] = nc; changed = 1; }
        }
        qsort(c, (size_t)Kr, sizeof(float), cmp_float);
        if (!changed) break;
    }
    free(sum); free(cnt); free(sorted);
    return Kr;
}

/* cpu/codebook.cpp:161-171 */
void oracle_reconstruct(const uint8_t* codes, int64_t n, int d, int M, int B,
                        const float* c1d, float* out) {
    int Ds = d / M, bpd = B / Ds, mask = (1 << bpd) - 1;
    for (int64_t i = 0; i < n; ++i)
        for (int m = 0; m < M; ++m) {
            uint8_t cm = codes[i * M + m];
            for (int k = 0; k < Ds; ++k)
                out[i * d + m * Ds + k] = c1d[(cm >> (k * bpd)) & mask];
        }
}

/* ---------------------------------------------------------------------- */
/* encode                                                                  */
/* ---------------------------------------------------------------------- */

/* y = Pi x (cpu/jl_transform.cpp:58-70; jhq_gpu_index.cu:444-448),
 * evaluated as a sequential fma chain over c. */
void oracle_rotate(const float* P, int d, const float* x, int64_t n, float* y) {
    /* c-outer loop with one accumulator per output j: every y_j is still the
       in-order chain over c, but rows of P are read contiguously. */
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float* xi = x + i * d;
        float* yi = y + i * d;
        for (int j = 0; j < d; ++j) yi[j] = 0.0f;
        for (int c = 0; c < d; ++c) {
            const float xc = xi[c];
            const float* pc = P + (size_t)c * d;
            for (int j = 0; j < d; ++j) yi[j] = fmaf(pc[j], xc, yi[j]);
        }
    }
}

/* encode.cu:20-41 / cpu/codebook.cpp:96-110 */
void oracle_encode_primary(const float* y, int64_t n, int d, int M, int B,
                           const float* c1d, uint8_t* codes) {
    int Ds = d / M, bpd = B / Ds, K1D = 1 << bpd;
    for (int64_t i = 0; i < n; ++i)
        for (int m = 0; m < M; ++m) {
            const float* ym = y + i * d + m * Ds;
            unsigned cm = 0;
            for (int k = 0; k < Ds; ++k) cm |= (unsigned)nearest_sorted(c1d, K1D, ym[k]) << (k * bpd);
            codes[i * M + m] = (uint8_t)cm;
        }
}

/* encode.cu:43-86 — residual scalar code (Br = 4: even dim in the low nibble)
 * and corr = 2 * fma-chain sum of yhat_j * rhat_j. */
void oracle_encode_residual(const float* y, const uint8_t* codes, int64_t n,
                            int d, int M, int B, const float* c1d,
                            const float* res_c1d, int Br,
                            uint8_t* res_codes, float* corr) {
    oracle_encode_residual_ps(y, codes, n, d, M, B, c1d, res_c1d, Br, 0, res_codes, corr);
}

/* Per-subspace residual codebooks (per_sub != 0): dim j is coded against
 * codebook m = j / Ds, res_c1d[m * Kr .. m * Kr + Kr); one global codebook
 * otherwise (the reference's format). */
void oracle_encode_residual_ps(const float* y, const uint8_t* codes, int64_t n,
                               int d, int M, int B, const float* c1d,
                               const float* res_c1d_all, int Br, int per_sub,
                               uint8_t* res_codes, float* corr) {
    int Ds = d / M, bpd = B / Ds, kmask = (1 << bpd) - 1, Kr = 1 << Br;
    int bpv = (d * Br + 7) / 8;
    for (int64_t i = 0; i < n; ++i) {
        const float* yi = y + i * d;
        const uint8_t* pc = codes + i * M;
        uint8_t* rc = res_codes + i * bpv;
        memset(rc, 0, (size_t)bpv);
        float dot = 0.0f;
        for (int j = 0; j < d; ++j) {
            int m = j / Ds, k = j % Ds;
            float yh = c1d[(pc[m] >> (k * bpd)) & kmask];
            float r = yi[j] - yh;
            const float* res_c1d = res_c1d_all + (per_sub ? (size_t)m * Kr : 0);
            int ri = nearest_sorted(res_c1d, Kr, r);
            if (Br == 4) {
                if ((j & 1) == 0) rc[j / 2] = (uint8_t)(ri & 0x0F);
                else rc[j / 2] |= (uint8_t)((ri & 0x0F) << 4);
            } else {
                rc[j] = (uint8_t)ri;
            }
            dot = fmaf(yh, res_c1d[ri], dot);
        }
        corr[i] = 2.0f * dot;
    }
}

/* ---------------------------------------------------------------------- */
/* IVF                                                                     */
/* ---------------------------------------------------------------------- */

static inline float dot_chain(const float* a, const float* b, int d) {
    float acc = 0.0f;
    for (int j = 0; j < d; ++j) acc = fmaf(a[j], b[j], acc);
    return acc;
}

/* jhq_gpu_index.cu:243-249 — |c|^2 in double, stored as float. */
void oracle_cent_norms(const float* cents, int nlist, int d, float* norms) {
    for (int c = 0; c < nlist; ++c) {
        double s = 0.0;
        for (int j = 0; j < d; ++j) s += (double)cents[(size_t)c * d + j] * cents[(size_t)c * d + j];
        norms[c] = (float)s;
    }
}

/* jhq_gpu_index.cu:23-39 — argmin_c |c|^2 - 2 <y, c>, first minimum wins. */
void oracle_assign(const float* y, int64_t n, int d, const float* cents,
                   const float* norms, int nlist, int32_t* assign) {
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float* yi = y + i * d;
        float best = norms[0] - 2.0f * dot_chain(yi, cents, d);
        int bi = 0;
        for (int c = 1; c < nlist; ++c) {
            float s = norms[c] - 2.0f * dot_chain(yi, cents + (size_t)c * d, d);
            if (s < best) { best = s; bi = c; }
        }
        assign[i] = bi;
    }
}

/* jhq_gpu_index.cu:228-299 — Lloyd k-means in the rotated space. */
void oracle_train_ivf(const float* y, int64_t n, int d, int nlist, int iters, float* cents) {
    for (int c = 0; c < nlist; ++c) {
        int64_t src = (int64_t)c * n / nlist;
        memcpy(cents + (size_t)c * d, y + src * d, sizeof(float) * (size_t)d);
    }
    float* norms = (float*)malloc(sizeof(float) * nlist);
    int32_t* as = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
    double* sums = (double*)malloc(sizeof(double) * (size_t)nlist * d);
    int* counts = (int*)malloc(sizeof(int) * nlist);
    for (int iter = 0; iter < iters; ++iter) {
        oracle_cent_norms(cents, nlist, d, norms);
        oracle_assign(y, n, d, cents, norms, nlist, as);
        memset(sums, 0, sizeof(double) * (size_t)nlist * d);
        memset(counts, 0, sizeof(int) * nlist);
        for (int64_t i = 0; i < n; ++i) {
            int c = as[i];
            counts[c]++;
            double* sc = sums + (size_t)c * d;
            for (int j = 0; j < d; ++j) sc[j] += y[i * d + j];
        }
        for (int c = 0; c < nlist; ++c) {
            float* cc = cents + (size_t)c * d;
            if (counts[c] == 0) {
                int64_t src = ((int64_t)c * 1103515245 + (int64_t)(iter * 12345)) % n;
                memcpy(cc, y + src * d, sizeof(float) * (size_t)d);
                continue;
            }
            double inv = 1.0 / (double)counts[c];
            for (int j = 0; j < d; ++j) cc[j] = (float)(sums[(size_t)c * d + j] * inv);
        }
    }
    free(norms); free(as); free(sums); free(counts);
}

/* ---------------------------------------------------------------------- */
/* search                                                                  */
/* ---------------------------------------------------------------------- */

/* byte LUT (search.cu:65-91, cpu/codebook.cpp:112-129), nibble-split order. */
void oracle_byte_lut(const float* q_rot, int d, int M, int B, const float* c1d, float* lut) {
    int Ds = d / M, bpd = B / Ds, kmask = (1 << bpd) - 1;
    int split = (bpd <= 4) && (4 % bpd == 0);
    for (int m = 0; m < M; ++m) {
        const float* qm = q_rot + m * Ds;
        for (int b = 0; b < 256; ++b) {
            float lo = 0.0f, hi = 0.0f;
            for (int k = 0; k < Ds; ++k) {
                float diff = qm[k] - c1d[(b >> (k * bpd)) & kmask];
                if (!split || k * bpd < 4) lo = fmaf(diff, diff, lo);
                else hi = fmaf(diff, diff, hi);
            }
            lut[m * 256 + b] = split ? lo + hi : lo;
        }
    }
}

/* search.cu:146-151 — sequential sum over m. */
float oracle_adc(const float* lut, int M, const uint8_t* code) {
    float dist = 0.0f;
    for (int m = 0; m < M; ++m) dist += lut[m * 256 + code[m]];
    return dist;
}

/* search.cu:216-242 — residual term, in the 32-lane order of the CUDA refine:
 * lane l owns 16-byte chunks l, l+32, ...; inside a chunk the dims ascend. */
float oracle_residual(const float* q_rot, int d, int Br, const float* res_c1d,
                      const uint8_t* rc) {
    return oracle_residual_ps(q_rot, d, 1, Br, res_c1d, 0, rc);
}

float oracle_residual_ps(const float* q_rot, int d, int Ds, int Br, const float* res_c1d_all,
                         int per_sub, const uint8_t* rc) {
    int bpv = (d * Br + 7) / 8;
    int nchunks = (bpv + 15) / 16;
    int dpc = 128 / Br, mask = (1 << Br) - 1;          /* dims per 16-byte chunk */
    float p[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int c = l; c < nchunks; c += 32) {
            for (int t = 0; t < dpc; ++t) {
                int j = c * dpc + t;
                if (j >= d) break;
                int byte = (t * Br) / 8, shift = (t * Br) % 8;
                int ri = (rc[16 * c + byte] >> shift) & mask;
                const float* res_c1d = res_c1d_all + (per_sub ? (size_t)(j / Ds) * (mask + 1) : 0);
                float diff = q_rot[j] - res_c1d[ri];
                acc = fmaf(diff, diff, acc);
            }
        }
        p[l] = acc;
    }
    for (int o = 16; o >= 1; o >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = p[l] + p[l ^ o];
        memcpy(p, t, sizeof(p));
    }
    return p[0];
}

/* search.cu:408 */
int oracle_ck(int k, float alpha) {
    int c = (int)ceilf(alpha * (float)k);
    return c > k ? c : k;
}

static inline int better(float da, int ia, float db, int ib) {
    return da < db || (da == db && ia < ib);   /* jhq_v3_ivf/search.cu:22-24 */
}

/* insert (d, i) into a sorted top-K list of length K (bd/bi), if it beats the tail */
static inline void topk_insert(float* bd, int* bi, int K, float dv, int iv) {
    if (!better(dv, iv, bd[K - 1], bi[K - 1])) return;
    int pos = K - 1;
    while (pos > 0 && better(dv, iv, bd[pos - 1], bi[pos - 1])) {
        bd[pos] = bd[pos - 1]; bi[pos] = bi[pos - 1]; --pos;
    }
    bd[pos] = dv; bi[pos] = iv;
}

int oracle_search(const float* q_rot, int64_t nq, int d, int M, int B, int Br,
                  const float* c1d, const float* res_c1d,
                  const uint8_t* codes, const uint8_t* res, const float* corr,
                  const int32_t* assign, int64_t n,
                  const float* cents, const float* norms, int nlist, int nprobe,
                  int k, float alpha, int nthreads,
                  float* out_dists, int32_t* out_ids) {
    return oracle_search_ps(q_rot, nq, d, M, B, Br, c1d, res_c1d, 0, codes, res, corr, assign, n,
                            cents, norms, nlist, nprobe, k, alpha, nthreads, out_dists, out_ids);
}

int oracle_search_ps(const float* q_rot, int64_t nq, int d, int M, int B, int Br,
                     const float* c1d, const float* res_c1d, int per_sub,
                     const uint8_t* codes, const uint8_t* res, const float* corr,
                     const int32_t* assign, int64_t n,
                     const float* cents, const float* norms, int nlist, int nprobe,
                     int k, float alpha, int nthreads,
                     float* out_dists, int32_t* out_ids) {
    if (d <= 0 || M <= 0 || d % M || k <= 0 || nlist <= 0 || nprobe <= 0) return 1;
    if (nprobe > nlist) nprobe = nlist;
    int bpv = (d * Br + 7) / 8;
    int ck = oracle_ck(k, alpha);

    /* CSR of ids by list, ids ascending inside each list */
    int64_t* off = (int64_t*)calloc((size_t)nlist + 1, sizeof(int64_t));
    for (int64_t i = 0; i < n; ++i) off[assign[i] + 1]++;
    for (int c = 0; c < nlist; ++c) off[c + 1] += off[c];
    int32_t* members = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n > 0 ? n : 1));
    int64_t* fill = (int64_t*)malloc(sizeof(int64_t) * (size_t)nlist);
    for (int c = 0; c < nlist; ++c) fill[c] = off[c];
    for (int64_t i = 0; i < n; ++i) members[fill[assign[i]]++] = (int32_t)i;
    free(fill);

#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
    #pragma omp parallel
    {
        float* lut = (float*)malloc(sizeof(float) * (size_t)M * 256);
        float* s = (float*)malloc(sizeof(float) * (size_t)nlist);
        float* pd = (float*)malloc(sizeof(float) * (size_t)nprobe);
        int* pi = (int*)malloc(sizeof(int) * (size_t)nprobe);
        float* cd = (float*)malloc(sizeof(float) * (size_t)ck);
        int* ci = (int*)malloc(sizeof(int) * (size_t)ck);
        float* fd = (float*)malloc(sizeof(float) * (size_t)k);
        int* fi = (int*)malloc(sizeof(int) * (size_t)k);
        #pragma omp for schedule(dynamic, 1)
        for (int64_t qi = 0; qi < nq; ++qi) {
            const float* q = q_rot + qi * d;
            /* probes: search.cu:13-62 semantics, exact (s, c) order (v3 :46-85) */
            for (int p = 0; p < nprobe; ++p) { pd[p] = INFINITY; pi[p] = -1; }
            for (int c = 0; c < nlist; ++c) {
                float sc = norms[c] - 2.0f * dot_chain(q, cents + (size_t)c * d, d);
                if (pi[nprobe - 1] < 0 || better(sc, c, pd[nprobe - 1], pi[nprobe - 1])) {
                    int pos = nprobe - 1;
                    while (pos > 0 && (pi[pos - 1] < 0 || better(sc, c, pd[pos - 1], pi[pos - 1]))) {
                        pd[pos] = pd[pos - 1]; pi[pos] = pi[pos - 1]; --pos;
                    }
                    pd[pos] = sc; pi[pos] = c;
                }
            }
            (void)s;
            oracle_byte_lut(q, d, M, B, c1d, lut);
            /* top-ck by (primary, id) over probed lists */
            for (int i = 0; i < ck; ++i) { cd[i] = INFINITY; ci[i] = 0x7fffffff; }
            for (int p = 0; p < nprobe; ++p) {
                int c = pi[p];
                if (c < 0) continue;
                for (int64_t t = off[c]; t < off[c + 1]; ++t) {
                    int id = members[t];
                    float dist = oracle_adc(lut, M, codes + (size_t)id * M);
                    topk_insert(cd, ci, ck, dist, id);
                }
            }
            /* refine + final top-k by (comp, id) */
            for (int i = 0; i < k; ++i) { fd[i] = INFINITY; fi[i] = 0x7fffffff; }
            for (int i = 0; i < ck; ++i) {
                if (ci[i] == 0x7fffffff) continue;
                int id = ci[i];
                float r = oracle_residual_ps(q, d, d / M, Br, res_c1d, per_sub,
                                             res + (size_t)id * bpv);
                float comp = (cd[i] + r) + corr[id];
                topk_insert(fd, fi, k, comp, id);
            }
            for (int i = 0; i < k; ++i) {
                int valid = fi[i] != 0x7fffffff;
                out_dists[qi * k + i] = valid ? fd[i] : INFINITY;
                out_ids[qi * k + i] = valid ? fi[i] : -1;
            }
        }
        free(lut); free(s); free(pd); free(pi); free(cd); free(ci); free(fd); free(fi);
    }
    free(off); free(members);
    return 0;
}

/* Exact rerank over stored vectors (the hblock indexes' exact L2 stage,
 * hblock_v34/search.cu:531-690, applied behind the JHQ refine). For each query,
 * the first kr ids of cand [nq][kr] (-1 = none) are re-scored by ||q - x||^2
 * summed as 32 lane partials (lane l takes dims 4c..4c+3 for c = l, l+32, ...,
 * an in-order fma chain) joined by an xor butterfly, then the k smallest by
 * (distance, id) are written, missing ones as (+inf, -1). */
static float exact_l2_lanes(const float* q, const float* x, int d) {
    float p[32];
    int c4 = d / 4;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int c = l; c < c4; c += 32)
            for (int t = 0; t < 4; ++t) {
                float diff = q[4 * c + t] - x[4 * c + t];
                acc = fmaf(diff, diff, acc);
            }
        p[l] = acc;
    }
    for (int o = 16; o >= 1; o >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = p[l] + p[l ^ o];
        memcpy(p, t, sizeof(p));
    }
    return p[0];
}

int oracle_rerank(const float* q, int64_t nq, int d, const float* x, int64_t n,
                  const int32_t* cand, int kr, int k, float* out_dists, int32_t* out_ids) {
    if (d % 4 != 0 || kr <= 0 || k <= 0) return 1;
    #pragma omp parallel for schedule(dynamic, 4)
    for (int64_t qi = 0; qi < nq; ++qi) {
        float* bd = out_dists + qi * k;
        int32_t* bi = out_ids + qi * k;
        for (int i = 0; i < k; ++i) { bd[i] = INFINITY; bi[i] = -1; }
        for (int i = 0; i < kr; ++i) {
            int32_t id = cand[qi * kr + i];
            if (id < 0 || id >= n) continue;
            float dv = exact_l2_lanes(q + qi * d, x + (int64_t)id * d, d);
            if (!better(dv, id, bd[k - 1], bi[k - 1])) continue;
            int j = k - 1;
            while (j > 0 && better(dv, id, bd[j - 1], bi[j - 1])) {
                bd[j] = bd[j - 1]; bi[j] = bi[j - 1]; --j;
            }
            bd[j] = dv; bi[j] = id;
        }
    }
    return 0;
}
