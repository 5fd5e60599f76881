// pilot.cu — a pruning bound per query for the flat ADC scan.
//
// A flat index (nlist = 1) scans every vector, so the scan's pruning bounds
// (a warp's, a CTA's and the query's global ck-th key) start at +inf and a
// warp only ever sees a small share of the vectors: its bound stays far above
// the query's true ck-th distance. train() therefore also groups the rotated
// training rows into a few dozen k-means "pilot" clusters and add() records
// each vector's cluster. Before the scan, per query:
//   1. the nearest pilot centroid (fp32 scores);
//   2. the members of that cluster get their ADC keys with the scan's own
//      arithmetic (same nibble tables, same sequential sum over m); each of
//      PILOT_SPLIT CTAs scores a share and keeps its ck smallest keys;
//   3. the ck-th smallest of those lowers the query's global bound to
//      (that key + 1).
// ck stored vectors have keys at or below that key, so the query's exact
// top-ck does too, and the scan (which keeps keys strictly below its bound)
// loses none of them. Which cluster is picked, and which members are scored,
// only affects how tight the bound is, never the result.
#include "device_utils.cuh"
#include "jhq_common.h"
#include "kernels.cuh"

namespace jhq {
namespace {

constexpr int PL_THREADS = 256;
constexpr int PL_GMAX = 16;                  // 16-byte code groups per row held in registers

// Stage 1: CTA (q, g) scores pilot centroids [16g, 16g + 16) for query q
// (fp32, any order: the choice of cluster only affects how tight the bound
// is): 16 threads per centroid, each summing an interleaved slice of float4s.
constexpr int PN_CENTS = 16;
__global__ void __launch_bounds__(PL_THREADS)
pilot_nearest_kernel(PilotArgs a) {
    constexpr int S = PL_THREADS / PN_CENTS;
    const int q = blockIdx.x, tid = threadIdx.x, sl = tid % S;
    if (a.d_nvalid && q >= *a.d_nvalid) return;
    const int c = blockIdx.y * PN_CENTS + tid / S;
    const float* qr = a.q_rot + (int64_t)q * a.d;
    float dot = 0.0f;
    if (c < a.P) {
        const float* pc = a.pcents + (int64_t)c * a.d;
        if ((a.d & 3) == 0) {
            const float4* p4 = reinterpret_cast<const float4*>(pc);
            const float4* q4 = reinterpret_cast<const float4*>(qr);
            const int d4 = a.d / 4;
            for (int j0 = sl; j0 < d4; j0 += 8 * S) {
                float4 v[8], w[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (j0 + u * S < d4) { v[u] = __ldg(p4 + j0 + u * S); w[u] = __ldg(q4 + j0 + u * S); }
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (j0 + u * S < d4) dot += v[u].x * w[u].x + v[u].y * w[u].y + v[u].z * w[u].z + v[u].w * w[u].w;
            }
        } else {
            for (int j = sl; j < a.d; j += S) dot += __ldg(pc + j) * __ldg(qr + j);
        }
    }
#pragma unroll
    for (int o = S >> 1; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (c < a.P && sl == 0) a.pscores[(int64_t)q * a.P + c] = a.pnorms[c] - 2.0f * dot;
}

// Stage 2: CTA (q, part) scores its share (at most PILOT_CHUNK) of the
// query's pilot-cluster members and writes its ck smallest keys
// (KEY_EMPTY-padded) to pkeys[q][part][0..ck).
__global__ void __launch_bounds__(PL_THREADS)
pilot_keys_kernel(PilotArgs a) {
    extern __shared__ float psm[];
    __shared__ uint64_t buf[PILOT_CHUNK];
    __shared__ int cq_sh;
    const int q = blockIdx.x, part = blockIdx.y, tid = threadIdx.x;
    if (a.d_nvalid && q >= *a.d_nvalid) return;
    uint64_t* out = a.pkeys + ((int64_t)q * PILOT_SPLIT + part) * a.ck;
    float* tab = psm;                            // [M][32]: lo nibble 0..15, hi 16..31
    float* qs = tab + (size_t)a.M * 32;
    float* c1d = qs + a.d;
    for (int j = tid; j < a.d; j += PL_THREADS) qs[j] = a.q_rot[(int64_t)q * a.d + j];
    __syncthreads();
    // nearest pilot cluster from the stage-1 scores (ties: lowest centroid);
    // every CTA of the query reads the same scores, so all pick the same one
    {
        uint64_t key = KEY_EMPTY;
        for (int c = tid; c < a.P; c += PL_THREADS) {
            const uint64_t k = ((uint64_t)float_order(a.pscores[(int64_t)q * a.P + c]) << 32) | (uint32_t)c;
            key = k < key ? k : key;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const uint64_t other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other < key ? other : key;
        }
        if ((tid & 31) == 0) buf[tid >> 5] = key;
        __syncthreads();
        if (tid == 0) {
            uint64_t m = buf[0];
            for (int w = 1; w < PL_THREADS / 32; ++w) m = buf[w] < m ? buf[w] : m;
            cq_sh = (int)(uint32_t)(m & 0xffffffffu);
        }
        __syncthreads();
    }
    const int cq = cq_sh;
    const int off0 = a.pilot_off[cq];
    const int cnt = min(a.pilot_off[cq + 1] - off0, PILOT_SPLIT * PILOT_CHUNK);
    const int chunk = (cnt + PILOT_SPLIT - 1) / PILOT_SPLIT;
    const int i0 = part * chunk, i1 = min(cnt, i0 + chunk);
    if (i0 >= i1) {                              // uniform: nothing to score
        for (int i = tid; i < a.ck; i += PL_THREADS) out[i] = KEY_EMPTY;
        return;
    }
    const int Ds = a.d / a.M, bpd = a.B / Ds, kmask = (1 << bpd) - 1, kpn = 4 / bpd;
    const int K1D = 1 << bpd;
    for (int j = tid; j < K1D; j += PL_THREADS) c1d[j] = a.c1d[j];
    __syncthreads();
    // the scan's nibble tables (build_tables<1> in scan.cu), entry for entry
    for (int i = tid; i < a.M * 32; i += PL_THREADS) {
        const int m = i >> 5, t = i & 31, half = t >> 4, n = t & 15;
        float acc = 0.0f;
        const int k0 = half ? kpn : 0;
        const int k1 = half ? Ds : min(kpn, Ds);
        for (int k = k0; k < k1; ++k) {
            const float diff = qs[m * Ds + k] - c1d[(n >> ((k - k0) * bpd)) & kmask];
            acc = __fmaf_rn(diff, diff, acc);
        }
        tab[i] = acc;
    }
    __syncthreads();
    // members' keys: dist = sum over m in order of (lo + hi) (add_group<1> in scan.cu)
    for (int i = i0 + tid; i < i1; i += PL_THREADS) {
        const int id = a.pilot_ids[off0 + i];
        const uint8_t* code = a.pcodes + (int64_t)id * a.M;
        float dist = 0.0f;
        if ((a.M & 15) == 0 && a.M <= 16 * PL_GMAX) {
            uint4 cv[PL_GMAX];                   // the whole code row in flight at once
#pragma unroll
            for (int g = 0; g < PL_GMAX; ++g)
                if (g < a.M / 16) cv[g] = __ldg(reinterpret_cast<const uint4*>(code) + g);
#pragma unroll
            for (int g = 0; g < PL_GMAX; ++g) {
                if (g >= a.M / 16) break;
                const uint4 v = cv[g];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const uint32_t w = wi == 0 ? v.x : wi == 1 ? v.y : wi == 2 ? v.z : v.w;
#pragma unroll
                    for (int bb = 0; bb < 4; ++bb) {
                        const int m = g * 16 + wi * 4 + bb;
                        const uint32_t b = (w >> (8 * bb)) & 255u;
                        const float lo = tab[m * 32 + (b & 15u)];
                        const float hi = tab[m * 32 + 16 + (b >> 4)];
                        dist = __fadd_rn(dist, __fadd_rn(lo, hi));
                    }
                }
            }
        } else {
            for (int m = 0; m < a.M; ++m) {
                const uint32_t b = code[m];
                dist = __fadd_rn(dist, __fadd_rn(tab[m * 32 + (b & 15u)], tab[m * 32 + 16 + (b >> 4)]));
            }
        }
        buf[i - i0] = make_key(dist, id);
    }
    const int n = i1 - i0;
    for (int i = tid; i < a.ck; i += PL_THREADS) out[i] = KEY_EMPTY;
    __syncthreads();
    // keys are distinct (ids), so a key's rank = the number of smaller keys
    for (int i = tid; i < n; i += PL_THREADS) {
        const uint64_t k = buf[i];
        int r = 0;
        for (int j = 0; j < n; ++j) r += buf[j] < k;
        if (r < a.ck) out[r] = k;
    }
}

// Stage 3, one block per query: the ck-th smallest of the PILOT_SPLIT lists
// (found by rank counting; the keys are distinct) lowers the query's global
// bound to (that key + 1).
__global__ void __launch_bounds__(PL_THREADS)
pilot_select_kernel(PilotArgs a) {
    extern __shared__ uint64_t ksm[];
    const int q = blockIdx.x, tid = threadIdx.x;
    if (a.d_nvalid && q >= *a.d_nvalid) return;
    const int n = PILOT_SPLIT * a.ck;
    const uint64_t* in = a.pkeys + (int64_t)q * n;
    for (int i = tid; i < n; i += PL_THREADS) ksm[i] = in[i];
    __syncthreads();
    for (int i = tid; i < n; i += PL_THREADS) {
        const uint64_t k = ksm[i];
        if (k == KEY_EMPTY) continue;
        int r = 0;
        for (int j = 0; j < n; ++j) r += ksm[j] < k;
        if (r == a.ck - 1)
            atomicMin(reinterpret_cast<unsigned long long*>(a.gthr + q), (unsigned long long)(k + 1));
    }
}

}  // namespace

size_t pilot_smem_bytes(int M, int d) { return ((size_t)M * 32 + d + 256) * sizeof(float); }

void pilot_bound(const PilotArgs& a, cudaStream_t st) {
    if (a.nq <= 0) return;
    const size_t smem = pilot_smem_bytes(a.M, a.d);
    const size_t smem3 = (size_t)PILOT_SPLIT * a.ck * sizeof(uint64_t);
    static std::atomic<uint64_t> attr{0};
    once_per_device(attr, [] {
        JHQ_CUDA(cudaFuncSetAttribute(pilot_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      160 * 1024));
        JHQ_CUDA(cudaFuncSetAttribute(pilot_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      160 * 1024));
    });
    if (smem > 160 * 1024 || smem3 > 160 * 1024) fail(JHQ_EINVAL, "pilot_bound: sizes too large");
    pilot_nearest_kernel<<<dim3((unsigned)a.nq, (unsigned)((a.P + PN_CENTS - 1) / PN_CENTS)),
                           PL_THREADS, 0, st>>>(a);
    JHQ_LAUNCH_CHECK();
    count_launch();
    pilot_keys_kernel<<<dim3((unsigned)a.nq, PILOT_SPLIT), PL_THREADS, smem, st>>>(a);
    JHQ_LAUNCH_CHECK();
    count_launch();
    pilot_select_kernel<<<(unsigned)a.nq, PL_THREADS, smem3, st>>>(a);
    JHQ_LAUNCH_CHECK();
    count_launch();
}

}  // namespace jhq
