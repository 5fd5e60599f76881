// ivf_tc.cuh — the IVF ADC scan on the tensor cores for 2-bit-per-dimension
// codes (K1D = 4: B = 8 with Ds = 4, the C3 / C4 shapes). Included by
// coarse_tc.cu, whose tcgen05 helpers and error flag it uses.
//
// With four codewords c0..c3 per dimension and the two code bits (l, h) of
// dimension j (level l + 2h),
//   c[b_j] = c0 + e1 l_j + e2 h_j + e3 l_j h_j,
//   e1 = c1 - c0, e2 = c2 - c0, e3 = c3 - c2 - c1 + c0,
// so the ADC distance of query q to vector v is
//   s_v = sum_j (q_j - c[b_j])^2 = Sq' - 2 w . bits(v) + cn(v),
//   Sq' = sum_j q_j^2 - 2 c0 sum_j q_j,  w = (e1 q | e2 q | e3 q),
//   bits(v) = (L | H | L&H) (3 x 128 zero-one entries),
//   cn(v) = sum_j c[b_j]^2 (from the level counts of v).
// The scan is two passes over the batch's probed lists:
//   1. ivf_tc_kernel: per work unit (list l, up to 64 of the queries probing l,
//      one tile of 128 slots = 4 pages of l) the bit planes of the tile are
//      expanded to s8 0/1 rows in shared memory, w is quantised (per query,
//      int16 split in two s8 planes, exactly as in the flat scan), and one
//      tcgen05 kind::i8 GEMM gives w . bits exactly up to the quantisation.
//      Only the per-query minimum of the approximate score over the tile is
//      written (the scores themselves never leave the SM);
//   2. ivf_tc_select_kernel: per query, tau = the ck-th smallest tile minimum;
//      ck distinct vectors have s~ <= tau, so every exact top-ck member has
//      s~ <= tau + 2E (E bounds |s~ - s*| up to a per-query constant), and its
//      tile's minimum is <= tau + 2E. The slots of those tiles are rescored with
//      the scan's own arithmetic (nibble tables lo + hi, in-order sum over the
//      Mp subspaces from 0: the oracle's key), giving the exact top-ck by
//      (distance, id) as the query's single candidate slot for the refine.
// Results are those of the SIMT scan, bit for bit.

namespace {

constexpr int IT_THREADS = 256;               // pass 1: two threads per tile row
constexpr int IT_NQ = 64;                     // queries per work unit (B rows: 64 hi + 64 lo)
constexpr int IT_KP = 384;                    // K: three planes of 128 dims
constexpr int IT_KB = IT_KP / 128;            // 128-byte K blocks
constexpr int IT_A_BYTES = 128 * IT_KP;       // 48 KB
constexpr int IT_B_BYTES = 2 * IT_NQ * IT_KP; // 24 KB
constexpr int IT_SMEM = IT_A_BYTES + IT_B_BYTES + 1024 /* align */;
constexpr int IS_THREADS = 256;               // pass 2: one CTA per query
constexpr int IS_CAP = 1024;                  // exact keys held before a compaction
constexpr int IS_TK = 8192;                   // tile minima held in shared memory (more: global)

// Per query q < nq (128 threads): the s8 planes qw[q][0] = hi, qw[q][1] = lo of
// W = rint(w / s), s = max|w| / 32000, and the constants of the query:
//   qc[q] = {Sq', -2 s, E, 0}.
// E bounds |s~ - s*| for every vector of the query, up to a per-query constant:
// the LUT path's roundings, the quantisation residual, and the roundings of cn
// and of the epilogue's fma.
constexpr int IP_THREADS = 128;
__global__ void __launch_bounds__(IP_THREADS)
ivf_prep_kernel(const float* __restrict__ q_rot, int nq, int d, int Mp, float c0, float e1,
                float e2, float e3, float cmax, int8_t* __restrict__ qw,
                float4* __restrict__ qc) {
    const int q = blockIdx.x;
    if (q >= nq) return;
    __shared__ float red[6][IP_THREADS / 32];
    __shared__ float s_sh;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float* x = q_rot + (int64_t)q * d;
    const float e[3] = {e1, e2, e3};
    auto wv = [&](int i) {                               // w_i in fp32 (0 past d)
        const int p = i >> 7, j = i & 127;
        return j < d ? e[p] * x[j] : 0.0f;
    };
    float amax = 0.0f;
    for (int i = threadIdx.x; i < IT_KP; i += IP_THREADS) amax = fmaxf(amax, fabsf(wv(i)));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[0][warp] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int w = 0; w < IP_THREADS / 32; ++w) a = fmaxf(a, red[0][w]);
        s_sh = a > 0.0f ? a / FT_QMAX : 1.0f;
    }
    __syncthreads();
    const float sc = s_sh;
    float r1 = 0.0f, l1w = 0.0f, sq = 0.0f, sx = 0.0f, V = 0.0f;
    for (int i = threadIdx.x; i < IT_KP; i += IP_THREADS) {
        const float w = wv(i);
        const float Wf = fminf(fmaxf(rintf(w / sc), -FT_QMAX), FT_QMAX);
        const int W = (int)Wf;
        const int wh = (W + 128) >> 8;                   // floor((W + 128) / 256)
        qw[((int64_t)q * 2) * IT_KP + i] = (int8_t)wh;
        qw[((int64_t)q * 2 + 1) * IT_KP + i] = (int8_t)(W - wh * 256);
        r1 += fabsf(__fmaf_rn(-sc, Wf, w));
        l1w += fabsf(w);
    }
    for (int j = threadIdx.x; j < d; j += IP_THREADS) {
        const float v = x[j], a = fabsf(v) + cmax;
        sq = __fmaf_rn(v, v, sq);
        sx += v;
        V = __fmaf_rn(a, a, V);
    }
    float vals[5] = {r1, l1w, sq, sx, V};
#pragma unroll
    for (int k = 0; k < 5; ++k) {
#pragma unroll
        for (int o = 16; o; o >>= 1) vals[k] += __shfl_xor_sync(0xffffffffu, vals[k], o);
    }
    __syncthreads();
    if (lane == 0)
        for (int k = 0; k < 5; ++k) red[k][warp] = vals[k];
    __syncthreads();
    if (threadIdx.x == 0) {
        float t[5] = {0, 0, 0, 0, 0};
        for (int k = 0; k < 5; ++k)
            for (int w = 0; w < IP_THREADS / 32; ++w) t[k] += red[k][w];
        const float u = 5.9604645e-08f;                  // 2^-24
        const float R1 = t[0] * 1.001f, L1w = t[1] * 1.001f;
        const float Sq = __fmaf_rn(-2.0f * c0, t[3], t[2]);
        const float G = L1w + R1;                        // bounds |w . bits| and s |W . bits|
        const float C = (float)d * cmax * cmax * 1.001f; // bounds cn(v)
        const float E = 1.1f * (t[4] * 1.001f * (float)(2 * Mp + 16) * u +
                                2.0f * (R1 + u * L1w) + 2.0f * u * G + 6.0f * u * C +
                                u * (fabsf(Sq) + C) + u * (fabsf(Sq) + C + 2.0f * G));
        qc[q] = make_float4(Sq, -2.0f * sc, E, 0.0f);
    }
}

// tmin[0 .. qtile[nq]) = all ones, the identity of the pass-1 atomicMin
__global__ void tmin_fill_kernel(uint32_t* __restrict__ tmin, const int64_t* __restrict__ qtile, int nq) {
    const int64_t n = qtile[nq];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        tmin[i] = 0xFFFFFFFFu;
}

// x holds bits only at even positions (x & 0x55555555 == x): bit 2j -> byte j
// as 0 / 1, 16 bytes. A byte b with bits 0, 2, 4, 6 times 0x41041 (shifts 0, 6,
// 12, 18) puts bit 2k at 8k; the other partial products land on odd bits or on
// bits 12 and 18 (with carries into 13 and 19), all masked off.
__device__ __forceinline__ uint4 spread_even(uint32_t x) {
    auto sp = [](uint32_t b) { return (b * 0x41041u) & 0x01010101u; };
    return make_uint4(sp(__byte_perm(x, 0u, 0x4440)), sp(__byte_perm(x, 0u, 0x4441)),
                      sp(__byte_perm(x, 0u, 0x4442)), sp(x >> 24));
}

// 128-byte swizzled K-major store of 16 bytes: row r, 16-byte chunk c of a
// K block whose rows are 128 bytes (8-row groups 1024 bytes apart)
__device__ __forceinline__ void sw128_store(uint8_t* blk, int r, int c, uint4 v) {
    *reinterpret_cast<uint4*>(blk + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)) = v;
}

// Pass 1. Work units are numbered list-major, then query group (64 queries of
// the list's bucket), then tile (4 pages), as plan_build(chunk_pages = 4,
// qg = 64) counts them; a CTA takes a contiguous range. Per unit:
//   1. (new list or group) the group's s8 query planes -> B (rows 0..63 hi,
//      64..127 lo, missing queries zero) and the group's constants;
//   2. two threads per slot (one per 16-subspace group) expand its codes into
//      the three bit planes of its A row and count the levels (cn);
//   3. one thread issues the 12 MMAs (K = 32 each) and commits; all wait
//      (bounded);
//   4. the eight warps read 32 TMEM lanes (rows) x 32 query columns each, form
//      s~ = (Sq' + cn) + (-2 s)(256 Gh + Gl), reduce each query column's
//      minimum over the tile and write it to tmin[qtile[q] + cpo[q][p] + t].
// NP = 3 K blocks (planes L, H, L&H) in general; NP = 2 when the codebook is
// symmetric (c0 = -c3, c1 = -c2), where the L&H weight c3 - c2 - c1 + c0 is
// zero and its query plane is all zeros: the third block would only add 0.
// The two-plane form needs 64 KB of operands, so three CTAs share an SM
// (registers capped at 85 a thread; the epilogue reads TMEM 16 columns at a
// time to fit).
template <int NP>
__host__ __device__ constexpr int it_smem_bytes() { return 2 * NP * 16384 + 1024; }
template <int NP>
constexpr int it_ctas_per_sm() { return NP == 2 ? 3 : 2; }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

template <int NP>
__global__ void __launch_bounds__(IT_THREADS, NP == 2 ? 3 : 0)
ivf_tc_kernel(const uint8_t* __restrict__ pages, const int32_t* __restrict__ slot_ids,
              const int32_t* __restrict__ lpo, PlanBufs pb, const int8_t* __restrict__ qw,
              const float4* __restrict__ qc, int nlist, int nprobe, int d, int Mp,
              float c0s, float c1s, float c2s, float c3s, uint32_t* __restrict__ tmin,
              long long wait_limit) {
    extern __shared__ uint8_t smem_raw[];
    // per-unit arrays by unit parity and per-group arrays by group parity: a
    // warp may still read unit u's while others fill unit u+1's
    __shared__ int cnt_s[2][2][128];                   // level counts per half row: nL | nH << 10 | nLH << 20
    __shared__ int id_s[2][128];
    __shared__ float2 sb_s[2][IT_NQ];                  // (Sq', -2 s) of each query of the group
    __shared__ int64_t base_s[2][IT_NQ];
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* As = smem;                                    // [3][128][128]
    uint8_t* Bs = smem + NP * 16384;                       // [NP][2 IT_NQ][128]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = Mp / 16;
    const int64_t U = pb.unit_off[nlist];
    const int64_t u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
    if (u0 >= u1) return;                                  // uniform: no TMEM, no barrier yet
    const uint32_t barp = smem_u32(&bar);
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(barp), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(&tmem_slot)), "r"(2 * IT_NQ));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;
    // s32 accumulate, A and B s8, K-major, N' = 2 IT_NQ, M = 128
    const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(2 * IT_NQ >> 3) << 17) |
                           ((uint32_t)(128 >> 4) << 24);

    // the unit u0: its list (last l with unit_off[l] <= u0), group and tile
    int l = 0;
    {
        int lo = 0, hi = nlist;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (pb.unit_off[mid] <= u0) lo = mid; else hi = mid;
        }
        l = lo;
    }
    int tiles_l = (lpo[l + 1] - lpo[l] + 3) >> 2;
    int g = (int)((u0 - pb.unit_off[l]) / tiles_l), t = (int)((u0 - pb.unit_off[l]) % tiles_l);
    int cur_l = -1, cur_g = -1, nqg = 0, gb = 1;
    uint32_t phase = 0;
    bool failed = false;
    // the A row of this thread in unit (L, T): slot id and code words, loaded
    // one unit ahead so that their latency overlaps the current unit
    const int row = tid & 127, hf = tid >> 7;             // tile row and its 16-subspace group
    auto load_row = [&](int L, int T, int& id, uint4& w) {
        const int pg = lpo[L] + 4 * T + (row >> 5);
        const bool okp = pg < lpo[L + 1];
        id = okp ? __ldg(slot_ids + (int64_t)pg * 32 + lane) : -1;
        const uint4* pp = reinterpret_cast<const uint4*>(pages) + ((int64_t)pg * G + hf) * 32 + lane;
        w = okp ? __ldg(pp) : make_uint4(0u, 0u, 0u, 0u);
    };
    int id_c, id_n = -1;
    uint4 w_c, w_n = make_uint4(0u, 0u, 0u, 0u);
    load_row(l, t, id_c, w_c);
    for (int64_t u = u0; u < u1; ++u) {
        // the next unit: tile, then group, then the next list with units
        int l2 = l, g2 = g, t2 = t + 1, tiles2 = tiles_l;
        if (u + 1 < u1) {
            if (t2 == tiles_l) {
                t2 = 0;
                const int ng = (pb.bucket_off[l + 1] - pb.bucket_off[l] + IT_NQ - 1) / IT_NQ;
                if (++g2 == ng) {
                    g2 = 0;
                    do { ++l2; } while (l2 < nlist - 1 && pb.unit_off[l2 + 1] == pb.unit_off[l2]);
                    tiles2 = (lpo[l2 + 1] - lpo[l2] + 3) >> 2;
                }
            }
            load_row(l2, t2, id_n, w_n);
        }
        const int ub = (int)(u & 1);
        if (cur_l != l || cur_g != g) {                    // the group's B rows and constants
            gb ^= 1;
            const int b0 = pb.bucket_off[l] + g * IT_NQ;
            nqg = min(IT_NQ, pb.bucket_off[l + 1] - b0);
            for (int i = tid; i < NP * 2 * IT_NQ * 8; i += IT_THREADS) {
                const int kb = i / (2 * IT_NQ * 8), r = (i >> 3) % (2 * IT_NQ), c = i & 7;
                const int j = r % IT_NQ;
                uint4 v = make_uint4(0u, 0u, 0u, 0u);
                if (j < nqg) {
                    const int q = pb.bucket[b0 + j].x;
                    v = __ldg(reinterpret_cast<const uint4*>(
                        qw + ((int64_t)q * 2 + r / IT_NQ) * IT_KP + kb * 128 + c * 16));
                }
                sw128_store(Bs + kb * (2 * IT_NQ * 128), r, c, v);
            }
            for (int j = tid; j < IT_NQ; j += IT_THREADS) {
                float sq = 0.0f, bq = 0.0f;
                int64_t base = 0;
                if (j < nqg) {
                    const int2 e = pb.bucket[b0 + j];
                    const float4 c = qc[e.x];
                    sq = c.x;
                    bq = c.y;
                    base = pb.qslot_off[e.x] + pb.cpo[(int64_t)e.x * (nprobe + 1) + e.y];
                }
                sb_s[gb][j] = make_float2(sq, bq);
                base_s[gb][j] = base;
            }
            cur_l = l;
            cur_g = g;
        }
        // A row `row`, dims 64 hf .. 64 hf + 63: slot (page, lane) of tile t of list l
        {
            int nL = 0, nH = 0, nLH = 0;
            const uint32_t w4[4] = {w_c.x, w_c.y, w_c.z, w_c.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {               // 4 subspaces = 16 dims
                // bit 2j of xl / xh is dim j's low / high code bit
                const uint32_t xl = w4[wi] & 0x55555555u, xh = (w4[wi] >> 1) & 0x55555555u;
                const uint32_t xlh = xl & xh;
                nL += __popc(xl);
                nH += __popc(xh);
                nLH += __popc(xlh);
                const int cg = hf * 4 + wi;                // 16-dim chunk of the 128 dims
                sw128_store(As + 0 * 16384, row, cg, spread_even(xl));
                sw128_store(As + 1 * 16384, row, cg, spread_even(xh));
                if (NP == 3) sw128_store(As + 2 * 16384, row, cg, spread_even(xlh));
            }
            cnt_s[ub][hf][row] = nL | (nH << 10) | (nLH << 20);
            if (hf == 0) id_s[ub][row] = id_c;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int kb = 0; kb < NP; ++kb) {
                const uint64_t da = sw128_desc(smem_u32(As + kb * 16384));
                const uint64_t db = sw128_desc(smem_u32(Bs + kb * (2 * IT_NQ * 128)));
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t accum = (kb | k) != 0;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                        :: "r"(tmem), "l"(da + 2 * k), "l"(db + 2 * k), "r"(idesc), "r"(accum));
                }
            }
            mma_commit(barp);
        }
        // thread 0 waits for the MMAs (bounded; a timeout ends the CTA's work) and
        // the barrier releases the rest, whose TMEM reads the fence below orders
        // after it; polling from one thread leaves the issue slots to the SM's
        // other CTAs
        const bool ok = tid == 0 ? mbar_wait(barp, phase, nullptr, wait_limit) : true;
        phase ^= 1u;
        if (!__syncthreads_and(ok)) { failed = true; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        {
            // warp w: TMEM lanes (rows) 32 (w % 4) .., query columns 32 (w / 4) ..
            const int q4 = warp & 3, cb = (warp >> 2) * 32, r = q4 * 32 + lane;
            if (cb < nqg) {                                // warp-uniform
                const int c0w = cnt_s[ub][0][r], c1w = cnt_s[ub][1][r];
                const int nL = (c0w & 1023) + (c1w & 1023), nH = ((c0w >> 10) & 1023) + ((c1w >> 10) & 1023);
                const int nLH = (c0w >> 20) + (c1w >> 20);
                float cn = __int_as_float(0x7f800000);     // empty slot: never a minimum
                if (id_s[ub][r] >= 0) {
                    const int n3 = nLH, n1 = nL - nLH, n2 = nH - nLH, n0 = d - nL - nH + nLH;
                    cn = __fmaf_rn(c3s, (float)n3,
                                   __fmaf_rn(c2s, (float)n2, __fmaf_rn(c1s, (float)n1, c0s * (float)n0)));
                }
#pragma unroll 1
                for (int hh = 0; hh < 32; hh += 16) {      // 16 query columns at a time
                    uint32_t rh[16], rl[16];
                    const uint32_t taddr = tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(cb + hh);
                    tmem_ld16(taddr, rh);
                    tmem_ld16(taddr + (uint32_t)IT_NQ, rl);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    float m[16];
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        // columns past nqg hold junk that never mixes with
                        // other columns and is never written out
                        const float2 sb = sb_s[gb][cb + hh + c];
                        const int gi = (int)rh[c] * 256 + (int)rl[c];
                        m[c] = __fmaf_rn(sb.y, (float)gi, __fadd_rn(sb.x, cn));
                    }
#pragma unroll
                    for (int h = 8; h; h >>= 1) {          // transpose-reduce: lane c <- column c & 15
                        const bool up = lane & h;
#pragma unroll
                        for (int j = 0; j < h; ++j) {
                            const float send = up ? m[j] : m[j + h];
                            const float keep = up ? m[j + h] : m[j];
                            m[j] = fminf(keep, __shfl_xor_sync(0xffffffffu, send, h));
                        }
                    }
                    m[0] = fminf(m[0], __shfl_xor_sync(0xffffffffu, m[0], 16));
                    // this warp's 32 rows; the four row quarters meet in tmin
                    // (preset to all ones): the minimum of order keys is the
                    // order key of the minimum
                    const int col = cb + hh + lane;
                    if (lane < 16 && col < nqg)
                        atomicMin(tmin + base_s[gb][col] + t, float_order(m[0]));
                }
            }
        }
        // TMEM reads before the next unit's MMAs (ordered by the next barriers)
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        l = l2; g = g2; t = t2; tiles_l = tiles2;
        id_c = id_n; w_c = w_n;
    }
    if (failed && tid == 0) atomicExch(&g_tc_error, 1);
    // no MMA may still read shared memory or write TMEM when the CTA frees them
    if (tid == 0) mbar_wait(barp, phase ^ 1u, nullptr);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(2 * IT_NQ));
}

// Pass 2, one CTA per query: tau (bisection over the order keys of the
// query's tile minima), then the tiles whose minimum is <= tau + 2E, 256 at a
// time. Their pages are rescored a warp per page (lane = slot, two pages per
// warp and step, all loads issued first) with the nibble tables; the keys go
// to buf, which is compacted to the best ck_pad when full, after which keys
// above the ck-th kept one are dropped. Finally the exact top-ck by
// (distance, id) is written as the query's single candidate slot
// (cand[q][ck], gthr[q], qslot_out[q] = q).
__global__ void __launch_bounds__(IS_THREADS, 1)
ivf_tc_select_kernel(const float* __restrict__ q_rot, const float* __restrict__ c1d_g,
                     const uint8_t* __restrict__ pages, const int32_t* __restrict__ slot_ids,
                     const int32_t* __restrict__ lpo, const int32_t* __restrict__ probes,
                     PlanBufs pb, const float4* __restrict__ qc, const uint32_t* __restrict__ tmin,
                     int nq, int nprobe, int d, int M, int Mp, int ck, int ck_pad,
                     uint64_t* __restrict__ cand, uint64_t* __restrict__ gthr,
                     int64_t* __restrict__ qslot_out, const int* __restrict__ d_nvalid) {
    extern __shared__ __align__(16) unsigned char is_smem[];
    __shared__ int cnt[2][IS_THREADS / 32];
    __shared__ int nhot_s, n_s;
    __shared__ int hot[IS_THREADS];
    __shared__ int cpo_s[129];
    __shared__ int lb_s[128], le_s[128];                   // page range of each probed list
    __shared__ float c1d[4];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = IS_THREADS / 32;
    const unsigned lt = (1u << lane) - 1u;
    const int q = blockIdx.x;
    if (q >= nq) return;
    if (tid == 0) {
        qslot_out[q + 1] = q + 1;
        if (q == 0) qslot_out[0] = 0;
    }
    if (d_nvalid && q >= *d_nvalid) {                      // padding row: no candidates
        for (int i = tid; i < ck; i += IS_THREADS) cand[(int64_t)q * ck + i] = KEY_EMPTY;
        if (tid == 0) gthr[q] = KEY_EMPTY;
        return;
    }
    float* tab = reinterpret_cast<float*>(is_smem);                              // [Mp][32]
    uint64_t* buf = reinterpret_cast<uint64_t*>(is_smem + (size_t)Mp * 32 * 4);  // [IS_CAP]
    uint32_t* tks = reinterpret_cast<uint32_t*>(buf + IS_CAP);                   // [IS_TK]
    const int64_t t0 = pb.qslot_off[q];
    const int ntq = (int)(pb.qslot_off[q + 1] - t0);
    const uint32_t* tq = tmin + t0;
    const bool in_smem = ntq <= IS_TK;
    if (tid < 4) c1d[tid] = c1d_g[tid];
    for (int p = tid; p <= nprobe; p += IS_THREADS) cpo_s[p] = pb.cpo[(int64_t)q * (nprobe + 1) + p];
    for (int p = tid; p < nprobe; p += IS_THREADS) {
        const int l = probes[(int64_t)q * nprobe + p];
        lb_s[p] = lpo[l];
        le_s[p] = lpo[l + 1];
    }
    if (in_smem)
        for (int i = tid; i < ntq; i += IS_THREADS) tks[i] = tq[i];
    if (tid == 0) { nhot_s = 0; n_s = 0; }
    __syncthreads();
    // the scan's nibble tables (lo: dims 0-1 of the subspace, hi: dims 2-3)
    const float* qv = q_rot + (int64_t)q * d;
    for (int i = tid; i < Mp * 32; i += IS_THREADS) {
        const int m = i >> 5, t = i & 31, half = t >> 4, n = t & 15;
        float acc = 0.0f;
        if (m < M) {
            const int k0 = half ? 2 : 0;
            for (int k = k0; k < k0 + 2; ++k) {
                const float diff = qv[m * 4 + k] - c1d[(n >> ((k - k0) * 2)) & 3];
                acc = __fmaf_rn(diff, diff, acc);
            }
        }
        tab[i] = acc;
    }
    const uint32_t* tk = in_smem ? tks : tq;
    // tau = the ck-th smallest tile minimum (one barrier per bisection step)
    float tau = __int_as_float(0x7f800000);
    if (ck <= ntq) {
        uint32_t lo = 0, hi = 0xFFFFFFFFu;
        int it = 0;
        while (lo < hi) {
            const uint32_t mid = lo + ((hi - lo) >> 1);
            int c = 0;
            for (int i = tid; i < ntq; i += IS_THREADS) c += tk[i] <= mid;
            c = __reduce_add_sync(0xffffffffu, c);
            if (lane == 0) cnt[it & 1][warp] = c;
            __syncthreads();
            int tot = 0;
#pragma unroll
            for (int w = 0; w < NW; ++w) tot += cnt[it & 1][w];
            if (tot >= ck) hi = mid; else lo = mid + 1;
            ++it;
        }
        tau = order_float(lo);
    }
    const float T = __fadd_ru(tau, 2.0f * qc[q].z);
    __syncthreads();                                       // tables complete
    const int G = Mp / 16;
    int n = 0;                                             // keys in buf (block-uniform)
    uint64_t thr = KEY_EMPTY;     // the ck-th key after a compaction: larger keys cannot enter
    for (int b0 = 0; b0 < ntq; b0 += IS_THREADS) {
        // this round's hot tiles
        const int i = b0 + tid;
        const bool in = i < ntq && order_float(tk[i]) <= T;
        const unsigned mk = __ballot_sync(0xffffffffu, in);
        int base = 0;
        if (lane == 0 && mk) base = atomicAdd(&nhot_s, __popc(mk));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (in) hot[base + __popc(mk & lt)] = i;
        __syncthreads();
        const int npg = nhot_s * 4;                        // their pages
        // a step: every warp scores two pages (lane = slot), all loads issued first
        for (int p0 = 0; p0 < npg; p0 += 2 * NW) {
            if (n + 2 * NW * 32 > IS_CAP) {                // keep the best ck_pad
                for (int k = n + tid; k < IS_CAP; k += IS_THREADS) buf[k] = KEY_EMPTY;
                __syncthreads();
                block_bitonic_sort(buf, IS_CAP);
                n = ck_pad;
                thr = buf[ck - 1];
                __syncthreads();
                if (tid == 0) n_s = n;
                __syncthreads();
            }
            int id[2];
            uint4 cw[2][2];
#pragma unroll
            for (int v = 0; v < 2; ++v) {
                const int pi = p0 + v * NW + warp;
                id[v] = -1;
                cw[v][0] = cw[v][1] = make_uint4(0u, 0u, 0u, 0u);
                if (pi < npg) {
                    const int ti = hot[pi >> 2];
                    int plo = 0, phi = nprobe;             // last p with cpo[p] <= ti
                    while (phi - plo > 1) {
                        const int mid = (plo + phi) >> 1;
                        if (cpo_s[mid] <= ti) plo = mid; else phi = mid;
                    }
                    const int pg = lb_s[plo] + 4 * (ti - cpo_s[plo]) + (pi & 3);
                    if (pg < le_s[plo]) {
                        id[v] = __ldg(slot_ids + (int64_t)pg * 32 + lane);
                        const uint4* pp = reinterpret_cast<const uint4*>(pages) + (int64_t)pg * G * 32 + lane;
                        cw[v][0] = __ldg(pp);
                        if (G > 1) cw[v][1] = __ldg(pp + 32);
                    }
                }
            }
#pragma unroll
            for (int v = 0; v < 2; ++v) {
                uint64_t key = KEY_EMPTY;
                if (id[v] >= 0) {
                    float dist = 0.0f;
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        if (g >= G) break;
                        const uint32_t ws[4] = {cw[v][g].x, cw[v][g].y, cw[v][g].z, cw[v][g].w};
#pragma unroll
                        for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                            for (int bb = 0; bb < 4; ++bb) {
                                const int m = g * 16 + wi * 4 + bb;
                                const uint32_t bt = (ws[wi] >> (bb * 8)) & 0xFFu;
                                dist = __fadd_rn(dist, __fadd_rn(tab[m * 32 + (bt & 15u)],
                                                                  tab[m * 32 + 16 + (bt >> 4)]));
                            }
                    }
                    key = make_key(dist, id[v]);
                    if (key > thr) key = KEY_EMPTY;
                }
                const unsigned km = __ballot_sync(0xffffffffu, key != KEY_EMPTY);
                int kb = 0;
                if (lane == 0 && km) kb = atomicAdd(&n_s, __popc(km));
                kb = __shfl_sync(0xffffffffu, kb, 0);
                if (key != KEY_EMPTY) buf[kb + __popc(km & lt)] = key;
            }
            __syncthreads();
            n = n_s;
        }
        if (tid == 0) nhot_s = 0;
        __syncthreads();
    }
    int P = ck_pad;
    while (P < n) P <<= 1;
    for (int k = n + tid; k < P; k += IS_THREADS) buf[k] = KEY_EMPTY;
    __syncthreads();
    block_bitonic_sort(buf, P);
    for (int k = tid; k < ck; k += IS_THREADS) cand[(int64_t)q * ck + k] = buf[k];
    if (tid == 0) gthr[q] = buf[ck - 1];
}

__host__ __device__ inline size_t is_smem_bytes(int Mp) {
    return (size_t)Mp * 32 * 4 + (size_t)IS_CAP * 8 + (size_t)IS_TK * 4;
}

}  // namespace

