// device_utils.cuh — small device helpers shared by the search kernels:
// order-preserving float keys, packed (distance, id) candidate keys and
// shared-memory bitonic sort networks (warp- and block-wide).
//
// A candidate is one uint64: high 32 bits = order-preserving image of the
// float distance, low 32 bits = the non-negative vector id. Sorting the
// uint64 values ascending therefore orders candidates by (distance, id),
// the tie rule of the reference's exact path (jhq_v3_ivf/search.cu:22-24).
// KEY_EMPTY (all ones) sorts after every real candidate.
#pragma once
#include <cstdint>

namespace jhq {

constexpr uint64_t KEY_EMPTY = ~0ull;

__device__ __forceinline__ uint32_t float_order(float f) {
    f = f + 0.0f;                                   // -0 -> +0, so +-0 tie
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}
__device__ __forceinline__ uint64_t make_key(float dist, int id) {
    return ((uint64_t)float_order(dist) << 32) | (uint32_t)id;
}
__device__ __forceinline__ float key_dist(uint64_t k) { return order_float((uint32_t)(k >> 32)); }
__device__ __forceinline__ int key_id(uint64_t k) { return (int)(uint32_t)(k & 0xffffffffu); }

// Ascending bitonic sort of s[0..n) (n a power of two) by one warp.
__device__ __forceinline__ void warp_bitonic_sort(uint64_t* s, int n, int lane) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < n; i += 32) {
                int p = i ^ j;
                if (p > i) {
                    uint64_t a = s[i], b = s[p];
                    bool up = (i & k) == 0;
                    if ((a > b) == up) { s[i] = b; s[p] = a; }
                }
            }
            __syncwarp();
        }
    }
}

// Ascending bitonic sort of s[0..n) (n a power of two) by a whole block.
// Caller must __syncthreads() before (data written) — this ends synced.
__device__ __forceinline__ void block_bitonic_sort(uint64_t* s, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                int p = i ^ j;
                if (p > i) {
                    uint64_t a = s[i], b = s[p];
                    bool up = (i & k) == 0;
                    if ((a > b) == up) { s[i] = b; s[p] = a; }
                }
            }
            __syncthreads();
        }
    }
}

// Merge two ascending runs s[0..h) and s[h..2h) into one ascending run of 2h
// (h a power of two) by a whole block: reverse the second run, then run the
// bitonic merge network. Caller syncs before; ends synced.
__device__ __forceinline__ void block_merge_halves(uint64_t* s, int h) {
    for (int i = threadIdx.x; i < h / 2; i += blockDim.x) {
        uint64_t t = s[h + i]; s[h + i] = s[2 * h - 1 - i]; s[2 * h - 1 - i] = t;
    }
    __syncthreads();
    for (int j = h; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < 2 * h; i += blockDim.x) {
            int p = i ^ j;
            if (p > i) {
                uint64_t a = s[i], b = s[p];
                if (a > b) { s[i] = b; s[p] = a; }
            }
        }
        __syncthreads();
    }
}

// Same merge by one warp.
__device__ __forceinline__ void warp_merge_halves(uint64_t* s, int h, int lane) {
    for (int i = lane; i < h / 2; i += 32) {
        uint64_t t = s[h + i]; s[h + i] = s[2 * h - 1 - i]; s[2 * h - 1 - i] = t;
    }
    __syncwarp();
    for (int j = h; j > 0; j >>= 1) {
        for (int i = lane; i < 2 * h; i += 32) {
            int p = i ^ j;
            if (p > i) {
                uint64_t a = s[i], b = s[p];
                if (a > b) { s[i] = b; s[p] = a; }
            }
        }
        __syncwarp();
    }
}

}  // namespace jhq
