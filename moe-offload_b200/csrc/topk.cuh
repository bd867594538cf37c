// Warp-level selection of the n largest 32-bit keys, shared by the router kernels.
#pragma once

#include "common.cuh"

// Selects the n largest of keys[0..E) (all distinct, all > 0) with warp 0, results in
// descending order. Each lane keeps its local maximum; only the winning lane rescans. Keys
// live in registers when E <= 512 and are rescanned from shared memory otherwise.
constexpr int kRegKeys = 16;   // keys per lane held in registers (E <= 512)

MOE_D void warp_select_desc(const uint32_t *keys, int E, int n, uint32_t *out) {
    const int lane = threadIdx.x & 31;
    if (E <= 32 * kRegKeys) {
        uint32_t kv[kRegKeys];
        uint32_t lmax = 0;
#pragma unroll
        for (int j = 0; j < kRegKeys; ++j) {
            const int e = lane + 32 * j;
            kv[j] = (e < E) ? keys[e] : 0u;
            lmax = max(lmax, kv[j]);
        }
        for (int r = 0; r < n; ++r) {
            const uint32_t win = __reduce_max_sync(0xffffffffu, lmax);
            if (lmax == win) {
                uint32_t nm = 0;
#pragma unroll
                for (int j = 0; j < kRegKeys; ++j) {
                    kv[j] = (kv[j] == win) ? 0u : kv[j];
                    nm = max(nm, kv[j]);
                }
                lmax = nm;
            }
            if (lane == 0) out[r] = win;
        }
    } else {
        __shared__ uint32_t taken[64];
        uint32_t lmax = 0;
        for (int e = lane; e < E; e += 32) lmax = max(lmax, keys[e]);
        for (int r = 0; r < n; ++r) {
            const uint32_t win = __reduce_max_sync(0xffffffffu, lmax);
            if (lane == 0) taken[r] = win;
            __syncwarp();
            if (lmax == win) {
                uint32_t nm = 0;
                for (int e = lane; e < E; e += 32) {
                    const uint32_t kv = keys[e];
                    bool used = false;
                    for (int q = 0; q <= r; ++q) used |= (kv == taken[q]);
                    if (!used) nm = max(nm, kv);
                }
                lmax = nm;
            }
            if (lane == 0) out[r] = win;
        }
    }
    __syncwarp();
}


// Block-level selection of the K largest of keys[0..E) (distinct, > 0) for E <= 32 * (number
// of warps) and K <= 32: every warp sorts its 32 keys with a bitonic network over shuffles,
// keeps its K largest in cand[], then warp 0 merges the sorted lists (K rounds of one
// warp-wide max over the list heads). out[0..K) receives the keys in descending order.
// Call with every thread of the block; synchronises internally.
MOE_D void block_select_desc(const uint32_t *keys, int E, int K, uint32_t *cand, uint32_t *out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t key = (warp * 32 + lane < E) ? keys[warp * 32 + lane] : 0u;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint32_t other = __shfl_xor_sync(0xffffffffu, key, j);
            const bool lower = (lane & j) == 0, asc = (lane & k) == 0;
            key = (lower == asc) ? min(key, other) : max(key, other);
        }
    }
    // ascending within the warp: lane 31 - i holds the i-th largest
    if (lane >= 32 - K) cand[warp * K + (31 - lane)] = key;
    __syncthreads();
    if (warp == 0) {
        int ptr = 0;
        uint32_t head = (lane < nw) ? cand[lane * K] : 0u;
        for (int r = 0; r < K; ++r) {
            const uint32_t win = __reduce_max_sync(0xffffffffu, head);
            if (lane < nw && head == win && win != 0u) {
                ++ptr;
                head = (ptr < K) ? cand[lane * K + ptr] : 0u;
            }
            if (lane == 0) out[r] = win;
        }
    }
    __syncthreads();
}
