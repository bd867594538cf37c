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

