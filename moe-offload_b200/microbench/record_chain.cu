// Record-chain microbenchmark on one B200 (148 CTAs x 512 threads, one per SM): how long one
// warp's short LDS + shuffle chain (the data movement of the decode kernel's activation record)
// takes while the other 15 warps are parked at bar.sync or spin on an mbarrier, with or without
// 184 KB of cp.async.bulk copies (no multicast) landing in shared memory. Every wait is bounded
// (a timeout sets a device flag, reported at the end). Build and run:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o record_chain \
//       moe-offload_b200/microbench/record_chain.cu && ./record_chain
#include <cstdio>
#include <cstdint>
#include <vector>
#include <algorithm>
#include <cuda_runtime.h>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e), __LINE__); return 1; } } while (0)
__device__ __forceinline__ uint64_t gtime() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }
__device__ int g_err;

__device__ __forceinline__ bool try_wait(unsigned bar, unsigned parity) {
    unsigned ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok;
}

// the record's data movement: one LDS, 4 dependent shuffle pairs, 8 independent shuffles
__device__ __noinline__ uint32_t chain(const uint2 *sact) {
    const int lane = threadIdx.x & 31;
    const uint2 q = sact[lane & 15];
    float mx = __uint_as_float(q.x << 16), sm = __uint_as_float(q.y & 0xffff0000u);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        sm += __shfl_xor_sync(0xffffffffu, sm, off);
    }
    uint32_t acc = __float_as_uint(mx) ^ __float_as_uint(sm);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        acc ^= __shfl_sync(0xffffffffu, q.x, (lane & 16) + j);
        acc += __shfl_sync(0xffffffffu, q.y, (lane & 16) + 4 + j);
    }
    return acc;
}

__global__ void __launch_bounds__(512, 1)
mio(const char *src, size_t region, int nreg, int launch, int mode, unsigned long long *out, uint32_t *sink) {
    extern __shared__ __align__(128) char smem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ uint2 sact[16];
    const int tid = threadIdx.x, warp = tid >> 5;
    const bool copies = mode & 1, spin = mode & 2;
    const unsigned b0 = (unsigned)__cvta_generic_to_shared(&bars[0]);   // copy barrier
    const unsigned b1 = (unsigned)__cvta_generic_to_shared(&bars[1]);   // "record done" barrier
    if (tid == 0) {
        asm volatile("mbarrier.init.shared.b64 [%0], 1;" :: "r"(b0));
        asm volatile("mbarrier.init.shared.b64 [%0], 1;" :: "r"(b1));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    if (tid < 16) sact[tid] = make_uint2(0x3f803f80u + tid, 0x40004000u + tid);
    __syncthreads();
    const char *base = src + (size_t)(launch % nreg) * region + (size_t)blockIdx.x * 188416;
    if (tid == 0 && copies) {
        asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" :: "r"(b0), "r"(188416) : "memory");
        for (int u = 0; u < 4; ++u)
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                         :: "r"((unsigned)__cvta_generic_to_shared(smem + u * 47104)), "l"(base + u * 47104), "r"(47104), "r"(b0) : "memory");
    }
    uint32_t acc = 0;
    if (warp == 0) {
        // four timed record chains
        for (int r = 0; r < 4; ++r) {
            const uint64_t t0 = gtime();
            acc += chain(sact);
            __syncwarp();
            const uint64_t t1 = gtime();
            if (tid == 0) out[blockIdx.x * 4 + r] = t1 - t0;
        }
        if (tid == 0) asm volatile("mbarrier.arrive.shared.b64 _, [%0];" :: "r"(b1) : "memory");
    } else if (spin) {
        bool done = false;
        for (long it = 0; it < (1L << 22) && !done; ++it) done = try_wait(b1, 0);
        if (!done) atomicExch(&g_err, 1);
    }
    __syncthreads();
    if (copies) {
        bool done = false;
        for (long it = 0; it < (1L << 24) && !done; ++it) done = try_wait(b0, 0);
        if (!done) atomicExch(&g_err, 2);
    }
    if (acc == 0x9e3779b9u) sink[blockIdx.x] = acc;
}

int main() {
    const size_t buf = 2ull << 30, region = 148ull * 188416;
    const int nreg = (int)(buf / region);
    char *src; CK(cudaMalloc(&src, buf));
    CK(cudaMemset(src, 1, buf));
    unsigned long long *out; CK(cudaMalloc(&out, 148 * 4 * sizeof(unsigned long long)));
    uint32_t *sink; CK(cudaMalloc(&sink, 148 * sizeof(uint32_t)));
    CK(cudaFuncSetAttribute(mio, cudaFuncAttributeMaxDynamicSharedMemorySize, 188416));
    const char *names[] = {"others at bar.sync", "others at bar.sync + 184 KB landing", "others spinning try_wait",
                           "others spinning + 184 KB landing"};
    std::vector<unsigned long long> h(148 * 4);
    int launch = 0;
    for (int mode = 0; mode < 4; ++mode) {
        std::vector<double> first, later;
        for (int i = 0; i < 40; ++i, ++launch) {
            mio<<<148, 512, 188416>>>(src, region, nreg, launch, mode, out, sink);
            CK(cudaGetLastError());
            CK(cudaDeviceSynchronize());
            CK(cudaMemcpy(h.data(), out, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
            if (i < 5) continue;
            for (int c = 0; c < 148; ++c) { first.push_back(h[c * 4] / 1000.0); later.push_back(h[c * 4 + 3] / 1000.0); }
        }
        std::sort(first.begin(), first.end());
        std::sort(later.begin(), later.end());
        printf("%-40s record chain: 1st %5.3f us (p90 %5.3f), 4th %5.3f us (p90 %5.3f)\n", names[mode],
               first[first.size() / 2], first[first.size() * 9 / 10], later[later.size() / 2], later[later.size() * 9 / 10]);
    }
    int e = 0; CK(cudaMemcpyFromSymbol(&e, g_err, sizeof(int)));
    printf("wait timeouts: %d\n", e);
    return 0;
}
