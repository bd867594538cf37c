// Copy-granularity microbenchmark on one B200: N CTAs (120 or 148, one per SM) pull B bytes
// each (184 KB, or 22.1 MB over 148 CTAs) from HBM into shared memory by cp.async.bulk (no
// multicast) in one copy or in 64 / 16 / 4 KB copies from one or 16 issuing lanes, by 16-byte
// cp.async, by ld.global.v4, or by bulk copies for a first part and ld.global.v4 for the rest.
// Every launch reads a fresh region of a 2 GB buffer (cold L2); per launch max(end) - min(start)
// over CTAs from %globaltimer, median over launches 10..59. Every wait is bounded (a timeout sets
// a device flag, reported at the end). Build and run:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o copy_granularity \
//       moe-offload_b200/microbench/copy_granularity.cu && ./copy_granularity
#include <cstdio>
#include <cstdint>
#include <vector>
#include <algorithm>
#include <cuda_runtime.h>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e), __LINE__); return 1; } } while (0)

__device__ __forceinline__ uint64_t gtime() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }

__device__ int g_err;

__global__ void __launch_bounds__(512, 1)
burst(const char *src, size_t region_bytes, int nregions, int launch, int bpc, int mode, int chunk,
      unsigned long long *stamps, float *sink) {
    extern __shared__ __align__(128) char sm[];
    __shared__ __align__(8) uint64_t bar;
    const int r = launch % nregions;
    const char *base = src + (size_t)r * region_bytes + (size_t)blockIdx.x * bpc;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared.b64 [%0], 1;" :: "r"((unsigned)__cvta_generic_to_shared(&bar)));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    __syncthreads();
    uint64_t t0 = gtime();
    const unsigned bar_s = (unsigned)__cvta_generic_to_shared(&bar);
    float acc = 0.f;
    if (mode == 0 || mode == 3) {
        // bulk copies: mode 0 one issuing thread, mode 3 one issuing lane per warp (16 issuers)
        const int issuers = mode == 0 ? 1 : 16;
        const int nchunks = (bpc + chunk - 1) / chunk;
        if (threadIdx.x == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" :: "r"(bar_s), "r"(bpc) : "memory");
        __syncthreads();
        const int issuer = mode == 0 ? (threadIdx.x == 0 ? 0 : -1) : ((threadIdx.x & 31) == 0 ? (int)(threadIdx.x >> 5) : -1);
        if (issuer >= 0) {
            for (int c = issuer; c < nchunks; c += issuers) {
                const int off = c * chunk;
                const int n = min(chunk, bpc - off);
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                             :: "r"((unsigned)__cvta_generic_to_shared(sm + off)), "l"(base + off), "r"(n), "r"(bar_s) : "memory");
            }
        }
        unsigned done = 0;
        for (long it = 0; it < (1L << 24) && !done; ++it)
            asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
                         : "=r"(done) : "r"(bar_s) : "memory");
        if (!done) atomicExch(&g_err, 1);
    } else if (mode == 1) {
        // cp.async 16 B per thread (LDGSTS), all in flight, then one wait
        for (int off = threadIdx.x * 16; off < bpc; off += blockDim.x * 16)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"((unsigned)__cvta_generic_to_shared(sm + off)), "l"(base + off) : "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (mode == 4) {
        // mixed: the first `chunk` bytes by 16 KB bulk copies (one issuer), the rest by ldg.v4
        const int nb = chunk;
        if (threadIdx.x == 0) {
            asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" :: "r"(bar_s), "r"(nb) : "memory");
            for (int off = 0; off < nb; off += 16384) {
                const int n = min(16384, nb - off);
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                             :: "r"((unsigned)__cvta_generic_to_shared(sm + off)), "l"(base + off), "r"(n), "r"(bar_s) : "memory");
            }
        }
        const int stride = blockDim.x * 16;
        for (int off0 = nb + threadIdx.x * 16; off0 < bpc; off0 += stride * 8) {
            int4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int off = off0 + u * stride;
                if (off < bpc) asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w) : "l"(base + off));
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int off = off0 + u * stride;
                if (off < bpc) *reinterpret_cast<int4 *>(sm + off) = v[u];
            }
        }
        unsigned done = 0;
        for (long it = 0; it < (1L << 24) && !done; ++it)
            asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
                         : "=r"(done) : "r"(bar_s) : "memory");
        if (!done) atomicExch(&g_err, 1);
    } else {
        // ld.global.v4 by all threads, 8 loads in flight per thread, stored to shared memory
        const int stride = blockDim.x * 16;
        for (int off0 = threadIdx.x * 16; off0 < bpc; off0 += stride * 8) {
            int4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int off = off0 + u * stride;
                if (off < bpc) asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w) : "l"(base + off));
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int off = off0 + u * stride;
                if (off < bpc) *reinterpret_cast<int4 *>(sm + off) = v[u];
            }
        }
    }
    __syncthreads();
    uint64_t t1 = gtime();
    acc += (float)sm[(threadIdx.x * 97) % bpc];
    if (threadIdx.x == 0) {
        stamps[2 * blockIdx.x] = t0;
        stamps[2 * blockIdx.x + 1] = t1;
        sink[blockIdx.x] = acc;
    }
}

int main() {
    const size_t buf = 2ull << 30;
    char *src; CK(cudaMalloc(&src, buf));
    CK(cudaMemset(src, 1, buf));
    unsigned long long *st; CK(cudaMalloc(&st, 148 * 2 * sizeof(unsigned long long)));
    float *sink; CK(cudaMalloc(&sink, 148 * sizeof(float)));
    const int smem = 200 * 1024;
    CK(cudaFuncSetAttribute(burst, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    struct Cfg { int nctas, bpc, mode, chunk; const char *name; };
    const int b120 = 188416;           // 184 KB (one c1 item)
    const int b148 = 149440;           // 22.1 MB over 148 CTAs
    std::vector<Cfg> cfgs = {
        {120, b120, 0, 188416, "bulk 1 copy"}, {120, b120, 0, 65536, "bulk 64K"}, {120, b120, 0, 16384, "bulk 16K"},
        {120, b120, 0, 4096, "bulk 4K"}, {120, b120, 3, 4096, "bulk 4K x16 issuers"}, {120, b120, 1, 16, "cp.async 16B"},
        {120, b120, 2, 16, "ldg.v4 x8"},
        {148, b148, 0, 65536, "bulk 64K"}, {148, b148, 0, 16384, "bulk 16K"}, {148, b148, 0, 4096, "bulk 4K"},
        {148, b148, 3, 4096, "bulk 4K x16 issuers"}, {148, b148, 1, 16, "cp.async 16B"}, {148, b148, 2, 16, "ldg.v4 x8"},
        {148, b120, 0, 16384, "bulk 16K (27.9 MB)"},
        {120, b120, 4, 98304, "bulk 96K + ldg rest"}, {120, b120, 4, 131072, "bulk 128K + ldg rest"},
        {148, b148, 4, 81920, "bulk 80K + ldg rest"},
    };
    std::vector<unsigned long long> h(148 * 2);
    int launch = 0;
    for (auto &c : cfgs) {
        const size_t region = (size_t)c.nctas * c.bpc;
        const int nregions = (int)(buf / region);
        std::vector<double> us;
        for (int i = 0; i < 60; ++i, ++launch) {
            burst<<<c.nctas, 512, smem>>>(src, region, nregions, launch, c.bpc, c.mode, c.chunk, st, sink);
            CK(cudaGetLastError());
            CK(cudaDeviceSynchronize());
            CK(cudaMemcpy(h.data(), st, c.nctas * 2 * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
            unsigned long long a = ~0ull, b = 0;
            for (int k = 0; k < c.nctas; ++k) { a = std::min(a, h[2 * k]); b = std::max(b, h[2 * k + 1]); }
            if (i >= 10) us.push_back((b - a) / 1000.0);
        }
        std::sort(us.begin(), us.end());
        const double med = us[us.size() / 2];
        printf("%3d CTAs x %6d B  %-22s median %6.2f us  min %6.2f  -> %6.0f GB/s\n", c.nctas, c.bpc, c.name, med,
               us[0], region / med / 1e3);
    }
    int e = 0; CK(cudaMemcpyFromSymbol(&e, g_err, sizeof(int)));
    printf("wait timeouts: %d\n", e);
    return 0;
}
