// Item-burst microbenchmark of the persistent decode kernel's copy phase on one B200: 28 layer
// regions of 512 packed experts (2,211,840 B each, 31.7 GB), per launch one layer and 10
// experts, 120 of 148 CTAs each copying one 184,320 B group block (8 x 15,360 B units + one
// 61,440 B down slice, nine cp.async.bulk copies on nine mbarriers, no multicast) into shared
// memory. Modes:
//   0 plain
//   1 plain + 15 warps reading shared memory (a separate 16 KB area) while the copies fly
//   2 plain, after the previous launch touched one 32 B word of every 2 MB page of this layer
//   3 the same bytes but contiguous (one 22 MB region, as a standalone burst)
// Per launch: max(end) - min(start) over CTAs from %globaltimer; median over launches 28..83.
// Every wait is bounded (a timeout sets a device flag, reported at the end). Build and run:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o item_burst \
//       moe-offload_b200/microbench/item_burst.cu && ./item_burst
#include <cstdio>
#include <cstdint>
#include <vector>
#include <algorithm>
#include <cuda_runtime.h>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e), __LINE__); return 1; } } while (0)

__device__ __forceinline__ uint64_t gtime() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }
__device__ int g_err;

constexpr int kE = 512, kL = 28, kNG = 12;
constexpr size_t kEB = 2211840, kGB = 184320, kUB = 15360, kDB = 61440;
constexpr size_t kLayerB = (size_t)kE * kEB;

__device__ __forceinline__ int pick(int launch, int k) {   // 10 distinct experts per launch
    const uint32_t h = ((uint32_t)launch * 2654435761u) >> 7;
    return (int)((h + (uint32_t)k * 51u) % (uint32_t)kE);
}

__global__ void __launch_bounds__(512, 1)
burst(const char *buf, int launch, int mode, unsigned long long *stamps, float *sink) {
    extern __shared__ __align__(128) char sm[];
    __shared__ __align__(8) uint64_t bars[9];
    const int c = blockIdx.x, tid = threadIdx.x;
    const int l = launch % kL;
    const char *src;
    if (mode == 3) {
        const size_t span = 120 * kGB, nreg = (kL * kLayerB) / span;
        src = buf + (size_t)(launch % nreg) * span + (size_t)c * kGB;
    } else {
        const int k = c / kNG, G = c % kNG;
        src = buf + (size_t)l * kLayerB + (size_t)pick(launch, k) * kEB + (size_t)G * kGB;
    }
    if (tid == 0) {
        for (int i = 0; i < 9; ++i)
            asm volatile("mbarrier.init.shared.b64 [%0], 1;" :: "r"((unsigned)__cvta_generic_to_shared(&bars[i])));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    __syncthreads();
    const uint64_t t0 = gtime();
    if (c < 120 && tid == 0) {
        for (int u = 0; u < 9; ++u) {
            const uint32_t off = u < 8 ? u * kUB : 8 * kUB;
            const uint32_t n = u < 8 ? kUB : kDB;
            const unsigned b = (unsigned)__cvta_generic_to_shared(&bars[u]);
            asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" :: "r"(b), "r"(n) : "memory");
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                         :: "r"((unsigned)__cvta_generic_to_shared(sm + off)), "l"(src + off), "r"(n), "r"(b) : "memory");
        }
    }
    float acc = 0.f;
    if (mode == 1 && tid >= 32) {
        // shared-memory reads of a separate area (after the 184,320 B region), ~3 us
        const uint4 *a = reinterpret_cast<const uint4 *>(sm + kGB);
        uint32_t x = 0;
#pragma unroll 1
        for (int i = 0; i < 400; ++i) {
            uint4 v;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                         : "r"((unsigned)__cvta_generic_to_shared(a + ((tid + i * 37) & 1023))) : "memory");
            x ^= v.x + v.y + v.z + v.w;
        }
        acc += (float)(x & 1);
        if (x == 0x12345678u) sink[c] = acc;
    }
    uint64_t t1 = t0, tu = t0;
    if (c < 120) {
        for (int u = 0; u < 9; ++u) {
            const unsigned b = (unsigned)__cvta_generic_to_shared(&bars[u]);
            unsigned done = 0;
            for (long it = 0; it < (1L << 24) && !done; ++it)
                asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
                             : "=r"(done) : "r"(b) : "memory");
            if (!done) atomicExch(&g_err, 1);
            if (u == 0) tu = gtime();
        }
        t1 = gtime();
    }
    __syncthreads();
    acc += (float)sm[(tid * 97) % kGB];
    if (tid == 0) {
        stamps[3 * c] = t0;
        stamps[3 * c + 1] = t1;
        stamps[3 * c + 2] = tu;
        sink[c] = acc;
    }
    // mode 2: touch every 2 MB page of the next launch's layer (after this launch's timing)
    if (mode == 2) {
        const char *nxt = buf + (size_t)((launch + 1) % kL) * kLayerB;
        const int npages = (int)((kLayerB + (2u << 20) - 1) / (2u << 20));
        for (int p = c * 512 + tid; p < npages; p += gridDim.x * 512) {
            const size_t off = (size_t)p << 21;
            if (off < kLayerB) acc += (float)__ldcg(nxt + off);
        }
        if (acc == 12345.f) sink[c] = acc;
    }
}

int main() {
    const size_t bytes = (size_t)kL * kLayerB;
    char *buf; CK(cudaMalloc(&buf, bytes));
    CK(cudaMemset(buf, 1, bytes));
    unsigned long long *st; CK(cudaMalloc(&st, 148 * 3 * sizeof(unsigned long long)));
    float *sink; CK(cudaMalloc(&sink, 148 * sizeof(float)));
    const int smem = kGB + 16384;
    CK(cudaFuncSetAttribute(burst, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    std::vector<unsigned long long> h(148 * 3);
    const char *names[] = {"scattered experts", "scattered + smem reads", "scattered, pages touched before", "contiguous 22 MB"};
    int launch = 0;
    for (int rep = 0; rep < 1; ++rep)
    for (int mode = 0; mode < 4; ++mode) {
        std::vector<double> tot, first;
        for (int i = 0; i < 84; ++i, ++launch) {
            burst<<<148, 512, smem>>>(buf, launch, mode, st, sink);
            CK(cudaGetLastError());
            CK(cudaDeviceSynchronize());
            CK(cudaMemcpy(h.data(), st, 148 * 3 * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
            unsigned long long a = ~0ull, b = 0;
            std::vector<double> fu;
            for (int k = 0; k < 120; ++k) { a = std::min(a, h[3 * k]); b = std::max(b, h[3 * k + 1]); fu.push_back((h[3 * k + 2] - h[3 * k]) / 1000.0); }
            std::sort(fu.begin(), fu.end());
            if (i >= 28) { tot.push_back((b - a) / 1000.0); first.push_back(fu[fu.size() / 2]); }
        }
        std::sort(tot.begin(), tot.end());
        std::sort(first.begin(), first.end());
        printf("%-34s all bytes: median %6.2f us (min %6.2f) -> %5.0f GB/s; unit 0 landed (median CTA) %5.2f us\n",
               names[mode], tot[tot.size() / 2], tot[0], 120.0 * kGB / tot[tot.size() / 2] / 1e3, first[first.size() / 2]);
    }
    int e = 0; CK(cudaMemcpyFromSymbol(&e, g_err, sizeof(int)));
    printf("wait timeouts: %d\n", e);
    return 0;
}
