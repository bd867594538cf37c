// Issue-rate microbenchmark of tcgen05.mma (kind::f16, cta_group::1, M = 128) on one B200, run
// on 148 CTAs (one per SM) with one issuing lane each. Two measurements:
//   1. back-to-back MMAs of N = 16 .. 256 into 1 .. 8 accumulators, A from TMEM or shared memory
//   2. the prefill GEMM's per-K-block pattern: 8 MMAs (two accumulators, A in 4 TMEM stages,
//      B in 8 shared-memory stages) followed by 0 / 1 / 2 commits, issued by one lane or by a
//      whole warp's loop with mbarrier waits, with zero or random operands
//   3. cta_group::2 on CTA pairs (clusters of 2, 74 pairs): M = 256 (128 rows in each CTA's
//      TMEM), N = 32 .. 256, issued by the even CTA; and the same K-block pattern as 2. with
//      M = 256, N = 64, each commit sent to both CTAs' mbarriers (two plain commits, the
//      second to the peer's barrier through mapa)
//   4. hand-off latencies: tcgen05.commit -> the mbarrier phase seen by the issuing thread,
//      with 0 or 8 MMAs (N = 64) in flight; an mbarrier ping-pong between two warps of a CTA,
//      and between the two CTAs of a pair (remote arrive on the peer's barrier)
// Every wait is bounded (a timeout sets a device flag, reported at the end). Build and run:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o tcgen05_issue_rate \
//       moe-offload_b200/microbench/tcgen05_issue_rate.cu && ./tcgen05_issue_rate
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <cuda_runtime.h>

__device__ unsigned int g_err;
__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t desc_sw128(uint32_t a) {
    return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
__host__ __device__ constexpr uint32_t idesc(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t id) {
    asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1;\n" ::"r"(d), "r"(a), "l"(b), "r"(id));
}
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t id) {
    asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1;\n" ::"r"(d), "l"(a), "l"(b), "r"(id));
}
template <int N, int R, bool ATMEM>
__global__ void __launch_bounds__(128) rate(int iters, long long *out) {
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char *base = (unsigned char *)(((uintptr_t)sm + 1023) & ~(uintptr_t)1023);
    unsigned char *A = base, *B = base + 16384;
    __shared__ uint64_t bar;
    __shared__ uint32_t tslot;
    for (int i = threadIdx.x; i < 48 * 1024 / 4; i += blockDim.x) ((uint32_t *)base)[i] = 0;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&bar)));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(saddr(&tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tm = tslot;
    if (threadIdx.x == 0) {
        constexpr uint32_t id = idesc(128, N);
        uint64_t bd[4], ad[4];
        for (int j = 0; j < 4; ++j) { bd[j] = desc_sw128(saddr(B) + 32u * j); ad[j] = desc_sw128(saddr(A) + 32u * j); }
        long long t0 = clock64();
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if constexpr (ATMEM) mma_ts(tm + r * N, tm + 384u + 8u * j, bd[j], id);
                    else mma_ss(tm + r * N, ad[j], bd[j], id);
                }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(&bar)) : "memory");
        uint32_t ok = 0;
        for (uint32_t i = 0; i < (1u << 26) && !ok; ++i)
            asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
                         : "=r"(ok) : "r"(saddr(&bar)) : "memory");
        long long t1 = clock64();
        if (!ok) atomicOr(&g_err, 1u);
        out[blockIdx.x] = t1 - t0;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tm));
}

template <int N, int R, bool AT>
void run_rate(long long *d) {
    const int smem = 48 * 1024 + 1024, iters = 64;
    cudaFuncSetAttribute(rate<N, R, AT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    rate<N, R, AT><<<148, 128, smem>>>(iters, d);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); exit(1); }
    long long h[148];
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double avg = 0;
    for (int i = 0; i < 148; ++i) avg += h[i];
    avg /= 148;
    const double per = avg / (iters * 4.0 * R);
    printf("%s N %3d R %d: %.1f cycles/mma, %.0f MAC/clk/SM\n", AT ? "A-tmem" : "A-smem", N, R, per, 128.0 * N * 16 / per);
}


__device__ __forceinline__ void mma_ts_acc(uint32_t d, uint32_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
                 ::"r"(d), "r"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar)) : "memory");
}
template <int C, bool MMA, int F = 0, bool RND = false>
__global__ void __launch_bounds__(128) kblock(int nkb, long long *out) {
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char *base = (unsigned char *)(((uintptr_t)sm + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bars[16];
    __shared__ uint64_t fin;
    __shared__ uint32_t tslot;
    for (int i = threadIdx.x; i < 8 * 8192 / 4; i += blockDim.x) {
        uint32_t h = (uint32_t)i * 2654435761u ^ 0x9E3779B9u;
        h ^= h >> 13; h *= 0x85EBCA6Bu; h ^= h >> 16;
        // two bf16 of magnitude in [2^-4, 2^4) with random signs and mantissas
        const uint32_t lo = 0x3B00u + (h & 0x7FFu) + ((h >> 11) & 1u) * 0x8000u;
        const uint32_t hi = 0x3B00u + ((h >> 12) & 0x7FFu) + ((h >> 23) & 1u) * 0x8000u;
        ((uint32_t *)base)[i] = RND ? (lo | (hi << 16)) : 0u;
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < 16; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&bars[i])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&fin)));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(saddr(&tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tm = tslot;
    if (threadIdx.x < 32) {
        const bool l0 = threadIdx.x == 0;
        constexpr uint32_t id = idesc(128, 48);
        long long t0 = clock64();
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb & 3, sb = kb & 7;
            const uint32_t at = tm + 256u + 64u * s;
            const uint32_t b0 = saddr(base + 8192 * sb);
            if (F & 1) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (F & 4) {   // a wait on an mbarrier phase that completed long ago
                uint32_t ok = 0;
                asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 1;\n selp.u32 %0, 1, 0, p;\n}\n"
                             : "=r"(ok) : "r"(saddr(&fin)) : "memory");
                if (!ok) atomicOr(&g_err, 2u);
            }
            if (l0 && MMA) {
#pragma unroll
                for (int mm = 0; mm < 2; ++mm)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        mma_ts_acc(tm + 128u * mm, at + 32u * mm + 8u * j, desc_sw128(b0 + 32u * j), id, (kb | j) != 0);
                    }
            }
            if (l0 && C >= 1) commit(&bars[s]);
            if (l0 && C >= 2) commit(&bars[8 + sb]);
            if (F & 2) __syncwarp();
        }
        if (l0) commit(&fin);
        uint32_t ok = 0;
        for (uint32_t i = 0; i < (1u << 26) && !ok; ++i)
            asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
                         : "=r"(ok) : "r"(saddr(&fin)) : "memory");
        long long t1 = clock64();
        if (!ok) atomicOr(&g_err, 1u);
        if (l0) out[blockIdx.x] = t1 - t0;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tm));
}
template <int C, bool MMA, int F = 0, bool RND = false>
void run_kblock(long long *d) {
    const int smem = 8 * 8192 + 1024, nkb = 512;
    cudaFuncSetAttribute(kblock<C, MMA, F, RND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kblock<C, MMA, F, RND><<<148, 128, smem>>>(nkb, d);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); exit(1); }
    long long h[148];
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double avg = 0;
    for (int i = 0; i < 148; ++i) avg += h[i];
    printf("commits/kblock %d mma %d flags %d random %d: %.1f cycles per K-block\n", C, MMA, F, (int)RND, avg / 148 / nkb);
}

// ------------------------------------------------------------------ cta_group::2
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
    uint32_t p;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(p) : "r"(local), "r"(rank));
    return p;
}
__device__ __forceinline__ void mma2_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
                 ::"r"(d), "r"(a), "l"(b), "r"(id), "r"(acc));
}
// commit to a shared::cluster mbarrier address (this CTA's or, through mapa, the peer's)
__device__ __forceinline__ void commit2(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool wait_parity(uint64_t *bar, uint32_t par) {
    uint32_t ok = 0;
    for (uint32_t i = 0; i < (1u << 26) && !ok; ++i)
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                     : "=r"(ok) : "r"(saddr(bar)), "r"(par) : "memory");
    return ok != 0;
}

// KB = 0: R x 4 back-to-back MMAs of M = 256 x N per iteration; KB > 0: the K-block pattern
// (8 MMAs of N into two accumulators, A in 4 TMEM stages, B in 8 shared stages) with KB - 1
// commit pairs per K-block
template <int N, int R, int KB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128) rate2(int iters, long long *out) {
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char *base = (unsigned char *)(((uintptr_t)sm + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bars[16];
    __shared__ uint64_t fin;
    __shared__ uint32_t tslot;
    for (int i = threadIdx.x; i < 8 * 8192 / 4; i += blockDim.x) ((uint32_t *)base)[i] = 0;
    const uint32_t rank = cluster_rank();
    if (threadIdx.x == 0) {
        for (int i = 0; i < 16; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&bars[i])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&fin)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(saddr(&tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    cluster_sync_all();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tm = tslot;
    if (threadIdx.x == 0) {
        long long t0 = clock64();
        if (rank == 0) {
            if constexpr (KB == 0) {
                constexpr uint32_t id = idesc(256, N);
                uint64_t bd[4];
                for (int j = 0; j < 4; ++j) bd[j] = desc_sw128(saddr(base) + 32u * j);
                for (int it = 0; it < iters; ++it) {
#pragma unroll
                    for (int r = 0; r < R; ++r)
#pragma unroll
                        for (int j = 0; j < 4; ++j) mma2_ts(tm + r * N, tm + 384u + 8u * j, bd[j], id, 1u);
                }
            } else {
                constexpr uint32_t id = idesc(256, N);
                for (int kb = 0; kb < iters; ++kb) {
                    const int s = kb & 3, sb = kb & 7;
                    const uint32_t at = tm + 256u + 64u * s;
                    const uint32_t b0 = saddr(base + 8192 * sb);
#pragma unroll
                    for (int mm = 0; mm < 2; ++mm)
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            mma2_ts(tm + 128u * mm, at + 32u * mm + 8u * j, desc_sw128(b0 + 32u * j), id, (kb | j) != 0);
                    if (KB >= 2) {
                        commit2(saddr(&bars[s]));
                        commit2(peer_addr(saddr(&bars[s]), 1));
                    }
                    if (KB >= 3) {
                        commit2(saddr(&bars[8 + sb]));
                        commit2(peer_addr(saddr(&bars[8 + sb]), 1));
                    }
                }
            }
            commit2(saddr(&fin));
            commit2(peer_addr(saddr(&fin), 1));
        }
        const bool ok = wait_parity(&fin, 0);
        long long t1 = clock64();
        if (!ok) atomicOr(&g_err, 4u);
        out[blockIdx.x] = t1 - t0;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    cluster_sync_all();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x < 32) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tm));
}

template <int N, int R, int KB>
void run_rate2(long long *d) {
    const int smem = 8 * 8192 + 1024, iters = KB ? 512 : 64;
    cudaFuncSetAttribute(rate2<N, R, KB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    rate2<N, R, KB><<<148, 128, smem>>>(iters, d);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); exit(1); }
    long long h[148];
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double avg = 0;
    for (int i = 0; i < 148; i += 2) avg += h[i];
    avg /= 74;
    if (KB == 0) {
        const double per = avg / (iters * 4.0 * R);
        printf("cta_group::2 A-tmem M 256 N %3d R %d: %.1f cycles/mma, %.0f MAC/clk per SM\n", N, R, per,
               128.0 * N * 16 / per);
    } else {
        printf("cta_group::2 K-block (8 MMAs M 256 N %d) + %d commit pairs: %.1f cycles per K-block\n", N, KB - 1,
               avg / iters);
    }
}

// ------------------------------------------------------------------ hand-off latencies
__device__ __forceinline__ void arrive_local(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// commit latency: thread 0 issues NM MMAs (0 or 8) then a commit and waits for the phase
template <int NM>
__global__ void __launch_bounds__(128) commit_lat(int reps, long long *out) {
    extern __shared__ __align__(1024) unsigned char sm[];
    unsigned char *base = (unsigned char *)(((uintptr_t)sm + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar;
    __shared__ uint32_t tslot;
    for (int i = threadIdx.x; i < 16 * 1024 / 4; i += blockDim.x) ((uint32_t *)base)[i] = 0;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&bar)));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(saddr(&tslot)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tm = tslot;
    if (threadIdx.x == 0) {
        constexpr uint32_t id = idesc(128, 64);
        long long tot = 0;
        bool allok = true;
        for (int r = 0; r < reps; ++r) {
            long long t0 = clock64();
#pragma unroll
            for (int i = 0; i < NM; ++i) mma_ts_acc(tm + 128u * (i >> 2), tm + 256u + 8u * (i & 3), desc_sw128(saddr(base) + 32u * (i & 3)), id, 1u);
            commit(&bar);
            allok &= wait_parity(&bar, (uint32_t)(r & 1));
            tot += clock64() - t0;
        }
        if (!allok) atomicOr(&g_err, 8u);
        out[blockIdx.x] = tot / reps;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tm));
}

// ping-pong: lane 0 of warp 0 arrives on `ping` and waits on `pong`; lane 0 of the partner
// (warp 1 of the same CTA, or warp 0 of the pair's other CTA) waits on `ping` and arrives on
// `pong`. Reports one round trip (two hand-offs).
template <bool PAIR>
__global__ void __launch_bounds__(64) pingpong(int reps, long long *out) {
    __shared__ uint64_t ping, pong;
    uint32_t rank = 0;
    if (PAIR) rank = cluster_rank();
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&ping)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(saddr(&pong)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (PAIR) cluster_sync_all();
    const bool initiator = PAIR ? (rank == 0 && threadIdx.x == 0) : threadIdx.x == 0;
    const bool partner = PAIR ? (rank == 1 && threadIdx.x == 0) : threadIdx.x == 32;
    if (initiator) {
        // PAIR: ping lives in the partner CTA, pong here
        const uint32_t ping_addr = PAIR ? peer_addr(saddr(&ping), 1) : saddr(&ping);
        long long t0 = clock64();
        bool ok = true;
        for (int r = 0; r < reps; ++r) {
            if (PAIR) arrive_remote(ping_addr);
            else arrive_local(&ping);
            ok &= wait_parity(&pong, (uint32_t)(r & 1));
        }
        if (!ok) atomicOr(&g_err, 16u);
        out[blockIdx.x] = (clock64() - t0) / reps;
    } else if (partner) {
        const uint32_t pong_addr = PAIR ? peer_addr(saddr(&pong), 0) : saddr(&pong);
        bool ok = true;
        for (int r = 0; r < reps; ++r) {
            ok &= wait_parity(&ping, (uint32_t)(r & 1));
            if (PAIR) arrive_remote(pong_addr);
            else arrive_local(&pong);
        }
        if (!ok) atomicOr(&g_err, 32u);
    }
    __syncthreads();
    if (PAIR) cluster_sync_all();
}

template <int NM>
void run_commit_lat(long long *d) {
    const int smem = 16 * 1024 + 1024, reps = 256;
    cudaFuncSetAttribute(commit_lat<NM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    commit_lat<NM><<<148, 128, smem>>>(reps, d);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); exit(1); }
    long long h[148];
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double avg = 0;
    for (int i = 0; i < 148; ++i) avg += h[i];
    printf("commit -> phase seen by the issuer, %d MMAs before it: %.0f cycles\n", NM, avg / 148);
}

void run_pingpong(long long *d, bool pair) {
    const int reps = 1024;
    if (pair) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(148);
        cfg.blockDim = dim3(64);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, pingpong<true>, reps, d);
    } else {
        pingpong<false><<<148, 64>>>(reps, d);
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { printf("error %s\n", cudaGetErrorString(e)); exit(1); }
    long long h[148];
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double avg = 0;
    int n = 0;
    for (int i = 0; i < 148; i += pair ? 2 : 1, ++n) avg += h[i];
    printf("mbarrier ping-pong round trip, %s: %.0f cycles\n", pair ? "two CTAs of a pair (remote arrive)" : "two warps of a CTA", avg / n);
}

int main() {
    long long *d;
    cudaMalloc(&d, 148 * sizeof(long long));
    run_rate<40, 1, true>(d); run_rate<40, 4, true>(d); run_rate<40, 8, true>(d);
    run_rate<64, 1, true>(d); run_rate<64, 4, true>(d); run_rate<16, 8, true>(d);
    run_rate<128, 1, true>(d); run_rate<128, 2, true>(d); run_rate<256, 1, true>(d);
    run_rate<40, 1, false>(d); run_rate<64, 4, false>(d); run_rate<128, 2, false>(d); run_rate<256, 1, false>(d);
    run_kblock<0, true, 0>(d); run_kblock<1, true, 0>(d); run_kblock<2, true, 0>(d);
    run_kblock<2, true, 0, true>(d);
    run_kblock<2, true, 2>(d); run_kblock<2, true, 7>(d); run_kblock<2, false, 7>(d);
    run_rate2<32, 8, 0>(d); run_rate2<64, 1, 0>(d); run_rate2<64, 4, 0>(d); run_rate2<128, 2, 0>(d);
    run_rate2<256, 1, 0>(d);
    run_rate2<64, 1, 1>(d); run_rate2<64, 1, 2>(d); run_rate2<64, 1, 3>(d);
    run_commit_lat<0>(d); run_commit_lat<8>(d);
    run_pingpong(d, false); run_pingpong(d, true);
    unsigned int err = 0;
    cudaMemcpyFromSymbol(&err, g_err, 4);
    printf("device error word %u (0: every wait completed)\n", err);
    return err != 0;
}
