// Expert-parallel decode of one MoE layer across the GPUs of one node (one process per GPU).
//
// Rank r of N holds experts [e0, e0 + n) of every layer (contiguous blocks of E/N) and the
// whole router (3 MB per layer at E 512, H 3072: reading it costs less than the collective
// latency an all-gather of sharded logits would add, and every rank then routes the batch
// identically, bit for bit). Per layer, on every rank:
//
//   router        the full router over the T rows, exact softmax / MLX-order top-k, int8 MMA
//                 records of the (normalised) input for the expert kernels
//   gate/up       the T*K routed (token, expert) slots whose expert is local; the others are
//                 skipped (slot id outside [e0, e0 + n))
//   down          unweighted expert outputs yk [T][K][H] (bf16, zero where not local)
//   exchange +    ONE kernel: every rank stores its owned yk rows straight into every rank's
//   combine       receive buffer over NVLink (peer pointers from CUDA IPC), signals with a
//                 release store of its epoch into each peer's flag word, waits (bounded) until
//                 every rank has signalled, then combines y = bf16(resid + sum_k bf16(yk * s))
//                 sequentially in MLX order -- the same bits on every rank and the same bits
//                 as the single-GPU decode layer (every slot has exactly one writer).
//
// Receive buffers are double-buffered by epoch parity: a rank can only start writing epoch
// e + 2 into a buffer after every rank has signalled e + 1, which each rank does only after
// its kernel for epoch e (the last reader of that parity) has finished.
//
// Batches of kEpGemmT tokens or more run the local experts as the prefill path's grouped
// tensor-core GEMMs (each routed expert's weights read once for all of its tokens; the
// arithmetic of moe_prefill_layer), smaller batches as per-slot int8 GEMVs (the arithmetic of
// moe_decode_layer); the exchange and combine are the same.
//
// Reference semantics: the decode body of the reference's hook (mlx-qwen38/loader.py:903-922)
// with the experts split across devices, as the expert-parallel configuration asks; the
// reference itself runs on one device.
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kMaxRanks = 16;
constexpr int kExThreads = 512;
constexpr unsigned long long kPeerWaitNs = 2000000000ull;   // a peer that has not signalled in 2 s is lost
constexpr size_t kHeaderBytes = 256;

struct EpHeader {
    unsigned long long flags[kMaxRanks];   // the epoch each rank last signalled into this buffer
    unsigned int arrive;                    // CTAs of the running exchange that have stored
    unsigned int epoch;                     // exchanges this rank has completed
};
static_assert(sizeof(EpHeader) <= kHeaderBytes, "header size");

MOE_HD size_t recv_bytes(int T, int K, int H) { return al256((size_t)T * K * H * 2); }

struct ExArgs {
    unsigned char *const *peers;   // [nranks] exchange buffers; peers[rank] is this rank's
    int rank, nranks, T, K, H;
    uint32_t e0, n;                // local experts [e0, e0 + n)
    const uint32_t *inds;          // [T][K]
    const uint16_t *scores;        // [T][K]
    const uint16_t *yk;            // [T][K][H]
    const uint16_t *resid;         // [T][H] or null
    uint16_t *y;                   // [T][H]
};

MOE_D unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

MOE_D unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

MOE_D void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Cooperative launch (all CTAs co-resident: the last one to store signals for the rank).
__global__ void __launch_bounds__(kExThreads) exchange_combine_kernel(ExArgs a) {
    unsigned char *own = a.peers[a.rank];
    EpHeader *hdr = reinterpret_cast<EpHeader *>(own);
    __shared__ unsigned int s_epoch;
    if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned int *>(&hdr->epoch) + 1u;
    __syncthreads();
    const unsigned int e = s_epoch;
    const size_t par_off = kHeaderBytes + (size_t)(e & 1u) * recv_bytes(a.T, a.K, a.H);
    const int cpr = a.H / 8;                     // 16-byte chunks per row
    const size_t nwork = (size_t)a.T * a.K * cpr;
    const size_t stride = (size_t)gridDim.x * blockDim.x;

    // owned rows -> every rank's receive buffer (this rank's included); only threads that
    // stored need the system-scope fence that orders their stores before the signal
    bool stored = false;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nwork; i += stride) {
        const size_t row = i / cpr;
        const int c = (int)(i % cpr);
        if (a.inds[row] - a.e0 >= a.n) continue;
        const uint4 v = *reinterpret_cast<const uint4 *>(a.yk + row * a.H + (size_t)c * 8);
        const size_t off = par_off + (row * a.H + (size_t)c * 8) * 2;
        for (int p = 0; p < a.nranks; ++p) *reinterpret_cast<uint4 *>(a.peers[p] + off) = v;
        stored = true;
    }
    if (stored) __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int old = atomicAdd(&hdr->arrive, 1u);
        if (old + 1u == gridDim.x) {             // the last CTA: every store of this rank is done
            hdr->arrive = 0u;
            hdr->epoch = e;
            __threadfence_system();
            for (int p = 0; p < a.nranks; ++p)
                st_release_sys(&reinterpret_cast<EpHeader *>(a.peers[p])->flags[a.rank], e);
        }
        const unsigned long long t0 = globaltimer_ns();
        for (int q = 0; q < a.nranks; ++q) {
#pragma unroll 1
            while (ld_acquire_sys(&hdr->flags[q]) < e) {
                if (globaltimer_ns() - t0 > kPeerWaitNs) {
                    atomicOr(&g_moe_device_error, MOE_DEVERR_PEER_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();

    // combine: sequential bf16 sum over k in MLX order, then the residual
    const uint16_t *recv = reinterpret_cast<const uint16_t *>(own + par_off);
    const size_t n = (size_t)a.T * a.H;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t t = i / a.H, h = i % a.H;
        float acc = 0.f;
        for (int k = 0; k < a.K; ++k) {
            const float yv = bf16_bits_to_f32(__ldcg(recv + (t * a.K + k) * a.H + h));
            const float pk = bf16r(yv * bf16_bits_to_f32(a.scores[t * a.K + k]));
            acc = (k == 0) ? pk : bf16r(acc + pk);
        }
        if (a.resid) acc = bf16r(bf16_bits_to_f32(a.resid[i]) + acc);
        a.y[i] = f32_to_bf16_bits(acc);
    }
}

// batches of at least this many tokens run the local experts as grouped tensor-core GEMMs
// (each routed expert's weights read once for all its tokens) instead of per-slot GEMVs
constexpr int kEpGemmT = 32;

struct EpWs {
    unsigned int *tickets;
    uint16_t *logits;
    uint2 *xrec;
    float *xscale, *xsum;
    uint16_t *act;
    uint2 *arec;
    float *ascale, *asum;
    unsigned int *acnt;
    uint16_t *yk;
    uint16_t *xn;            // normalised rows (GEMM path)
    void *pws;               // grouped-GEMM workspace (GEMM path)
    size_t pws_bytes;
    size_t bytes;
};

EpWs carve(void *base, int T, int H, int I, int E, int K) {
    EpWs w{};
    const int ngH = H / 64, ngI = I / 64;
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t n) { char *q = p ? p + off : nullptr; off += al256(n); return q; };
    w.tickets = reinterpret_cast<unsigned int *>(take((size_t)T * 4));
    w.acnt = reinterpret_cast<unsigned int *>(take((size_t)T * K * ngI * 4));
    w.logits = reinterpret_cast<uint16_t *>(take((size_t)T * E * 2));
    w.xrec = reinterpret_cast<uint2 *>(take((size_t)T * ngH * 128));
    w.xscale = reinterpret_cast<float *>(take((size_t)T * pad4(ngH) * 4));
    w.xsum = reinterpret_cast<float *>(take((size_t)T * pad4(ngH) * 4));
    w.act = reinterpret_cast<uint16_t *>(take((size_t)T * K * I * 2));
    w.arec = reinterpret_cast<uint2 *>(take((size_t)T * K * ngI * 128));
    w.ascale = reinterpret_cast<float *>(take((size_t)T * pad4(K * ngI) * 4));
    w.asum = reinterpret_cast<float *>(take((size_t)T * pad4(K * ngI) * 4));
    w.yk = reinterpret_cast<uint16_t *>(take((size_t)T * K * H * 2));
    if (T >= kEpGemmT) {
        w.xn = reinterpret_cast<uint16_t *>(take((size_t)T * H * 2));
        w.pws_bytes = moe_prefill_workspace_bytes(T, H, I, E, K);
        w.pws = take(w.pws_bytes);
    }
    w.bytes = off;
    return w;
}

}  // namespace

extern "C" size_t moe_ep_buffer_bytes(int T, int K, int H) {
    if (T <= 0 || K <= 0 || H <= 0) return 0;
    return kHeaderBytes + 2 * recv_bytes(T, K, H);
}

extern "C" int moe_ep_buffer_alloc(size_t bytes, void **out_ptr, void *out_handle) {
    if (!out_ptr || !out_handle || bytes < kHeaderBytes) return moe_set_error(MOE_EINVAL, "ep_buffer_alloc: bad arguments");
    void *p = nullptr;
    MOE_CUDA_TRY(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return moe_set_cuda_error(e);
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == MOE_EP_HANDLE_BYTES, "IPC handle size");
    memcpy(out_handle, &h, sizeof(h));
    *out_ptr = p;
    return MOE_OK;
}

extern "C" int moe_ep_buffer_open(const void *handle, void **out_ptr) {
    if (!handle || !out_ptr) return moe_set_error(MOE_EINVAL, "ep_buffer_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    MOE_CUDA_TRY(cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return MOE_OK;
}

extern "C" int moe_ep_buffer_close(void *ptr) {
    if (ptr) MOE_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return MOE_OK;
}

extern "C" int moe_ep_buffer_free(void *ptr) {
    if (ptr) MOE_CUDA_TRY(cudaFree(ptr));
    return MOE_OK;
}

extern "C" size_t moe_ep_workspace_bytes(int T, int H, int I, int E, int K) {
    if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || K <= 0) return 0;
    return carve(nullptr, T, H, I, E, K).bytes;
}

extern "C" int moe_ep_decode_layer(const void *x, int T, int H, int I, int E, int K, int e_begin, int e_count,
                                   const void *router_w, const uint32_t *wg, const void *sg, const void *bg,
                                   const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                                   const void *sd, const void *bd, int sb_fp16, int norm, const void *resid,
                                   void *const *peers, int rank, int nranks, uint32_t *out_inds, void *out_scores,
                                   void *y, void *workspace, size_t workspace_bytes, void *stream) {
    if (!x || !router_w || !peers || !out_inds || !out_scores || !y || !workspace)
        return moe_set_error(MOE_EINVAL, "ep_decode_layer: null pointer");
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return moe_set_error(MOE_EINVAL, "ep_decode_layer: rank %d of %d (at most %d ranks)", rank, nranks, kMaxRanks);
    if (e_begin < 0 || e_count <= 0 || e_begin + e_count > E || H % 64 || I % 64)
        return moe_set_error(MOE_EINVAL, "ep_decode_layer: bad shard [%d, %d) of %d experts or H=%d I=%d", e_begin,
                             e_begin + e_count, E, H, I);
    const size_t need = moe_ep_workspace_bytes(T, H, I, E, K);
    if (workspace_bytes < need)
        return moe_set_error(MOE_EINVAL, "ep_decode_layer: workspace of %zu bytes needed, %zu given", need,
                             workspace_bytes);
    EpWs w = carve(workspace, T, H, I, E, K);
    int rc;
    if (T >= kEpGemmT) {
        // normalised rows, router on them, local experts as grouped GEMMs (the arithmetic of
        // moe_prefill_layer), unweighted outputs in assignment order for the exchange
        const void *xin = x;
        if (norm) {
            rc = moe_pow2_rows_launch(x, T, H, w.xn, stream);
            if (rc) return rc;
            xin = w.xn;
        }
        rc = moe_router_launch(xin, T, H, E, K, router_w, nullptr, nullptr, 16, 64, 0, nullptr, nullptr, nullptr, 0,
                               nullptr, nullptr, nullptr, out_inds, out_scores, nullptr, w.tickets, w.logits, nullptr,
                               nullptr, nullptr, nullptr, 0, stream);
        if (rc) return rc;
        rc = moe_prefill_experts_ex(xin, T, H, I, e_count, K, out_inds, (uint32_t)e_begin, 0, nullptr, wg, sg, bg, wu,
                                    su, bu, wd, sd, bd, sb_fp16, nullptr, nullptr, w.yk, nullptr, w.pws, w.pws_bytes,
                                    stream);
        if (rc) return rc;
    } else {
        rc = moe_router_launch(x, T, H, E, K, router_w, nullptr, nullptr, 16, 64, 0, nullptr, nullptr, nullptr, 0,
                               nullptr, nullptr, nullptr, out_inds, out_scores, nullptr, w.tickets, w.logits, nullptr,
                               w.xrec, w.xscale, w.xsum, norm, stream);
        if (rc) return rc;
        rc = moe_experts_gateup_ex(x, w.xrec, w.xscale, w.xsum, T, H, I, K, e_count, out_inds, wg, sg, bg, wu, su, bu,
                                   2, 64, sb_fp16, w.act, w.arec, w.ascale, w.asum, w.acnt, stream, (uint32_t)e_begin);
        if (rc) return rc;
        rc = moe_experts_down_ex(w.act, w.arec, w.ascale, w.asum, T, H, I, K, e_count, out_inds, nullptr, wd, sd, bd, 2,
                                 64, sb_fp16, nullptr, nullptr, nullptr, w.yk, stream, (uint32_t)e_begin);
        if (rc) return rc;
    }
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    ExArgs a{reinterpret_cast<unsigned char *const *>(peers), rank, nranks, T, K, H, (uint32_t)e_begin,
             (uint32_t)e_count, out_inds, static_cast<const uint16_t *>(out_scores), w.yk,
             static_cast<const uint16_t *>(resid), static_cast<uint16_t *>(y)};
    void *kargs[] = {&a};
    // grid sized to the work (16-byte chunks of the T*K rows and 8 outputs per thread), at
    // most one CTA per SM (the CTAs wait for one another: cooperative launch)
    const size_t chunks = (size_t)T * K * (H / 8);
    const int grid = (int)std::min<size_t>((size_t)sms, std::max<size_t>(2, (chunks + 4 * kExThreads - 1) / (4 * kExThreads)));
    MOE_CUDA_TRY(cudaLaunchCooperativeKernel((const void *)exchange_combine_kernel, dim3(grid), dim3(kExThreads), kargs,
                                             0, as_stream(stream)));
    return MOE_OK;
}
