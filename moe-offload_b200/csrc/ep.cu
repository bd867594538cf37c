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
#include <stddef.h>
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

// ====================================================================================
// Token-sharded expert parallelism: routed all-to-all dispatch and combine.
//
// For batches with several tokens per GPU (c4's decode batches of 8 per GPU and its 4,096-
// token prefill) every rank owns a contiguous block of ceil(T/N) tokens and their hidden
// states. Per layer, rank r:
//   router     the power-of-two normalised rows of its own tokens, exact softmax / top-k
//   dispatch   ONE kernel: each own token's normalised row is stored (peer stores over NVLink)
//              into the receive rows of every rank that owns one of its routed experts -- once
//              per (token, rank), however many of its experts that rank holds -- and its
//              routing row (experts, scores) into every rank's routing table; epoch flags, a
//              bounded wait for every rank's signal
//   experts    the rank's experts over every token routed to them (rows from the receive
//              buffer, routing from the table): grouped tensor-core GEMMs for batches of 32
//              tokens or more, per-slot int8 GEMVs below
//   combine    ONE kernel: each expert output row (token, k) computed here is stored into the
//              owning rank's return rows; signal, bounded wait, then the owner combines its
//              tokens in MLX order with the residual
// Every (token, k) output crosses NVLink once (the replicated path above stores every row in
// every rank), and the results equal the single-GPU layer bit for bit (each row is computed
// by the same kernels with the same arithmetic, each output slot has one writer).
//
// The buffers need no double buffering: a rank writes layer l+1's rows and routing into a
// peer only after every rank signalled the combine of layer l, which a rank does only after
// its expert kernels of layer l (the last readers of rows and routing) have finished; it
// writes layer l+1's returned rows only after every rank signalled the dispatch of l+1, sent
// only after that rank's combine of layer l (the last reader of the returned rows).
// ====================================================================================

struct A2aHeader {
    unsigned long long flag_d[kMaxRanks];   // dispatch epochs signalled into this buffer
    unsigned long long flag_c[kMaxRanks];   // combine epochs
    unsigned int arrive_d, arrive_c;        // CTAs of the running kernels that have stored
    unsigned int epoch;                     // layers this rank has completed
};
constexpr size_t kA2aHeaderBytes = 512;
static_assert(sizeof(A2aHeader) <= kA2aHeaderBytes, "a2a header size");

// after the header: received rows [T][H] (batches of kEpGemmT tokens or more: the GEMMs
// take bf16 rows) or received int8 MMA records of the rows [T][H/64][128 B] with their scales
// and sums [T][pad4(H/64)] (smaller batches: the GEMV kernels take records, built once by the
// owner's router), routing [T][K] (u32 experts, u16 scores), returned expert rows [Tl][K][H]
// of this rank's tokens
struct A2aRegion {
    size_t rows, rec, rscale, rsum, inds, scores, back, bytes;
    MOE_HD A2aRegion(int T, int Tl, int K, int H) {
        const size_t ng = (size_t)H / 64, fb = (size_t)pad4((int)ng) * 4;
        rows = kA2aHeaderBytes;
        rec = rows;                                   // the two forms share the space
        rscale = rec + al256((size_t)T * ng * 128);
        rsum = rscale + al256((size_t)T * fb);
        const size_t payload = std::max(al256((size_t)T * H * 2), rsum + al256((size_t)T * fb) - rows);
        inds = rows + payload;
        scores = inds + al256((size_t)T * K * 4);
        back = scores + al256((size_t)T * K * 2);
        bytes = back + al256((size_t)Tl * K * H * 2);
    }
};

struct A2aArgs {
    unsigned char *const *peers;
    int rank, nranks, T, Tl, K, H;
    int e_first[kMaxRanks + 1];             // rank q holds experts [e_first[q], e_first[q + 1])
    int g0, tn;                             // this rank's tokens [g0, g0 + tn)
    const uint16_t *xn;                     // [tn][H] own normalised rows (rows form)
    const uint2 *xrec;                      // [tn][H/64][16] own records (records form), or null
    const float *xscale, *xsum;             // [tn][pad4(H/64)]
    const uint32_t *inds;                   // [tn][K] own routing
    const uint16_t *scores;                 // [tn][K]
    const uint16_t *yk;                     // [T][K][H] expert outputs computed here (combine)
    const uint16_t *resid;                  // [tn][H] or null (combine)
    uint16_t *y;                            // [tn][H] (combine)
};

MOE_D int owner_of_expert(const A2aArgs &a, uint32_t e) {
    int q = 0;
#pragma unroll 1
    while (q + 1 < a.nranks && (uint32_t)a.e_first[q + 1] <= e) ++q;
    return q;
}

// the last CTA to arrive signals `e` into flag[rank] of every rank's header; every CTA's
// thread 0 then waits (bounded, 2 s) until every rank has signalled into this rank's header
MOE_D void a2a_signal_wait(const A2aArgs &a, unsigned int *arrive, size_t flag_off, unsigned int e) {
    unsigned char *own = a.peers[a.rank];
    if (threadIdx.x == 0) {
        const unsigned int old = atomicAdd(arrive, 1u);
        if (old + 1u == gridDim.x) {
            *arrive = 0u;
            __threadfence_system();
            for (int p = 0; p < a.nranks; ++p)
                st_release_sys(reinterpret_cast<unsigned long long *>(a.peers[p] + flag_off) + a.rank, e);
        }
        const unsigned long long *flags = reinterpret_cast<const unsigned long long *>(own + flag_off);
        const unsigned long long t0 = globaltimer_ns();
        for (int q = 0; q < a.nranks; ++q) {
#pragma unroll 1
            while (ld_acquire_sys(flags + q) < e) {
                if (globaltimer_ns() - t0 > kPeerWaitNs) {
                    atomicOr(&g_moe_device_error, MOE_DEVERR_PEER_TIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kExThreads) a2a_dispatch_kernel(A2aArgs a) {
    unsigned char *own = a.peers[a.rank];
    A2aHeader *hdr = reinterpret_cast<A2aHeader *>(own);
    __shared__ unsigned int s_epoch;
    if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned int *>(&hdr->epoch) + 1u;
    __syncthreads();
    const unsigned int e = s_epoch;
    const A2aRegion R(a.T, a.Tl, a.K, a.H);
    const int cpr = a.H / 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    bool stored = false;
    // payload per token: the bf16 row, or its records (8 chunks of 16 bytes per 64-value group)
    // followed by the group scales and sums; (token, destination rank, 16-byte chunk), a
    // destination gets a token's payload once
    const int ng = a.H / 64, fw = pad4(ng);
    const int rec_chunks = ng * 8, f_chunks = fw / 4;
    const int pay = a.xrec ? rec_chunks + 2 * f_chunks : cpr;
    const size_t nrow = (size_t)a.tn * a.nranks * pay;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nrow; i += stride) {
        const int t = (int)(i / ((size_t)a.nranks * pay));
        const int q = (int)((i / pay) % a.nranks);
        const int c = (int)(i % pay);
        bool to_q = false;
        for (int k = 0; k < a.K && !to_q; ++k) to_q = owner_of_expert(a, a.inds[(size_t)t * a.K + k]) == q;
        if (!to_q) continue;
        const size_t g = (size_t)(a.g0 + t);
        const uint4 *src;
        unsigned char *dst;
        if (!a.xrec) {
            src = reinterpret_cast<const uint4 *>(a.xn + (size_t)t * a.H) + c;
            dst = a.peers[q] + R.rows + (g * a.H) * 2 + (size_t)c * 16;
        } else if (c < rec_chunks) {
            src = reinterpret_cast<const uint4 *>(a.xrec + (size_t)t * ng * 16) + c;
            dst = a.peers[q] + R.rec + g * ng * 128 + (size_t)c * 16;
        } else if (c < rec_chunks + f_chunks) {
            src = reinterpret_cast<const uint4 *>(a.xscale + (size_t)t * fw) + (c - rec_chunks);
            dst = a.peers[q] + R.rscale + g * fw * 4 + (size_t)(c - rec_chunks) * 16;
        } else {
            src = reinterpret_cast<const uint4 *>(a.xsum + (size_t)t * fw) + (c - rec_chunks - f_chunks);
            dst = a.peers[q] + R.rsum + g * fw * 4 + (size_t)(c - rec_chunks - f_chunks) * 16;
        }
        *reinterpret_cast<uint4 *>(dst) = *src;
        stored = true;
    }
    // the routing rows of this rank's tokens into every rank's table
    const size_t nrt = (size_t)a.tn * a.K * a.nranks;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nrt; i += stride) {
        const int q = (int)(i % a.nranks);
        const size_t tk = i / a.nranks;
        const size_t gk = (size_t)a.g0 * a.K + tk;
        *reinterpret_cast<uint32_t *>(a.peers[q] + R.inds + gk * 4) = a.inds[tk];
        *reinterpret_cast<uint16_t *>(a.peers[q] + R.scores + gk * 2) = a.scores[tk];
        stored = true;
    }
    if (stored) __threadfence_system();
    __syncthreads();
    a2a_signal_wait(a, &hdr->arrive_d, offsetof(A2aHeader, flag_d), e);
}

__global__ void __launch_bounds__(kExThreads) a2a_combine_kernel(A2aArgs a) {
    unsigned char *own = a.peers[a.rank];
    A2aHeader *hdr = reinterpret_cast<A2aHeader *>(own);
    __shared__ unsigned int s_epoch;
    if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned int *>(&hdr->epoch) + 1u;
    __syncthreads();
    const unsigned int e = s_epoch;
    const A2aRegion R(a.T, a.Tl, a.K, a.H);
    const uint32_t *inds = reinterpret_cast<const uint32_t *>(own + R.inds);
    const uint32_t lo = (uint32_t)a.e_first[a.rank], hi = (uint32_t)a.e_first[a.rank + 1];
    const int cpr = a.H / 8;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    bool stored = false;
    // every (token, k) computed here goes back to the token's owner, once
    const size_t nw = (size_t)a.T * a.K * cpr;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nw; i += stride) {
        const size_t gk = i / cpr;
        const int c = (int)(i % cpr);
        const uint32_t ex = __ldcg(inds + gk);
        if (ex < lo || ex >= hi) continue;
        const int g = (int)(gk / a.K), k = (int)(gk % a.K);
        const int o = g / a.Tl;
        const uint4 v = *reinterpret_cast<const uint4 *>(a.yk + gk * a.H + (size_t)c * 8);
        const size_t dst = ((size_t)(g - o * a.Tl) * a.K + k) * a.H + (size_t)c * 8;
        *reinterpret_cast<uint4 *>(a.peers[o] + R.back + dst * 2) = v;
        stored = true;
    }
    if (stored) __threadfence_system();
    __syncthreads();
    a2a_signal_wait(a, &hdr->arrive_c, offsetof(A2aHeader, flag_c), e);
    // the epoch advances once every CTA has read it (they all passed the wait above)
    if (blockIdx.x == 0 && threadIdx.x == 0) hdr->epoch = e;
    // this rank's tokens: sequential bf16 sum over k in MLX order, then the residual
    const uint16_t *back = reinterpret_cast<const uint16_t *>(own + R.back);
    const size_t n = (size_t)a.tn * a.H;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const size_t t = i / a.H, h = i % a.H;
        float acc = 0.f;
        for (int k = 0; k < a.K; ++k) {
            const float yv = bf16_bits_to_f32(__ldcg(back + (t * a.K + k) * a.H + h));
            const float pk = bf16r(yv * bf16_bits_to_f32(a.scores[t * a.K + k]));
            acc = (k == 0) ? pk : bf16r(acc + pk);
        }
        if (a.resid) acc = bf16r(bf16_bits_to_f32(a.resid[i]) + acc);
        a.y[i] = f32_to_bf16_bits(acc);
    }
}

struct A2aWs {
    unsigned int *tickets;
    uint16_t *logits, *xn, *act, *yk;
    uint2 *xrec;                            // own records (batches below kEpGemmT)
    float *xscale, *xsum;
    void *pws;
    size_t pws_bytes, bytes;
};

A2aWs carve_a2a(void *base, int T, int Tl, int H, int I, int E, int K) {
    A2aWs w{};
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t n) { char *q = p ? p + off : nullptr; off += al256(n); return q; };
    w.tickets = reinterpret_cast<unsigned int *>(take((size_t)Tl * 4));
    w.logits = reinterpret_cast<uint16_t *>(take((size_t)Tl * E * 2));
    w.xn = reinterpret_cast<uint16_t *>(take((size_t)Tl * H * 2));
    w.yk = reinterpret_cast<uint16_t *>(take((size_t)T * K * H * 2));
    if (T >= kEpGemmT) {
        w.pws_bytes = moe_prefill_workspace_bytes(T, H, I, E, K);
        w.pws = take(w.pws_bytes);
    } else {
        w.act = reinterpret_cast<uint16_t *>(take((size_t)T * K * I * 2));
        w.xrec = reinterpret_cast<uint2 *>(take((size_t)Tl * (H / 64) * 128));
        w.xscale = reinterpret_cast<float *>(take((size_t)Tl * pad4(H / 64) * 4));
        w.xsum = reinterpret_cast<float *>(take((size_t)Tl * pad4(H / 64) * 4));
    }
    w.bytes = off;
    return w;
}

int local_tokens(int T, int nranks, int rank, int *g0) {
    const int Tl = (T + nranks - 1) / nranks;
    *g0 = std::min(T, rank * Tl);
    return std::min(T, *g0 + Tl) - *g0;
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

extern "C" size_t moe_ep_a2a_buffer_bytes(int T, int K, int H, int nranks) {
    if (T <= 0 || K <= 0 || H <= 0 || nranks <= 0) return 0;
    return A2aRegion(T, (T + nranks - 1) / nranks, K, H).bytes;
}

extern "C" size_t moe_ep_a2a_workspace_bytes(int T, int H, int I, int E, int K, int nranks) {
    if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || K <= 0 || nranks <= 0) return 0;
    return carve_a2a(nullptr, T, (T + nranks - 1) / nranks, H, I, E, K).bytes;
}

extern "C" int moe_ep_a2a_local_tokens(int T, int nranks, int rank, int *first) {
    if (T <= 0 || nranks <= 0 || rank < 0 || rank >= nranks || !first) return 0;
    return local_tokens(T, nranks, rank, first);
}

extern "C" int moe_ep_a2a_layer(const void *x, int T, int H, int I, int E, int K, const int *e_first,
                                const void *router_w, const uint32_t *wg, const void *sg, const void *bg,
                                const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd, const void *sd,
                                const void *bd, int sb_fp16, int norm, const void *resid, void *const *peers,
                                const void *own_buffer, int rank, int nranks, uint32_t *out_inds, void *out_scores,
                                void *y, void *workspace, size_t workspace_bytes, void *stream) {
    if (!router_w || !peers || !own_buffer || !workspace || !e_first)
        return moe_set_error(MOE_EINVAL, "ep_a2a_layer: null pointer");
    if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks)
        return moe_set_error(MOE_EINVAL, "ep_a2a_layer: rank %d of %d (at most %d ranks)", rank, nranks, kMaxRanks);
    if (T <= 0 || H % 64 || I % 64 || K <= 0 || K > E || e_first[0] != 0 || e_first[nranks] != E)
        return moe_set_error(MOE_EINVAL, "ep_a2a_layer: bad sizes T=%d H=%d I=%d E=%d K=%d or expert split", T, H,
                             I, E, K);
    for (int q = 0; q < nranks; ++q)
        if (e_first[q + 1] <= e_first[q])
            return moe_set_error(MOE_EINVAL, "ep_a2a_layer: rank %d holds no experts", q);
    const size_t need = moe_ep_a2a_workspace_bytes(T, H, I, E, K, nranks);
    if (workspace_bytes < need)
        return moe_set_error(MOE_EINVAL, "ep_a2a_layer: workspace of %zu bytes needed, %zu given", need,
                             workspace_bytes);
    const int Tl = (T + nranks - 1) / nranks;
    int g0 = 0;
    const int tn = local_tokens(T, nranks, rank, &g0);
    if (tn > 0 && (!x || !out_inds || !out_scores || !y))
        return moe_set_error(MOE_EINVAL, "ep_a2a_layer: null token buffers");
    A2aWs w = carve_a2a(workspace, T, Tl, H, I, E, K);
    const int e0 = e_first[rank], n = e_first[rank + 1] - e_first[rank];
    const A2aRegion R(T, Tl, K, H);
    const unsigned char *own = static_cast<const unsigned char *>(own_buffer);
    const uint16_t *rows = reinterpret_cast<const uint16_t *>(own + R.rows);
    const uint32_t *all_inds = reinterpret_cast<const uint32_t *>(own + R.inds);
    int rc;
    const bool gemm = T >= kEpGemmT;
    // own tokens: routing, and what the experts take -- normalised bf16 rows (GEMMs), or the
    // int8 records of the normalised rows built by the router (GEMVs)
    if (tn > 0) {
        if (gemm) {
            if (norm) {
                rc = moe_pow2_rows_launch(x, tn, H, w.xn, stream);
                if (rc) return rc;
            } else {
                MOE_CUDA_TRY(
                    cudaMemcpyAsync(w.xn, x, (size_t)tn * H * 2, cudaMemcpyDeviceToDevice, as_stream(stream)));
            }
            rc = moe_router_launch(w.xn, tn, H, E, K, router_w, nullptr, nullptr, 16, 64, 0, nullptr, nullptr, nullptr,
                                   0, nullptr, nullptr, nullptr, out_inds, out_scores, nullptr, w.tickets, w.logits,
                                   nullptr, nullptr, nullptr, nullptr, 0, stream);
        } else {
            rc = moe_router_launch(x, tn, H, E, K, router_w, nullptr, nullptr, 16, 64, 0, nullptr, nullptr, nullptr, 0,
                                   nullptr, nullptr, nullptr, out_inds, out_scores, nullptr, w.tickets, w.logits,
                                   nullptr, w.xrec, w.xscale, w.xsum, norm, stream);
        }
        if (rc) return rc;
    }
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    A2aArgs a{};
    a.peers = reinterpret_cast<unsigned char *const *>(peers);
    a.rank = rank;
    a.nranks = nranks;
    a.T = T;
    a.Tl = Tl;
    a.K = K;
    a.H = H;
    for (int q = 0; q <= nranks; ++q) a.e_first[q] = e_first[q];
    a.g0 = g0;
    a.tn = tn;
    a.xn = w.xn;
    a.xrec = gemm ? nullptr : w.xrec;
    a.xscale = gemm ? nullptr : w.xscale;
    a.xsum = gemm ? nullptr : w.xsum;
    a.inds = out_inds;
    a.scores = static_cast<const uint16_t *>(out_scores);
    a.yk = w.yk;
    a.resid = static_cast<const uint16_t *>(resid);
    a.y = static_cast<uint16_t *>(y);
    void *kargs[] = {&a};
    const size_t dchunks = (size_t)std::max(tn, 1) * nranks * (H / 8 + 32);
    const int gd =
        (int)std::min<size_t>((size_t)sms, std::max<size_t>(2, (dchunks + 4 * kExThreads - 1) / (4 * kExThreads)));
    MOE_CUDA_TRY(cudaLaunchCooperativeKernel((const void *)a2a_dispatch_kernel, dim3(gd), dim3(kExThreads), kargs, 0,
                                             as_stream(stream)));
    // this rank's experts over every token routed to them (rows and routing in its buffer)
    if (gemm) {
        rc = moe_prefill_experts_ex(rows, T, H, I, n, K, all_inds, (uint32_t)e0, 0, nullptr, wg, sg, bg, wu, su, bu, wd,
                                    sd, bd, sb_fp16, nullptr, nullptr, w.yk, nullptr, w.pws, w.pws_bytes, stream);
    } else {
        rc = moe_experts_gateup_ex(rows, own + R.rec, reinterpret_cast<const float *>(own + R.rscale),
                                   reinterpret_cast<const float *>(own + R.rsum), T, H, I, K, n, all_inds, wg, sg, bg,
                                   wu, su, bu, 2, 64, sb_fp16, w.act, nullptr, nullptr, nullptr, nullptr, stream,
                                   (uint32_t)e0);
        if (rc) return rc;
        rc = moe_experts_down_ex(w.act, nullptr, nullptr, nullptr, T, H, I, K, n, all_inds, nullptr, wd, sd, bd, 2, 64,
                                 sb_fp16, nullptr, nullptr, nullptr, w.yk, stream, (uint32_t)e0);
    }
    if (rc) return rc;
    const size_t cchunks = (size_t)T * K * (H / 8) / nranks + (size_t)std::max(tn, 1) * H / 8;
    const int gc =
        (int)std::min<size_t>((size_t)sms, std::max<size_t>(2, (cchunks + 4 * kExThreads - 1) / (4 * kExThreads)));
    MOE_CUDA_TRY(cudaLaunchCooperativeKernel((const void *)a2a_combine_kernel, dim3(gc), dim3(kExThreads), kargs, 0,
                                             as_stream(stream)));
    return MOE_OK;
}
