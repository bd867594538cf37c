// Persistent decode kernel: one token through all L resident MoE layers in ONE cooperative
// launch (one CTA per SM), two grid barriers per layer. Expert weights are in the packed
// layout of moe_pack_experts. Per layer l:
//
//   phase A  every CTA loads the layer's router logits (fp64 accumulators, see phase B) and
//            h_l through L2, rounds the logits once to bf16 and runs the softmax / MLX-order
//            top-k / renorm itself. Work item q = (routed expert k, activation group G of
//            64 values), K * I/64 items over the CTAs: the CTA fetches the item's packed
//            slice with 1-D TMA bulk copies (8 gate/up units + the down slice), builds the
//            int8 MMA records of h_l while they are in flight, runs the 8 units (one warp
//            pair each, as soon as its bytes land), keeps the 64 SwiGLU activations in
//            shared memory, builds their one record, and runs the down slice: a split-K
//            partial of expert k's output over all H rows, written to global memory
//                                                                     -> grid barrier
//   phase B  each CTA owns 8-row blocks of h: sums the I/64 partials of every routed
//            expert for its rows (fixed order), rounds each expert output to bf16,
//            combines with the routing scores and the residual into its rows of h_{l+1}
//            (kept in shared memory across layers), and adds its rows' contribution to
//            layer l+1's router logits (transposed router slices fetched during phase A,
//            exact products, fp64 atomics)                             -> grid barrier
//
// The router logit of expert e is the double-precision sum of per-CTA partial sums, each an
// exact product sum; the bf16 rounding of that value equals the single rounding of the
// exact dot product unless the exact value lies within ~2^-50 (relative) of a bf16 rounding
// midpoint, so indices match the CPU oracle bit-for-bit in practice.
//
// Reference semantics: the resident-layer decode body of mlx-qwen38/loader.py:903-922 run
// for every layer of the stack (OffloadEngine.generate_greedy, loader.py:1176-1195).
#include <algorithm>

#include "common.cuh"
#include "f3core.cuh"
#include "gemv_i8.cuh"

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kUnits = 8;                   // gate/up units (8 rows) per activation group
constexpr int kMaxBlocks = 4;               // 8-row blocks of h per CTA in phase B
constexpr int kMaxE = 2048;
constexpr int kMaxK = 32;
constexpr int kMaxH = 4096;
constexpr int kHPass = kMaxH / 64 / (kThreads / 16);   // record passes over h
constexpr uint32_t kGridSpinLimit = 1u << 24;
constexpr int kAccCopies = 4;               // replicas of the logit accumulators (spread the atomics)
static_assert(kWarps == 2 * kUnits, "one warp pair per unit");

// Phase timestamps for profiling builds (compiled with -DMOE_STACK_TRACE, see build.py
// --trace): thread 0 of every CTA records %globaltimer at fixed points of every layer into
// g_stack_trace[cta][layer][slot], read back with moe_stack_trace_read. stack_kernel's slots:
// 0 layer start, 1 routed, 2 slice copies issued, 3 gate/up units done (after the block
// barrier), 4 item work done, 6 first grid barrier passed, 7 phase B done, 10 down-slice bytes
// waited for, 14 unit bytes waited for, 15 unit MMA loop done. f3moe_kernel's: 0 layer start,
// 1 write + norm sums done, 2 barrier passed, 5 mixer down done, 6 barrier, 7 mixer up + router
// partial done, 8 barrier, 9 routed, 11 shared gate / up done, 3 / 10 / 14 / 15 as above,
// 4 items done, 12 barrier, 13 phase B done. The library build compiles them out.
#ifdef MOE_STACK_TRACE
constexpr int kTraceCtas = 160, kTraceLayers = 64, kTraceSlots = 16;
__device__ unsigned long long g_stack_trace[kTraceCtas * kTraceLayers * kTraceSlots];
MOE_D void stamp(int layer, int slot) {
    if (threadIdx.x == 0 && blockIdx.x < kTraceCtas && layer < kTraceLayers) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_stack_trace[((size_t)blockIdx.x * kTraceLayers + layer) * kTraceSlots + slot] = t;
    }
}
#define STAMP(l, s) stamp((l), (s))
#else
#define STAMP(l, s) ((void)0)
#endif

// device-side copy of moe_stack_layer (include/moe_b200.h), same layout
struct StackLayer {
    const uint16_t *router_t;             // [H][E] bf16 (router transposed)
    const unsigned char *experts;         // [E] packed experts (moe_pack_experts)
};
static_assert(sizeof(StackLayer) == sizeof(moe_stack_layer), "layer descriptor layout");

// packed expert layout (pack.cu)
struct PackDims {
    uint32_t ub, dco, dso, dbytes, gbytes;
    size_t ebytes;
    MOE_HD PackDims(int H, int I) {
        ub = 5u * (uint32_t)H;            // unit: gate codes, up codes, scale records
        dco = 8u * ub;                    // down codes of the group (16 bytes per row)
        dso = dco + 16u * (uint32_t)H;    // down scale pairs (4 bytes per row)
        dbytes = 20u * (uint32_t)H;
        gbytes = 60u * (uint32_t)H;
        ebytes = (size_t)(I / 64) * gbytes;
    }
};

struct StackArgs {
    const StackLayer *layers;
    int L, H, I, E, K;
    const uint16_t *x_in;                 // [H]
    uint16_t *y_out;                      // [H]
    uint32_t *inds_out;                   // [L][K]
    uint16_t *scores_out;                 // [L][K]
    uint16_t *hs_out;                     // [L+1][H] every layer's input (+ final output), or null
    double *acc;                          // [2][kAccCopies][E] zero at launch
    double *ss;                           // [2]      sum of squares of h_l (norm), zero at launch
    int norm;                             // power-of-two RMS normalisation of each layer's input
    uint16_t *hbuf;                       // [2][H]
    float *yp;                            // [K][I/64][H] partial down outputs (work item q = k * I/64 + G)
    unsigned int *bar;                    // grid barrier counter, zero at launch
    unsigned int region;                  // bytes of the weight region in shared memory
};

// stride (in entries) of the entry-major record table of h: = 4 (mod 16) so that the eight
// B lanes of an MMA step read eight different bank pairs
MOE_HD int rec_stride(int ngroups) { return (ngroups + 15) / 16 * 16 + 4; }

struct SmemLayout {
    size_t bars, region, xrec, xscale, xsum, arec, ascale, sact, ypart, hown, red, cand, comp, redu, redd, sinds,
        sscores, dtr, total;
    MOE_HD SmemLayout(int H, int I, int K, size_t region_bytes) {
        const int ngH = H / 64;
        bars = 0;                                                 // 16 mbarriers
        region = 128;
        xrec = region + al128(region_bytes);
        xscale = xrec + (size_t)16 * rec_stride(ngH) * 8;
        xsum = xscale + al16((size_t)ngH * 4);
        arec = xsum + al128((size_t)ngH * 4);
        ascale = arec + 128;                                      // scale, sum
        sact = ascale + 16;
        ypart = sact + 128;
        hown = ypart + al16((size_t)K * kMaxBlocks * 8 * 4);
        red = hown + al16((size_t)kMaxBlocks * 8 * 4);
        cand = red + (size_t)kUnits * 2 * 8 * 2 * 4;
        comp = cand + (size_t)kWarps * kMaxK * 4;
        redu = comp + (size_t)kWarps * kMaxK * 4;
        redd = redu + kWarps * 4;
        sinds = redd + kWarps * 8;
        sscores = sinds + kMaxK * 4;
        dtr = al16(sscores + kMaxK * 4);                          // [kWarps][64] int dot products
        total = dtr + (size_t)kWarps * 64 * 4;
    }
};

MOE_D unsigned int ld_acquire(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier for a cooperative launch: the counter only grows within a launch;
// barrier n waits for (n + 1) * gridDim.x arrivals. Bounded: on timeout the device error word
// records it and the CTA proceeds.
MOE_D void grid_sync(unsigned int *bar, unsigned int n) {
    __syncthreads();
    if (threadIdx.x == 0) {
        // release: the block's writes (ordered before by the block barrier) become visible
        // to every CTA whose acquire load observes this arrival
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const unsigned int target = (n + 1) * gridDim.x;
        uint32_t it = 0;
#pragma unroll 1
        while (ld_acquire(bar) < target) {
            if (++it > kGridSpinLimit) {
                atomicOr(&g_moe_device_error, MOE_DEVERR_MBAR_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

// barrier over the two warps of unit pair p (named barriers 1..kUnits)
MOE_D void pair_sync(int p) { asm volatile("bar.sync %0, 64;" ::"r"(1 + p) : "memory"); }

MOE_D double block_sum_d(double v, double *redd) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) redd[warp] = v;
    __syncthreads();
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) s += redd[i];
    return s;
}

// order-preserving map of floats to unsigned integers
MOE_D uint32_t f2ord(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
MOE_D float ord2f(uint32_t o) { return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o); }

// warp 0, lane k holding the MLX-position-k selection (bf16 probability << 16 | expert):
// sequential bf16 sum of the K probabilities in MLX order, then bf16(p / S) per expert
MOE_D void renorm_mlx(uint32_t sel, int K, uint32_t *comp, uint32_t *sinds, float *sscores) {
    const int lane = threadIdx.x & 31;
    if (lane < K) comp[lane] = sel;
    __syncwarp();
    float S = bf16_bits_to_f32((uint16_t)(comp[0] >> 16));
#pragma unroll 4
    for (int k = 1; k < K; ++k) S = bf16r(S + bf16_bits_to_f32((uint16_t)(comp[k] >> 16)));
    if (lane < K) {
        sinds[lane] = sel & 0xffffu;
        sscores[lane] = bf16r(__fdiv_rn(bf16_bits_to_f32((uint16_t)(sel >> 16)), S));
    }
}

// Softmax (double, one bf16 rounding per probability) + MLX-order top-k + renorm of one
// token's logits. kKeysT logits per thread: av[j] holds the fp64 logit accumulator of expert
// tid + j * kThreads; xmul rescales them (power of two). With one key per thread warp 0
// selects the K largest of all keys directly; with more, every warp selects its K largest and
// warp 0 merges the sorted lists. Warp 0 writes the K experts in MLX order (ascending
// probability, then index) with their renormalised scores to sinds / sscores. All selection
// rounds are branch-free; the results are visible to the whole block on return.
template <int kKeysT>
MOE_D void route(const double (&av)[kKeysT], double xmul, int E, int K, uint32_t *redu, double *redd,
                 uint32_t *cand, uint32_t *comp, uint32_t *sinds, float *sscores) {
    static_assert(kWarps <= 32, "one list head per lane");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float lg[kKeysT];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKeysT; ++j) {
        const int e = tid + j * kThreads;
        lg[j] = (e < E) ? bf16_bits_to_f32(f64_to_bf16_bits(av[j] * xmul)) : -INFINITY;
        mx = fmaxf(mx, lg[j]);
    }
    uint32_t om = __reduce_max_sync(0xffffffffu, f2ord(mx));
    if (lane == 0) redu[warp] = om;
    __syncthreads();
    om = redu[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) om = max(om, redu[w]);
    const double mxd = (double)ord2f(om);
    double ev[kKeysT];
    double s = 0.0;
#pragma unroll
    for (int j = 0; j < kKeysT; ++j) {
        ev[j] = (tid + j * kThreads < E) ? exp((double)lg[j] - mxd) : 0.0;
        s += ev[j];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) redd[warp] = s;
    __syncthreads();
    s = 0.0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += redd[w];
    // keys ((p_bf16 << 16) | e) + 1: larger probability first, ties to the larger index
    uint32_t key[kKeysT];
    uint32_t lmax = 0;
#pragma unroll
    for (int j = 0; j < kKeysT; ++j) {
        const int e = tid + j * kThreads;
        key[j] = (e < E) ? ((((uint32_t)f64_to_bf16_bits(ev[j] / s)) << 16) | (uint32_t)e) + 1u : 0u;
        lmax = max(lmax, key[j]);
    }
    if constexpr (kKeysT == 1) {
        // E <= kThreads: all keys to shared memory; warp 0 holds kThreads/32 of them per lane
        // and runs K rounds of (lane max -> warp max -> the owner clears it): the r-th winner
        // is MLX position K-1-r
        cand[tid] = key[0];
        __syncthreads();
        if (warp == 0) {
            constexpr int kPer = kThreads / 32;
            uint32_t kk[kPer];
#pragma unroll
            for (int i = 0; i < kPer; ++i) kk[i] = cand[lane + 32 * i];
            uint32_t sel = 0;
#pragma unroll 1
            for (int r = 0; r < K; ++r) {
                uint32_t m = kk[0];
#pragma unroll
                for (int i = 1; i < kPer; ++i) m = max(m, kk[i]);
                const uint32_t w = __reduce_max_sync(0xffffffffu, m);
                sel = (lane == K - 1 - r) ? w - 1u : sel;
#pragma unroll
                for (int i = 0; i < kPer; ++i) kk[i] = (kk[i] == w) ? 0u : kk[i];
            }
            renorm_mlx(sel, K, comp, sinds, sscores);
        }
    } else {
        // this warp's K largest, descending, lane r holding the r-th
        uint32_t mine = 0;
#pragma unroll 1
        for (int r = 0; r < K; ++r) {
            const uint32_t w = __reduce_max_sync(0xffffffffu, lmax);
            mine = (lane == r) ? w : mine;
            lmax = 0;
#pragma unroll
            for (int j = 0; j < kKeysT; ++j) {
                key[j] = (key[j] == w) ? 0u : key[j];
                lmax = max(lmax, key[j]);
            }
        }
        if (lane < K) cand[warp * K + lane] = mine;
        __syncthreads();
        if (warp == 0) {
            // merge of the kWarps sorted lists: lane w < kWarps holds the head of list w and has the
            // element after it loaded already; K rounds of one warp-wide max
            const int lw = lane < kWarps ? lane : 0;
            uint32_t head = (lane < kWarps) ? cand[lw * K] : 0u;
            uint32_t nxt = (lane < kWarps && K > 1) ? cand[lw * K + 1] : 0u;
            int ptr = 1;                                  // list position of nxt
            uint32_t sel = 0;
#pragma unroll 1
            for (int r = 0; r < K; ++r) {
                const uint32_t w = __reduce_max_sync(0xffffffffu, head);
                sel = (lane == K - 1 - r) ? w - 1u : sel;         // lane k: MLX position k (ascending)
                const bool win = head == w;
                head = win ? nxt : head;
                ptr += win ? 1 : 0;
                const uint32_t ld = cand[lw * K + min(ptr, K - 1)];
                nxt = win ? ((ptr < K) ? ld : 0u) : nxt;
            }
            __syncwarp();
            renorm_mlx(sel, K, comp, sinds, sscores);
        }
    }
    __syncthreads();
}

// This CTA's rows' contribution to the next layer's router logits: waits for the router
// slices, then every thread adds sum_r router_t[row r][e] * h[row r] (exact fp32 products of
// bf16 values, double sums) into acc[e] with one fp64 atomic per expert. The loop is bound by
// instruction issue and the f32 -> f64 conversions: the eight shared loads of a row group go
// out before any arithmetic (twice as fast as a load-convert-add chain per row).
MOE_D void router_partial(uint64_t *rbar, uint32_t &rphase, const unsigned char *rbuf, const float *hown, int nrows,
                          int E, double *acc) {
    const bool ok = mbar_wait(rbar, rphase);
    rphase ^= 1u;
    if (!ok) return;
    const uint16_t *rs = reinterpret_cast<const uint16_t *>(rbuf);
#pragma unroll 1
    for (int e = threadIdx.x; e < E; e += kThreads) {
        double p[4] = {0.0, 0.0, 0.0, 0.0};
        int r0 = 0;
#pragma unroll 1
        for (; r0 + 8 <= nrows; r0 += 8) {
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = rs[(r0 + i) * E + e];
#pragma unroll
            for (int i = 0; i < 8; ++i) p[i & 3] += (double)(bf16_bits_to_f32((uint16_t)w[i]) * hown[r0 + i]);
        }
#pragma unroll 1
        for (; r0 < nrows; ++r0) p[0] += (double)(bf16_bits_to_f32(rs[r0 * E + e]) * hown[r0]);
        atomicAdd(acc + e, (p[0] + p[1]) + (p[2] + p[3]));
    }
}

// issues the copies of work item q's packed slice (thread 0): the 8 units in order, then the
// down slice, so the bytes land in the order they are consumed (measured ~1 % faster per token
// than nine threads issuing at once, whose copies land in no fixed order)
MOE_D void issue_item(const StackLayer &ly, const PackDims &P, const uint32_t *sinds, int q, int ngI,
                      unsigned char *region, uint64_t *ubar, uint64_t *dbar) {
    if (threadIdx.x != 0) return;
    const int k = q / ngI, G = q % ngI;
    const unsigned char *src = ly.experts + (size_t)sinds[k] * P.ebytes + (size_t)G * P.gbytes;
#pragma unroll 1
    for (int u = 0; u < kUnits; ++u) {
        mbar_arrive_expect_tx(&ubar[u], P.ub);
        tma_load_1d(region + (size_t)u * P.ub, src + (size_t)u * P.ub, P.ub, &ubar[u]);
    }
    mbar_arrive_expect_tx(dbar, P.dbytes);
    tma_load_1d(region + P.dco, src + P.dco, P.dbytes, dbar);
}

// Work item q = (routed expert k, activation group G of 64 values) of phase A, once its
// packed slice is being copied into `region` (issue_item; the unit and down copies complete on
// ubar[] / dbar at parity qphase): the 8 gate/up units (one warp pair each, as soon as its
// bytes land) on the records of the layer input, the 64 SwiGLU activations and their one
// record, and the down slice: a split-K partial of expert k's output over all H rows into
// yp[q][H]. Ends with a block barrier (the region may be reissued after it).
template <bool kFp16>
MOE_D void run_item(int q, int l, const PackDims &P, unsigned char *region, uint64_t *ubar, uint64_t *dbar,
                    uint32_t qphase, const uint2 *xrec, const float *xscale, const float *xsum, int xst, float *red,
                    uint16_t *sact, uint2 *arec, float *ascale, int *dtr, float *yp, int H) {
    (void)l;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int ngH = H / 64, NT = H / 16;
    // gate/up unit p = warp pair, H split in halves between the two warps
    {
        const int p = warp >> 1, half = warp & 1;
        const bool wok = mbar_wait(&ubar[p], qphase);
        STAMP(l, 14);
        const unsigned char *ubase = region + (size_t)p * P.ub;
        const uint4 *gc = reinterpret_cast<const uint4 *>(ubase);
        const uint4 *uc = reinterpret_cast<const uint4 *>(ubase + 2 * H);
        const uint2 *sr = reinterpret_cast<const uint2 *>(ubase + 4 * H);
        const int nsteps = ngH >> 2;
        const int s0 = half * nsteps / 2, s1 = (half + 1) * nsteps / 2;
        const bool bact = rec_lane_active(lane);
        const int part = rec_lane_part(lane);
        float accg = 0.f, accu = 0.f;
        if (wok) {
#pragma unroll 1
            for (int j = s0; j < s1; ++j) {
                const int Gj = 4 * j + t;
                const uint4 wv = gc[j * 32 + lane], uv = uc[j * 32 + lane];
                const uint2 sb = sr[j * 32 + lane];
                int dg, du;
                mma_step_i8t(wv, uv, xrec + Gj, xst, bact, part, dg, du);
                const float sc = xscale[Gj], sm = xsum[Gj];
                accg += sb_to_f32<kFp16>((uint16_t)sb.x) * ((float)dg * sc) +
                        sb_to_f32<kFp16>((uint16_t)(sb.x >> 16)) * sm;
                accu += sb_to_f32<kFp16>((uint16_t)sb.y) * ((float)du * sc) +
                        sb_to_f32<kFp16>((uint16_t)(sb.y >> 16)) * sm;
            }
        }
        STAMP(l, 15);
        accg += __shfl_xor_sync(0xffffffffu, accg, 1);
        accu += __shfl_xor_sync(0xffffffffu, accu, 1);
        accg += __shfl_xor_sync(0xffffffffu, accg, 2);
        accu += __shfl_xor_sync(0xffffffffu, accu, 2);
        if (t == 0) {
            red[((p * 2 + half) * 8 + g) * 2 + 0] = accg;
            red[((p * 2 + half) * 8 + g) * 2 + 1] = accu;
        }
        pair_sync(p);
        if (half == 0 && lane < 8) {
            const float gs = red[((p * 2) * 8 + lane) * 2 + 0] + red[((p * 2 + 1) * 8 + lane) * 2 + 0];
            const float us = red[((p * 2) * 8 + lane) * 2 + 1] + red[((p * 2 + 1) * 8 + lane) * 2 + 1];
            const float gv = bf16r(gs), uv = bf16r(us);
            const float sig = bf16r(1.0f / (1.0f + expf(-gv)));
            const float avv = wok ? bf16r(bf16r(gv * sig) * uv) : 0.f;
            sact[p * 8 + lane] = f32_to_bf16_bits(avv);
        }
    }
    __syncthreads();
    STAMP(l, 3);
    // the one record of the 64 activations, built by the last warp: warp 0 holds the thread
    // that issues the copies and (in the profiling build) stamps the timeline, and its global
    // stores slowed its shuffles ~10x there, hiding this step's true cost (~0.3 us)
    if (warp == kWarps - 1) {
        const uint2 qv = (lane < 16) ? reinterpret_cast<const uint2 *>(sact)[lane] : make_uint2(0u, 0u);
        rec_from_regs(qv, lane < 16, arec, ascale, ascale + 1, 1.0f);
    }
    __syncthreads();
    // down slice: split-K partial of expert k's output over all H rows. One MMA pair per
    // 16 rows: lane (g, t) feeds word t of rows g and g+8; B columns 0 / 1 carry the
    // record's hi / lo parts (lanes 0..7), so D columns 0 / 1 of lane quad t = 0 hold
    // the row's integer dot. A warp runs the MMAs of up to four of its tiles, parks the
    // 64 dots in its transpose buffer, and then every lane finishes two adjacent rows
    // (one 8-byte scale load, one 8-byte store) instead of 8 lanes per tile.
    {
        const bool wok = mbar_wait(dbar, qphase);
        STAMP(l, 10);
        const uint32_t *dc = reinterpret_cast<const uint32_t *>(region + P.dco);
        const uint32_t *ds = reinterpret_cast<const uint32_t *>(region + P.dso);
        const int n = lane >> 2;
        const uint2 bx = (lane < 8) ? arec[(0 * 4 + t) * 2 + n] : make_uint2(0u, 0u);
        const uint2 by = (lane < 8) ? arec[(1 * 4 + t) * 2 + n] : make_uint2(0u, 0u);
        const float asc = ascale[0], asm_ = ascale[1];
        float *ypq = yp + (size_t)q * H;
        int *yb = dtr + warp * 64;
        const int ntw = NT / kWarps;               // tiles per warp (H is a multiple of 256)
#pragma unroll 1
        for (int j0 = 0; j0 < ntw; j0 += 4) {
            const int jn = min(4, ntw - j0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (j < jn) {                      // warp-uniform
                    const int tile = warp + (j0 + j) * kWarps;
                    const uint32_t wa = dc[tile * 64 + lane], wb = dc[tile * 64 + 32 + lane];
                    int dx[4] = {0, 0, 0, 0}, dy[4] = {0, 0, 0, 0};
                    mma_u8s8_16832(dx, wa & 0x03030303u, wb & 0x03030303u, (wa >> 2) & 0x03030303u,
                                   (wb >> 2) & 0x03030303u, bx.x, bx.y);
                    mma_u8s8_16832(dy, wa & 0x30303030u, wb & 0x30303030u, (wa >> 2) & 0x30303030u,
                                   (wb >> 2) & 0x30303030u, by.x, by.y);
                    if (t == 0) {
                        yb[j * 16 + g] = (dx[0] + (dy[0] >> 4)) * 128 + (dx[1] + (dy[1] >> 4));
                        yb[j * 16 + 8 + g] = (dx[2] + (dy[2] >> 4)) * 128 + (dx[3] + (dy[3] >> 4));
                    }
                }
            }
            __syncwarp();
            const int j = lane >> 3, rr = 2 * (lane & 7);
            if (j < jn) {
                const int row = (warp + (j0 + j) * kWarps) * 16 + rr;
                const int2 dd = *reinterpret_cast<const int2 *>(yb + j * 16 + rr);
                const uint2 sp = *reinterpret_cast<const uint2 *>(ds + row);
                float2 o;
                o.x = sb_to_f32<kFp16>((uint16_t)sp.x) * ((float)dd.x * asc) +
                      sb_to_f32<kFp16>((uint16_t)(sp.x >> 16)) * asm_;
                o.y = sb_to_f32<kFp16>((uint16_t)sp.y) * ((float)dd.y * asc) +
                      sb_to_f32<kFp16>((uint16_t)(sp.y >> 16)) * asm_;
                if (!wok) o = make_float2(0.f, 0.f);
                *reinterpret_cast<float2 *>(ypq + row) = o;
            }
            __syncwarp();
        }
    }
    __syncthreads();
}

template <bool kFp16, int kKeysT>
__global__ void __launch_bounds__(kThreads, 1) stack_kernel(StackArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int H = a.H, I = a.I, E = a.E, K = a.K, L = a.L;
    const int G = gridDim.x, c = blockIdx.x;
    const int tid = threadIdx.x;
    // NB: 8-row blocks of h (phase B)
    const int ngH = H / 64, ngI = I / 64, NQ = K * ngI, NB = H / 8;
    const int xst = rec_stride(ngH);
    const PackDims P(H, I);
    const SmemLayout S(H, I, K, a.region);
    const int b0 = (int)((long long)c * NB / G), nb = (int)((long long)(c + 1) * NB / G) - b0;
    const int nrows = nb * 8;

    uint64_t *ubar = reinterpret_cast<uint64_t *>(smem + S.bars);          // [kUnits]
    uint64_t *dbar = ubar + kUnits;                                         // [1]
    uint64_t *rbar = dbar + 1;                                              // [1]
    unsigned char *region = smem + S.region;
    uint2 *xrec = reinterpret_cast<uint2 *>(smem + S.xrec);                // [16][xst]
    float *xscale = reinterpret_cast<float *>(smem + S.xscale);
    float *xsum = reinterpret_cast<float *>(smem + S.xsum);
    uint2 *arec = reinterpret_cast<uint2 *>(smem + S.arec);
    float *ascale = reinterpret_cast<float *>(smem + S.ascale);
    uint16_t *sact = reinterpret_cast<uint16_t *>(smem + S.sact);
    float *ypart = reinterpret_cast<float *>(smem + S.ypart);
    float *hown = reinterpret_cast<float *>(smem + S.hown);
    float *red = reinterpret_cast<float *>(smem + S.red);
    uint32_t *cand = reinterpret_cast<uint32_t *>(smem + S.cand);
    uint32_t *comp = reinterpret_cast<uint32_t *>(smem + S.comp);
    uint32_t *redu = reinterpret_cast<uint32_t *>(smem + S.redu);
    double *redd = reinterpret_cast<double *>(smem + S.redd);
    uint32_t *sinds = reinterpret_cast<uint32_t *>(smem + S.sinds);
    float *sscores = reinterpret_cast<float *>(smem + S.sscores);
    int *dtr = reinterpret_cast<int *>(smem + S.dtr);

    if (tid == 0) {
        for (int i = 0; i < kUnits + 2; ++i) mbar_init(&ubar[i], 1);
        fence_barrier_init();
    }
    __syncthreads();

    unsigned int nbar = 0;
    uint32_t rphase = 0, qphase = 0;
    const uint32_t rsb = 8u * (uint32_t)E * 2u;    // router slice of one 8-row block

    // --------------------------------------------------------------- prologue: h_0 and layer-0 logits
    if (tid == 0 && nb > 0) {
        mbar_arrive_expect_tx(rbar, rsb * nb);
#pragma unroll 1
        for (int bi = 0; bi < nb; ++bi)
            tma_load_1d(region + (size_t)bi * rsb, a.layers[0].router_t + (size_t)(b0 + bi) * 8 * E, rsb, rbar);
    }
    double ssp = 0.0;
#pragma unroll 1
    for (int r = tid; r < nrows; r += kThreads) {
        const uint16_t v = a.x_in[b0 * 8 + r];
        a.hbuf[b0 * 8 + r] = v;
        if (a.hs_out) a.hs_out[b0 * 8 + r] = v;
        hown[r] = bf16_bits_to_f32(v);
        ssp = fma((double)hown[r], (double)hown[r], ssp);
    }
    ssp = block_sum_d(ssp, redd);
    if (tid == 0 && a.norm && nb > 0) atomicAdd(a.ss, ssp);
    __syncthreads();
    if (nb > 0) router_partial(rbar, rphase, region, hown, nrows, E, a.acc + (size_t)(c % kAccCopies) * E);
    grid_sync(a.bar, nbar++);

#pragma unroll 1
    for (int l = 0; l < L; ++l) {
        const StackLayer ly = a.layers[l];
        const double *accl = a.acc + (size_t)(l & 1) * kAccCopies * E;
        const uint16_t *hcur = a.hbuf + (size_t)(l & 1) * H;
        uint16_t *hnext = a.hbuf + (size_t)((l + 1) & 1) * H;
        STAMP(l, 0);

        // ---------------------------------------------------------- phase A
        // loads through L2 (written by other SMs): logits, h_l, sum of squares
        double av[kKeysT];
#pragma unroll
        for (int j = 0; j < kKeysT; ++j) {
            const int e = tid + j * kThreads;
            av[j] = 0.0;
            if (e < E) {
#pragma unroll
                for (int r = 0; r < kAccCopies; ++r) av[j] += __ldcg(accl + (size_t)r * E + e);
            }
        }
        uint2 hq[kHPass];
#pragma unroll
        for (int p = 0; p < kHPass; ++p) {
            const int Gp = (tid >> 4) + p * (kThreads / 16);
            hq[p] = (Gp < ngH) ? __ldcg(reinterpret_cast<const uint2 *>(hcur + (size_t)Gp * 64) + (tid & 15))
                               : make_uint2(0u, 0u);
        }
        const double xmul = a.norm ? ldexp(1.0, -pow2_rms_shift(__ldcg(a.ss + (l & 1)), H)) : 1.0;

        route<kKeysT>(av, xmul, E, K, redu, redd, cand, comp, sinds, sscores);
        STAMP(l, 1);
        if (c == 0 && tid < K) {
            a.inds_out[(size_t)l * K + tid] = sinds[tid];
            a.scores_out[(size_t)l * K + tid] = f32_to_bf16_bits(sscores[tid]);
        }
        if (c < NQ) issue_item(ly, P, sinds, c, ngI, region, ubar, dbar);
        STAMP(l, 2);
        // records of h_l * xmul (entry-major) while the copies are in flight
#pragma unroll
        for (int p = 0; p < kHPass; ++p) {
            const int Gp = (tid >> 4) + p * (kThreads / 16);
            if (p * (kThreads / 16) < ngH)
                rec_from_regs(hq[p], Gp < ngH, xrec + Gp, xscale + Gp, xsum + Gp, (float)xmul, xst);
        }
        __syncthreads();
#pragma unroll 1
        for (int q = c; q < NQ; q += G) {
            run_item<kFp16>(q, l, P, region, ubar, dbar, qphase, xrec, xscale, xsum, xst, red, sact, arec, ascale, dtr,
                            a.yp, H);
            qphase ^= 1u;
            if (q + G < NQ) issue_item(ly, P, sinds, q + G, ngI, region, ubar, dbar);
        }
        STAMP(l, 4);
        // next layer's router slices into the consumed weight region
        if (tid == 0 && l + 1 < L && nb > 0) {
            mbar_arrive_expect_tx(rbar, rsb * nb);
#pragma unroll 1
            for (int bi = 0; bi < nb; ++bi)
                tma_load_1d(region + (size_t)bi * rsb, a.layers[l + 1].router_t + (size_t)(b0 + bi) * 8 * E, rsb,
                            rbar);
        }
        grid_sync(a.bar, nbar++);
        STAMP(l, 6);

        // ---------------------------------------------------------- phase B
        // expert outputs for this CTA's rows: thread (k, r) sums the I/64 partials of work
        // items (k, 0..) in a fixed order straight from L2 and rounds once to bf16
#pragma unroll 1
        for (int x = tid; x < K * nrows; x += kThreads) {
            const int k = x / nrows, r = x % nrows;
            const float *src = a.yp + (size_t)k * ngI * H + b0 * 8 + r;
            float v[16];                           // all partial loads of a row in flight at once
            float yk = 0.f;
#pragma unroll 1
            for (int g0 = 0; g0 < ngI; g0 += 16) {
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = (g0 + i < ngI) ? __ldcg(src + (size_t)(g0 + i) * H) : 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (g0 + i < ngI) yk += v[i];
            }
            ypart[k * nrows + r] = bf16r(yk);
        }
        __syncthreads();
        double ssn = 0.0;
#pragma unroll 1
        for (int r = tid; r < nrows; r += kThreads) {
            const int row = b0 * 8 + r;
            float accv = 0.f;
#pragma unroll 4
            for (int k = 0; k < K; ++k) {
                const float pk = bf16r(ypart[k * nrows + r] * sscores[k]);
                accv = (k == 0) ? pk : bf16r(accv + pk);
            }
            accv = bf16r(hown[r] + accv);
            const uint16_t hb = f32_to_bf16_bits(accv);
            hnext[row] = hb;
            if (a.hs_out) a.hs_out[(size_t)(l + 1) * H + row] = hb;
            if (l + 1 == L) a.y_out[row] = hb;
            hown[r] = accv;
            ssn = fma((double)accv, (double)accv, ssn);
        }
        ssn = block_sum_d(ssn, redd);
        if (tid == 0 && a.norm && nb > 0 && l + 1 < L) atomicAdd(a.ss + ((l + 1) & 1), ssn);
        __syncthreads();
        if (l + 1 < L && nb > 0)
            router_partial(rbar, rphase, region, hown, nrows, E,
                           a.acc + ((size_t)((l + 1) & 1) * kAccCopies + c % kAccCopies) * E);
        if (c == 0) {   // layer l's accumulators were consumed in phase A; ready them for l + 2
            double *accz = a.acc + (size_t)(l & 1) * kAccCopies * E;
#pragma unroll 1
            for (int e = tid; e < kAccCopies * E; e += kThreads) accz[e] = 0.0;
            if (tid == 0) a.ss[l & 1] = 0.0;
        }
        STAMP(l, 7);
        if (l + 1 < L) grid_sync(a.bar, nbar++);
    }
}


// ------------------------------------------------------------------ mixer + routed block + shared expert
//
// One token through L whole MoE decoder-layer halves in ONE cooperative launch (one CTA of 512
// threads per SM, at least 128). Per layer, five grid barriers:
//   P0a the write of the previous block into the streams and the norm's sums (f3core.cuh)   | barrier
//   P0b the norm into shared memory; P1 mixer down + inject rows                            | barrier
//   P2  mixer up + tail for the hidden indices j, j + G, ... this CTA owns (mixed), and their
//       contribution to the layer's router logits: the CTA's rows of the transposed router,
//       fetched during the previous phase B, exact products, fp64 atomics                  | barrier
//   A   every CTA: logits -> precise softmax -> MLX-order top-k -> renorm; the routed work
//       items (run_item, as stack_kernel's phase A) on the records of mixed; then the shared
//       expert's gate / up rows and scalar gate groups (at once on the CTAs without an item,
//       while the others' copies are in flight)                                          | barrier
//   B   the CTA's 8-row blocks of H: the shared down rows (scaled by the gate's sigmoid), the
//       routed partial sums, and branch = sum_k bf16(y_k * s_k) + shared (one bf16 rounding,
//       moe_experts_down with the shared output as its addend); then the next layer's router
//       rows are fetched                                                                     | barrier
// The normed streams and the router rows live in the weight region, which the routed items
// only use in phase A. After the last layer CTA 0 applies the last block's write.

// device-side copy of moe_f3moe_layer (include/moe_b200.h), same layout
struct F3MoeLayer {
    moe_f3_layer mix;
    const uint16_t *router_t;             // [H][E] bf16 (router transposed)
    const unsigned char *experts;         // [E] packed experts (moe_pack_experts)
};
static_assert(sizeof(F3MoeLayer) == sizeof(moe_f3moe_layer), "layer descriptor layout");

struct F3MoeArgs {
    const F3MoeLayer *layers;
    int L, H, R, Is, I, E, K;
    float eps;
    const uint16_t *h0, *branch0, *gate0;
    uint16_t *state_out, *branch_out, *inj_out, *branch_all, *mixed_all;
    uint32_t *inds_out;                   // [L][K]
    uint16_t *scores_out;                 // [L][K]
    moe_f3::F3Bufs bufs;
    uint16_t *state, *branch, *inj;       // [2][4H], [2][H], [2][4] (double-buffered by layer)
    double *acc;                          // [2][kAccCopies][E] router logit accumulators, zero at launch
    float *yp;                            // [K][I/64][H] partial down outputs
    unsigned int *bar;                    // grid barrier counter, zero at launch
    unsigned int region;                  // bytes of the weight region in shared memory
};

// shared memory: the routed block's layout followed by the mixer's staging buffers, this
// CTA's mixed values and its phase-B shared-expert outputs; inside the weight region the
// normed streams (offset 0) and the CTA's router rows (rslice)
struct F3MoeSmem {
    SmemLayout S;
    size_t sx, sv, spart, own, total, rslice;
    MOE_HD F3MoeSmem(int H, int R, int Is, int I, int K, int G, size_t region) : S(H, I, K, region) {
        const moe_f3::F3Smem F(H, R, Is, G, (size_t)kMaxBlocks * 8 * (Is / 64));
        sx = al128(S.total);
        sv = sx + (F.sv - F.sx);
        spart = sv + (F.spart - F.sv);
        own = spart + (F.total - F.spart);
        total = own + al128((size_t)((H + G - 1) / G) * 4);
        rslice = al128((size_t)moe_qlin::kHcStreams * H * 2);
    }
    // weight region bytes: the largest work item slice, or the normed streams + router rows
    MOE_HD static size_t region_bytes(int H, int I, int E, int G) {
        const size_t item = (size_t)PackDims(H, I).gbytes;
        const size_t mix = al128((size_t)moe_qlin::kHcStreams * H * 2) + (size_t)((H + G - 1) / G) * E * 2;
        return item > mix ? item : mix;
    }
};

template <bool kFp16Mix, bool kFp16Exp>
__global__ void __launch_bounds__(kThreads, 1) f3moe_kernel(F3MoeArgs a) {
    using namespace moe_f3;
    extern __shared__ __align__(128) unsigned char smem[];
    const int H = a.H, I = a.I, E = a.E, K = a.K, L = a.L, W = kHcStreams * H;
    const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
    const int ngH = H / 64, ngI = I / 64, NQ = K * ngI, NB = H / 8;
    const int xst = rec_stride(ngH);
    const PackDims P(H, I);
    const F3MoeSmem M(H, a.R, a.Is, I, K, G, a.region);
    const SmemLayout &S = M.S;
    const int b0 = (int)((long long)c * NB / G), nb = (int)((long long)(c + 1) * NB / G) - b0;
    const int nrows = nb * 8;

    uint64_t *ubar = reinterpret_cast<uint64_t *>(smem + S.bars);          // [kUnits]
    uint64_t *dbar = ubar + kUnits;                                         // [1]
    uint64_t *rbar = dbar + 1;                                              // [1]
    unsigned char *region = smem + S.region;
    uint2 *xrec = reinterpret_cast<uint2 *>(smem + S.xrec);                // [16][xst]
    float *xscale = reinterpret_cast<float *>(smem + S.xscale);
    float *xsum = reinterpret_cast<float *>(smem + S.xsum);
    uint2 *arec = reinterpret_cast<uint2 *>(smem + S.arec);
    float *ascale = reinterpret_cast<float *>(smem + S.ascale);
    uint16_t *sact = reinterpret_cast<uint16_t *>(smem + S.sact);
    float *ypart = reinterpret_cast<float *>(smem + S.ypart);
    float *red = reinterpret_cast<float *>(smem + S.red);
    uint32_t *cand = reinterpret_cast<uint32_t *>(smem + S.cand);
    uint32_t *comp = reinterpret_cast<uint32_t *>(smem + S.comp);
    uint32_t *redu = reinterpret_cast<uint32_t *>(smem + S.redu);
    double *redd = reinterpret_cast<double *>(smem + S.redd);
    uint32_t *sinds = reinterpret_cast<uint32_t *>(smem + S.sinds);
    float *sscores = reinterpret_cast<float *>(smem + S.sscores);
    int *dtr = reinterpret_cast<int *>(smem + S.dtr);
    float *own = reinterpret_cast<float *>(smem + M.own);                  // this CTA's mixed values
    unsigned char *rslice = region + M.rslice;                              // [nh][E] router rows
    __shared__ float srs[kHcStreams];
    F3Phases<kFp16Mix> f(H, a.R, a.Is, a.bufs, region, smem + M.sx, smem + M.sv, smem + M.spart, srs);

    if (tid == 0) {
        for (int i = 0; i < kUnits + 2; ++i) mbar_init(&ubar[i], 1);
        fence_barrier_init();
    }
    __syncthreads();

    unsigned int nbar = 0;
    uint32_t rphase = 0, qphase = 0;
    const uint32_t rrow = (uint32_t)E * 2u;
    // this CTA's rows of layer l's transposed router (hidden indices c, c + G, ...): lane q of
    // warp 0 copies row q (nh <= 32: H <= 32 G), after lane 0 has set the byte count
    auto fetch_router_rows = [&](int l) {
        if (tid < 32 && f.nh > 0) {
            if (tid == 0) mbar_arrive_expect_tx(rbar, rrow * (uint32_t)f.nh);
            __syncwarp();
            if (tid < f.nh)
                tma_load_1d(rslice + (size_t)tid * rrow, a.layers[l].router_t + (size_t)(c + tid * G) * E, rrow, rbar);
        }
    };
    fetch_router_rows(0);
    f.prefetch_mixer_down(a.layers[0].mix);

#pragma unroll 1
    for (int l = 0; l < L; ++l) {
        const F3MoeLayer &ly = a.layers[l];
        const moe_f3_layer &Ly = ly.mix;
        const uint16_t *hin = l == 0 ? a.h0 : a.state + (size_t)(l & 1) * W;
        const uint16_t *br = l == 0 ? a.branch0 : a.branch + (size_t)((l - 1) & 1) * H;
        const uint16_t *gt = l == 0 ? a.gate0 : a.inj + (size_t)((l - 1) & 1) * kHcStreams;
        uint16_t *wout = a.state + (size_t)((l + 1) & 1) * W;
        double *accl = a.acc + (size_t)(l & 1) * kAccCopies * E;

        // ---------------------------------------------------------- P0a, P0b + P1, P2
        STAMP(l, 0);
        f.write_and_sums(hin, br, gt, wout);
        STAMP(l, 1);
        grid_sync(a.bar, nbar++);
        STAMP(l, 2);
        f.norm(Ly, wout, a.eps);
        f.mixer_down(Ly);
        STAMP(l, 5);
        grid_sync(a.bar, nbar++);
        STAMP(l, 6);
        f.mixer_up(Ly, a.inj + (size_t)(l & 1) * kHcStreams, own, false);
        __syncthreads();
        if (a.mixed_all)
            for (int q = tid; q < f.nh; q += kThreads) a.mixed_all[(size_t)l * H + c + q * G] = f32_to_bf16_bits(own[q]);
        if (f.nh > 0) router_partial(rbar, rphase, rslice, own, f.nh, E, accl + (size_t)(c % kAccCopies) * E);
        STAMP(l, 7);
        grid_sync(a.bar, nbar++);
        STAMP(l, 8);

        // ---------------------------------------------------------- phase A
        double av[1] = {0.0};
        if (tid < E) {
#pragma unroll
            for (int r = 0; r < kAccCopies; ++r) av[0] += __ldcg(accl + (size_t)r * E + tid);
        }
        uint2 hq[kHPass];
#pragma unroll
        for (int p = 0; p < kHPass; ++p) {
            const int Gp = (tid >> 4) + p * (kThreads / 16);
            hq[p] = (Gp < ngH) ? __ldcg(reinterpret_cast<const uint2 *>(a.bufs.mixed + (size_t)Gp * 64) + (tid & 15))
                               : make_uint2(0u, 0u);
        }
        route<1>(av, 1.0, E, K, redu, redd, cand, comp, sinds, sscores);
        STAMP(l, 9);
        if (c == 0 && tid < K) {
            a.inds_out[(size_t)l * K + tid] = sinds[tid];
            a.scores_out[(size_t)l * K + tid] = f32_to_bf16_bits(sscores[tid]);
        }
        const StackLayer sl{ly.router_t, ly.experts};
        if (c < NQ) issue_item(sl, P, sinds, c, ngI, region, ubar, dbar);
        // records of mixed while the copies are in flight, then the routed items; then the shared
        // expert's gate / up rows (first thing on the CTAs without an item, while the others'
        // copies are in flight; after the item elsewhere, no longer competing with the copies)
#pragma unroll
        for (int p = 0; p < kHPass; ++p) {
            const int Gp = (tid >> 4) + p * (kThreads / 16);
            if (p * (kThreads / 16) < ngH) rec_from_regs(hq[p], Gp < ngH, xrec + Gp, xscale + Gp, xsum + Gp, 1.0f, xst);
        }
        stage_l2(f.sx, a.bufs.mixed, H);
        __syncthreads();
#pragma unroll 1
        for (int q = c; q < NQ; q += G) {
            run_item<kFp16Exp>(q, l, P, region, ubar, dbar, qphase, xrec, xscale, xsum, xst, red, sact, arec, ascale,
                               dtr, a.yp, H);
            qphase ^= 1u;
            if (q + G < NQ) issue_item(sl, P, sinds, q + G, ngI, region, ubar, dbar);
        }
        STAMP(l, 4);
        f.shared_gate_up(Ly, false, false);
        STAMP(l, 11);
        grid_sync(a.bar, nbar++);
        STAMP(l, 12);

        // ---------------------------------------------------------- phase B
        // the thread's first shared down item is loaded first; the routed partial sums run
        // while it is in flight
        if (tid < nrows * f.ng4) f.load4(Ly, tid, f.pf4, b0 * 8, 1);
#pragma unroll 1
        for (int x = tid; x < K * nrows; x += kThreads) {
            const int k = x / nrows, r = x % nrows;
            const float *src = a.yp + (size_t)k * ngI * H + b0 * 8 + r;
            float v[16];
            float yk = 0.f;
#pragma unroll 1
            for (int g0 = 0; g0 < ngI; g0 += 16) {
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = (g0 + i < ngI) ? __ldcg(src + (size_t)(g0 + i) * H) : 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (g0 + i < ngI) yk += v[i];
            }
            ypart[k * nrows + r] = bf16r(yk);
        }
        const float gsig = f.stage_down();
        f.shared_down_items(Ly, b0 * 8, 1, nrows, true);
        __syncthreads();
        uint16_t *bro = a.branch + (size_t)(l & 1) * H;
#pragma unroll 1
        for (int r = tid; r < nrows; r += kThreads) {
            const int row = b0 * 8 + r;
            float accv = 0.f;
#pragma unroll 4
            for (int k = 0; k < K; ++k) {
                const float pk = bf16r(ypart[k * nrows + r] * sscores[k]);
                accv = (k == 0) ? pk : bf16r(accv + pk);
            }
            accv = bf16r(accv + bf16_bits_to_f32(f.shared_down_out(r, gsig)));
            const uint16_t hb = f32_to_bf16_bits(accv);
            bro[row] = hb;
            if (a.branch_all) a.branch_all[(size_t)l * H + row] = hb;
        }
        if (l + 1 < L) {
            f.prefetch_mixer_down(a.layers[l + 1].mix);
            fetch_router_rows(l + 1);             // the region is free until the next phase A
        }
        if (c == 0) {   // layer l's logits were consumed in phase A; ready the buffer for l + 2
            double *accz = a.acc + (size_t)(l & 1) * kAccCopies * E;
#pragma unroll 1
            for (int e = tid; e < kAccCopies * E; e += kThreads) accz[e] = 0.0;
        }
        STAMP(l, 13);
        grid_sync(a.bar, nbar++);
    }

    // the last block's write into the state, and the last block output and gate
    if (c == 0) {
        const int l = L - 1;
        const uint16_t *st = a.state + (size_t)((l + 1) & 1) * W;
        const uint16_t *br = a.branch + (size_t)(l & 1) * H;
        const uint16_t *gt = a.inj + (size_t)(l & 1) * kHcStreams;
        for (int q = tid; q < W; q += kThreads) {
            const int cc = q / H, i = q - cc * H;
            const float gv = bf16_bits_to_f32(__ldcg(gt + cc));
            const float p = bf16r(__fmul_rn(bf16_bits_to_f32(__ldcg(br + i)), gv));
            a.state_out[q] = f32_to_bf16_bits(bf16r(__fadd_rn(bf16_bits_to_f32(__ldcg(st + q)), p)));
        }
        for (int q = tid; q < H; q += kThreads) a.branch_out[q] = __ldcg(br + q);
        if (tid < kHcStreams && a.inj_out) a.inj_out[tid] = __ldcg(gt + tid);
    }
}

struct F3MoeWs {
    size_t acc, bar, dv, iv, ssum, gsum, mixed, act, state, branch, inj, yp, total, zero;
    F3MoeWs(int H, int R, int Is, int I, int E, int K) {
        const size_t W = (size_t)moe_qlin::kHcStreams * H;
        acc = 0;
        bar = acc + al256((size_t)2 * kAccCopies * E * 8);
        zero = bar + 256;                                // acc + barrier: zero before every launch
        dv = zero;
        iv = dv + al256((size_t)R * 4);
        ssum = iv + al256(moe_qlin::kHcStreams * 4);
        gsum = ssum + al256(moe_qlin::kHcStreams * 32 * 8);
        mixed = gsum + al256((size_t)(H / 64) * 8);
        act = mixed + al256((size_t)H * 2);
        state = act + al256((size_t)Is * 2);
        branch = state + al256(2 * W * 2);
        inj = branch + al256(2 * (size_t)H * 2);
        yp = inj + 256;
        total = yp + al256((size_t)K * (I / 64) * H * 4);
    }
};

struct StackWs {
    double *acc, *ss;
    uint16_t *hbuf;
    float *yp;
    unsigned int *bar;
    size_t bytes;
};

StackWs carve(void *base, int H, int I, int E, int K) {
    StackWs w{};
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t n) { char *q = p ? p + off : nullptr; off += al256(n); return q; };
    w.acc = reinterpret_cast<double *>(take((size_t)(2 * kAccCopies * E + 2) * 8));
    w.ss = w.acc + 2 * kAccCopies * E;
    w.bar = reinterpret_cast<unsigned int *>(take(256));
    w.hbuf = reinterpret_cast<uint16_t *>(take((size_t)2 * H * 2));
    w.yp = reinterpret_cast<float *>(take((size_t)K * (I / 64) * H * 4));
    w.bytes = off;
    return w;
}

// bytes of the acc + barrier prefix that must be zero before every launch
size_t zero_prefix(int E) { return al256((size_t)(2 * kAccCopies * E + 2) * 8) + 256; }

}  // namespace

extern "C" size_t moe_stack_workspace_bytes(int H, int I, int E, int K) {
    if (H <= 0 || I <= 0 || E <= 0 || K <= 0) return 0;
    return carve(nullptr, H, I, E, K).bytes;
}

extern "C" int moe_stack_decode(const void *layers, int L, int H, int I, int E, int K, int sb_fp16,
                                int norm, const void *x, void *y, uint32_t *inds_out, void *scores_out, void *hs_out,
                                void *workspace, size_t workspace_bytes, int num_ctas, void *stream) {
    if (!layers || !x || !y || !inds_out || !scores_out || !workspace)
        return moe_set_error(MOE_EINVAL, "stack_decode: null pointer");
    if (L <= 0 || H % 256 || H > kMaxH || I % 64 || I <= 0 || E <= 0 || E > kMaxE || K <= 0 || K > kMaxK || K > E)
        return moe_set_error(MOE_EINVAL, "stack_decode: bad sizes L=%d H=%d I=%d E=%d K=%d", L, H, I, E, K);
    const size_t need = moe_stack_workspace_bytes(H, I, E, K);
    if (workspace_bytes < need)
        return moe_set_error(MOE_EINVAL, "stack_decode: workspace of %zu bytes needed, %zu given", need,
                             workspace_bytes);
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int G = num_ctas > 0 ? num_ctas : sms;
    if (G > sms) return moe_set_error(MOE_EINVAL, "stack_decode: %d CTAs > %d SMs", G, sms);
    if ((H / 8 + G - 1) / G > kMaxBlocks)
        return moe_set_error(MOE_EINVAL, "stack_decode: %d CTAs too few for %d row blocks", G, H / 8);
    const PackDims P(H, I);
    const size_t region = std::max((size_t)P.gbytes, (size_t)kMaxBlocks * 8 * E * 2);
    const SmemLayout S(H, I, K, region);
    if (S.total > 227 * 1024)
        return moe_set_error(MOE_EINVAL, "stack_decode: %zu bytes of shared memory needed", S.total);
    StackWs w = carve(workspace, H, I, E, K);
    auto st = as_stream(stream);
    MOE_CUDA_TRY(cudaMemsetAsync(workspace, 0, zero_prefix(E), st));
    StackArgs a{static_cast<const StackLayer *>(layers), L, H, I, E, K, static_cast<const uint16_t *>(x),
                static_cast<uint16_t *>(y), inds_out, static_cast<uint16_t *>(scores_out),
                static_cast<uint16_t *>(hs_out), w.acc, w.ss, norm, w.hbuf, w.yp, w.bar, (unsigned int)region};
    void *kargs[] = {&a};
    const void *kern = (E <= kThreads) ? (sb_fp16 ? (const void *)stack_kernel<true, 1> : (const void *)stack_kernel<false, 1>)
                                       : (sb_fp16 ? (const void *)stack_kernel<true, kMaxE / kThreads>
                                                  : (const void *)stack_kernel<false, kMaxE / kThreads>);
    // raise the kernel's shared-memory limit once per (kernel, size): not per launch, and
    // not while a launch is being captured
    static const void *set_kern[4] = {};
    static size_t set_bytes[4] = {};
    static int set_dev[4] = {-1, -1, -1, -1};
    const int ki = (E <= kThreads ? 0 : 2) + (sb_fp16 ? 1 : 0);
    if (set_kern[ki] != kern || set_bytes[ki] < S.total || set_dev[ki] != dev) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S.total));
        set_kern[ki] = kern;
        set_bytes[ki] = S.total;
        set_dev[ki] = dev;
    }
    MOE_CUDA_TRY(cudaLaunchCooperativeKernel(kern, dim3(G), dim3(kThreads), kargs, S.total, st));
    return MOE_OK;
}

extern "C" size_t moe_f3moe_stack_workspace_bytes(int H, int R, int Is, int I, int E, int K) {
    if (H <= 0 || R <= 0 || Is <= 0 || I <= 0 || E <= 0 || K <= 0) return 0;
    return F3MoeWs(H, R, Is, I, E, K).total;
}

extern "C" int moe_f3moe_stack_decode(const void *layers, int L, int H, int R, int Is, int I, int E, int K,
                                      int sb_fp16_mix, int sb_fp16_experts, float eps, const void *h,
                                      const void *branch0, const void *gate0, void *state_out, void *branch_out,
                                      void *inj_out, uint32_t *inds_out, void *scores_out, void *branch_all,
                                      void *mixed_all, void *workspace, size_t workspace_bytes, int num_ctas,
                                      void *stream) {
    if (!layers || !h || !state_out || !branch_out || !inds_out || !scores_out || !workspace)
        return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: null pointer");
    if (L <= 0 || H % 256 || H > kMaxH || R <= 0 || R % 64 || Is <= 0 || Is % 64 || I <= 0 || I % 64 || E <= 0 ||
        E % 8 || E > kThreads || K <= 0 || K > kMaxK || K > E)
        return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: bad sizes L=%d H=%d R=%d Is=%d I=%d E=%d K=%d", L, H, R, Is,
                             I, E, K);
    if ((branch0 == nullptr) != (gate0 == nullptr))
        return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: the first write needs both branch and gate");
    if (!(eps >= 0.f)) return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: eps must be >= 0");
    const F3MoeWs w(H, R, Is, I, E, K);
    if (workspace_bytes < w.total)
        return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: workspace of %zu bytes needed, %zu given", w.total,
                             workspace_bytes);
    const void *bufs[] = {h, branch0, state_out, branch_out, workspace, branch_all, mixed_all};
    for (const void *p : bufs)
        if (reinterpret_cast<uintptr_t>(p) % 16)
            return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: buffers must be 16-byte aligned");
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int G = num_ctas > 0 ? (num_ctas < sms ? num_ctas : sms) : sms;
    if (G < moe_qlin::kHcStreams * 32)
        return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: %d CTAs (the norm takes %d)", G,
                             moe_qlin::kHcStreams * 32);
    if ((H / 8 + G - 1) / G > kMaxBlocks || (H + G - 1) / G > 32)
        return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: %d CTAs too few for %d row blocks", G, H / 8);
    const size_t region = F3MoeSmem::region_bytes(H, I, E, G);
    const F3MoeSmem M(H, R, Is, I, K, G, region);
    if (M.total > 227 * 1024)
        return moe_set_error(MOE_EINVAL, "f3moe_stack_decode: %zu bytes of shared memory needed", M.total);
    auto st = as_stream(stream);
    MOE_CUDA_TRY(cudaMemsetAsync(workspace, 0, w.zero, st));
    char *p = static_cast<char *>(workspace);
    F3MoeArgs a{};
    a.layers = static_cast<const F3MoeLayer *>(layers);
    a.L = L, a.H = H, a.R = R, a.Is = Is, a.I = I, a.E = E, a.K = K, a.eps = eps;
    a.h0 = static_cast<const uint16_t *>(h);
    a.branch0 = static_cast<const uint16_t *>(branch0);
    a.gate0 = static_cast<const uint16_t *>(gate0);
    a.state_out = static_cast<uint16_t *>(state_out);
    a.branch_out = static_cast<uint16_t *>(branch_out);
    a.inj_out = static_cast<uint16_t *>(inj_out);
    a.branch_all = static_cast<uint16_t *>(branch_all);
    a.mixed_all = static_cast<uint16_t *>(mixed_all);
    a.inds_out = inds_out;
    a.scores_out = static_cast<uint16_t *>(scores_out);
    a.bufs.dv = reinterpret_cast<float *>(p + w.dv);
    a.bufs.iv = reinterpret_cast<float *>(p + w.iv);
    a.bufs.ssum = reinterpret_cast<double *>(p + w.ssum);
    a.bufs.gsum = reinterpret_cast<double *>(p + w.gsum);
    a.bufs.mixed = reinterpret_cast<uint16_t *>(p + w.mixed);
    a.bufs.act = reinterpret_cast<uint16_t *>(p + w.act);
    a.state = reinterpret_cast<uint16_t *>(p + w.state);
    a.branch = reinterpret_cast<uint16_t *>(p + w.branch);
    a.inj = reinterpret_cast<uint16_t *>(p + w.inj);
    a.acc = reinterpret_cast<double *>(p + w.acc);
    a.yp = reinterpret_cast<float *>(p + w.yp);
    a.bar = reinterpret_cast<unsigned int *>(p + w.bar);
    a.region = (unsigned int)region;
    void *kern = sb_fp16_mix ? (sb_fp16_experts ? (void *)f3moe_kernel<true, true> : (void *)f3moe_kernel<true, false>)
                             : (sb_fp16_experts ? (void *)f3moe_kernel<false, true> : (void *)f3moe_kernel<false, false>);
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)M.total));
    void *kargs[] = {&a};
    MOE_CUDA_TRY(cudaLaunchCooperativeKernel(kern, dim3(G), dim3(kThreads), kargs, M.total, st));
    return MOE_OK;
}

#ifdef MOE_STACK_TRACE
// copies the phase timestamps of the last launch (kTraceCtas x kTraceLayers x kTraceSlots
// u64, ns) to host memory
extern "C" int moe_stack_trace_read(unsigned long long *host, size_t n) {
    const size_t total = (size_t)kTraceCtas * kTraceLayers * kTraceSlots;
    MOE_CUDA_TRY(cudaMemcpyFromSymbol(host, g_stack_trace, (n < total ? n : total) * sizeof(unsigned long long)));
    return MOE_OK;
}
#endif
