// Persistent decode kernel: one token through all L resident MoE layers in ONE cooperative
// launch (one CTA per SM), two grid barriers per layer. Per layer l:
//
//   phase A  every CTA reads the layer's router logits (fp64 accumulators, see phase B),
//            rounds them once to bf16 and runs the softmax / MLX-order top-k / renorm
//            itself (no extra synchronisation); issues 1-D TMA bulk copies for its share of
//            the routed gate/up rows (units = 8 gate + 8 up rows of one expert), builds the
//            int8 MMA records of h_l, runs the units (2 warps per unit, H split in halves),
//            writes its act values, then issues the TMA copies of its down rows into the
//            freed unit buffers                                        -> grid barrier
//   phase B  builds the records of all K activation vectors, runs its down blocks (16
//            output rows x K experts), combines with the routing scores and the residual
//            into its rows of h_{l+1}, and adds its rows' contribution to layer l+1's
//            router logits (prefetched slice of the transposed router, exact products,
//            fp64 atomics)                                             -> grid barrier
//
// The router logit of expert e is the double-precision sum of per-CTA partial sums, each an
// exact product sum; the bf16 rounding of that value equals the single rounding of the
// exact dot product unless the exact value lies within ~2^-50 (relative) of a bf16 rounding
// midpoint, so indices match the CPU oracle bit-for-bit in practice.
//
// Reference semantics: the resident-layer decode body of mlx-qwen38/loader.py:903-922 run
// for every layer of the stack (OffloadEngine.generate_greedy, loader.py:1176-1195).
#include "common.cuh"
#include "gemv_i8.cuh"
#include "topk.cuh"

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kPairs = kWarps / 2;        // gate/up units in flight per CTA
constexpr int kMaxBlocks = 2;             // down blocks (16 rows) per CTA
constexpr int kMaxE = 2048;
constexpr uint32_t kGridSpinLimit = 1u << 24;

// device-side copy of moe_stack_layer (include/moe_b200.h), same layout
struct StackLayer {
    const uint16_t *router_t;             // [H][E] bf16 (router transposed)
    const uint32_t *wg, *wu, *wd;
    const uint16_t *sg, *bg, *su, *bu, *sd, *bd;
};
static_assert(sizeof(StackLayer) == sizeof(moe_stack_layer), "layer descriptor layout");

struct StackArgs {
    const StackLayer *layers;
    int L, H, I, E, K;
    const uint16_t *x_in;                 // [H]
    uint16_t *y_out;                      // [H]
    uint32_t *inds_out;                   // [L][K]
    uint16_t *scores_out;                 // [L][K]
    uint16_t *hs_out;                     // [L+1][H] every layer's input (+ final output), or null
    double *acc;                          // [2][E]   zero at launch
    double *ss;                           // [2]      sum of squares of h_l (norm), zero at launch
    int norm;                             // power-of-two RMS normalisation of each layer's input
    uint16_t *hbuf;                       // [2][H]
    uint16_t *act;                        // [K][I]
    unsigned int *bar;                    // grid barrier counter, zero at launch
};

struct SmemLayout {
    size_t bars, ubuf, ubytes, dbytes, rbuf, xrec, xscale, xsum, arec, ascale, asum, zrec, yk, hnew, red,
        keys, sel, prob, sinds, sscores, redd, cand, gexp, total;
    int ngH, ngI, umax;
    MOE_HD SmemLayout(int H, int I, int E, int K, int G) {
        ngH = H / 64;
        ngI = I / 64;
        const int U = K * (I / 8);
        umax = (U + G - 1) / G;
        ubytes = al128(16 * (size_t)(H / 4) + 4 * 8 * (size_t)ngH * 2);           // one gate/up unit
        dbytes = al128((size_t)K * (16 * (size_t)(I / 4) + 2 * 16 * (size_t)ngI * 2));  // one down block
        bars = 0;                                                                   // 16 mbarriers
        ubuf = 128;
        const size_t ureg = (size_t)umax * ubytes, dreg = kMaxBlocks * dbytes;
        rbuf = ubuf + (ureg > dreg ? ureg : dreg);
        xrec = rbuf + al128((size_t)kMaxBlocks * 16 * E * 2);
        xscale = xrec + (size_t)ngH * 128;
        xsum = xscale + al16((size_t)pad4(ngH) * 4);
        arec = xsum + al128((size_t)pad4(ngH) * 4);
        ascale = arec + (size_t)K * ngI * 128;
        asum = ascale + al16((size_t)pad4(K * ngI) * 4);
        zrec = asum + al128((size_t)pad4(K * ngI) * 4);
        yk = zrec + 128;
        hnew = yk + al16((size_t)kMaxBlocks * K * 16 * 4);
        red = hnew + kMaxBlocks * 16 * 8;
        keys = red + (size_t)kPairs * 2 * 8 * 2 * 4;
        sel = keys + al16((size_t)E * 4);
        prob = sel + 64 * 4;
        sinds = prob + al16((size_t)E * 8);
        sscores = sinds + 64 * 4;
        redd = sscores + 64 * 4;
        cand = redd + kWarps * 8 + 64;                // kWarps * 32 selection candidates
        gexp = cand + kWarps * 32 * 4;                // per-group exponents for the record builder
        total = gexp + al16((size_t)4 * (ngH > K * ngI ? ngH : K * ngI));
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
        __threadfence();
        atomicAdd(bar, 1u);
        const unsigned int target = (n + 1) * gridDim.x;
        uint32_t it = 0;
        while (ld_acquire(bar) < target) {
            if (++it > kGridSpinLimit) {
                atomicOr(&g_moe_device_error, MOE_DEVERR_MBAR_TIMEOUT);
                break;
            }
            __nanosleep(20);
        }
        __threadfence();
    }
    __syncthreads();
}

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

MOE_D float block_max_f(float v, double *redd) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *r = reinterpret_cast<float *>(redd);
    __syncthreads();
    if (lane == 0) r[warp] = v;
    __syncthreads();
    float m = r[0];
#pragma unroll
    for (int i = 1; i < kWarps; ++i) m = fmaxf(m, r[i]);
    return m;
}

// softmax (double, one bf16 rounding) + MLX-order top-k + renorm of one token's logits held
// in fp64 accumulators; results in sinds / sscores (shared memory) of every CTA.
MOE_D void softmax_topk(const double *acc, double xmul, int E, int K, uint32_t *keys, uint32_t *sel,
                        uint32_t *cand, double *prob, uint32_t *sinds, float *sscores, double *redd) {
    float mx = -INFINITY;
    for (int e = threadIdx.x; e < E; e += kThreads) {
        const float l = bf16_bits_to_f32(f64_to_bf16_bits(__ldcg(acc + e) * xmul));
        prob[e] = (double)l;
        mx = fmaxf(mx, l);
    }
    mx = block_max_f(mx, redd);
    double s = 0.0;
    for (int e = threadIdx.x; e < E; e += kThreads) {
        const double v = exp(prob[e] - (double)mx);
        prob[e] = v;
        s += v;
    }
    s = block_sum_d(s, redd);
    for (int e = threadIdx.x; e < E; e += kThreads) {
        const uint16_t p = f64_to_bf16_bits(prob[e] / s);
        keys[e] = (((uint32_t)p << 16) | (uint32_t)e) + 1u;
    }
    __syncthreads();
    if (E <= kThreads) {
        block_select_desc(keys, E, K, cand, sel);    // descending keys (+1 offset)
    } else {
        if (threadIdx.x < 32) warp_select_desc(keys, E, K, sel);
        __syncthreads();
    }
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        // MLX order = ascending (p, index): lane k takes the k-th smallest selected key
        const uint32_t key = (lane < K) ? sel[K - 1 - lane] - 1u : 0u;
        const float p = bf16_bits_to_f32((uint16_t)(key >> 16));
        float S = 0.f;
        for (int k = 0; k < K; ++k) {                 // sequential bf16 sum in that order
            const float pk = __shfl_sync(0xffffffffu, p, k);
            S = (k == 0) ? pk : bf16r(S + pk);
        }
        if (lane < K) {
            sinds[lane] = key & 0xffffu;
            sscores[lane] = bf16r(__fdiv_rn(p, S));
        }
    }
    __syncthreads();
}

template <bool kFp16>
__global__ void __launch_bounds__(kThreads, 1) stack_kernel(StackArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int H = a.H, I = a.I, E = a.E, K = a.K, L = a.L;
    const int G = gridDim.x, c = blockIdx.x;
    const SmemLayout S(H, I, E, K, G);
    const int ngH = S.ngH, ngI = S.ngI;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;

    uint64_t *ubar = reinterpret_cast<uint64_t *>(smem + S.bars);          // [kPairs] units
    uint64_t *dbar = ubar + kPairs;                                         // [kMaxBlocks] down blocks
    uint64_t *rbar = dbar + kMaxBlocks;                                     // [1] router slices
    unsigned char *ubuf = smem + S.ubuf;
    unsigned char *rbuf = smem + S.rbuf;
    uint2 *xrec = reinterpret_cast<uint2 *>(smem + S.xrec);
    float *xscale = reinterpret_cast<float *>(smem + S.xscale);
    float *xsum = reinterpret_cast<float *>(smem + S.xsum);
    uint2 *arec = reinterpret_cast<uint2 *>(smem + S.arec);
    float *ascale = reinterpret_cast<float *>(smem + S.ascale);
    float *asum = reinterpret_cast<float *>(smem + S.asum);
    uint2 *zrec = reinterpret_cast<uint2 *>(smem + S.zrec);
    float *yk = reinterpret_cast<float *>(smem + S.yk);
    double *hnew = reinterpret_cast<double *>(smem + S.hnew);
    float *red = reinterpret_cast<float *>(smem + S.red);
    uint32_t *keys = reinterpret_cast<uint32_t *>(smem + S.keys);
    uint32_t *sel = reinterpret_cast<uint32_t *>(smem + S.sel);
    double *prob = reinterpret_cast<double *>(smem + S.prob);
    uint32_t *sinds = reinterpret_cast<uint32_t *>(smem + S.sinds);
    float *sscores = reinterpret_cast<float *>(smem + S.sscores);
    double *redd = reinterpret_cast<double *>(smem + S.redd);
    uint32_t *cand = reinterpret_cast<uint32_t *>(smem + S.cand);
    int *gexp = reinterpret_cast<int *>(smem + S.gexp);

    // static work split: gate/up units u = k * (I/8) + rb, down blocks b (16 rows of H)
    const int U = K * (I / 8), NB = H / 16;
    const int u0 = (int)((long)c * U / G), u1 = (int)((long)(c + 1) * U / G);
    const int b0 = (int)((long)c * NB / G), b1 = (int)((long)(c + 1) * NB / G);
    const int nu = u1 - u0, nb = b1 - b0;
    const uint32_t ucb = 8u * (H / 4), usb = 8u * ngH * 2u;          // unit: code / scale bytes per matrix
    const uint32_t dcb = 16u * (I / 4), dsb = 16u * ngI * 2u;         // down: per expert
    const size_t dexp = al16((size_t)dcb + 2 * dsb);                   // bytes per expert inside a block
    const uint32_t rsb = 16u * E * 2u;                                  // router slice per block

    if (tid == 0) {
        for (int i = 0; i < kPairs; ++i) mbar_init(&ubar[i], 1);
        for (int i = 0; i < kMaxBlocks; ++i) mbar_init(&dbar[i], (uint32_t)K);   // one arrival per expert
        mbar_init(rbar, 1);
        fence_barrier_init();
    }
    if (tid < 32) zrec[tid >> 1] = make_uint2(0u, 0u);
    __syncthreads();

    unsigned int nbar = 0;
    uint32_t rphase = 0;

    // --------------------------------------------------------------- prologue: h_0 and layer-0 logits
    if (tid == 0 && nb > 0) {
        mbar_arrive_expect_tx(rbar, rsb * nb);
        for (int bi = 0; bi < nb; ++bi)
            tma_load_1d(rbuf + (size_t)bi * rsb, a.layers[0].router_t + (size_t)(b0 + bi) * 16 * E, rsb, rbar);
    }
    double ssp = 0.0;
    for (int r = tid; r < nb * 16; r += kThreads) {
        const uint16_t v = a.x_in[b0 * 16 + r];
        a.hbuf[b0 * 16 + r] = v;
        if (a.hs_out) a.hs_out[b0 * 16 + r] = v;
        hnew[r] = (double)bf16_bits_to_f32(v);
        ssp = fma(hnew[r], hnew[r], ssp);
    }
    ssp = block_sum_d(ssp, redd);
    if (tid == 0 && a.norm && nb > 0) atomicAdd(a.ss, ssp);
    __syncthreads();
    if (nb > 0) {
        const bool ok = mbar_wait(rbar, rphase);
        rphase ^= 1u;
        if (ok) {
            const uint16_t *rs = reinterpret_cast<const uint16_t *>(rbuf);
            for (int e = tid; e < E; e += kThreads) {
                double p = 0.0;
                for (int r = 0; r < nb * 16; ++r) p = fma((double)bf16_bits_to_f32(rs[(size_t)r * E + e]), hnew[r], p);
                atomicAdd(a.acc + e, p);
            }
        }
    }
    grid_sync(a.bar, nbar++);

    for (int l = 0; l < L; ++l) {
        const StackLayer ly = a.layers[l];
        const double *accl = a.acc + (size_t)(l & 1) * E;
        const uint16_t *hcur = a.hbuf + (size_t)(l & 1) * H;
        uint16_t *hnext = a.hbuf + (size_t)((l + 1) & 1) * H;
        const uint32_t lphase = (uint32_t)(l & 1);

        // ---------------------------------------------------------- phase A
        const double xmul = a.norm ? ldexp(1.0, -pow2_rms_shift(__ldcg(a.ss + (l & 1)), H)) : 1.0;
        softmax_topk(accl, xmul, E, K, keys, sel, cand, prob, sinds, sscores, redd);
        if (c == 0 && tid < K) {
            a.inds_out[(size_t)l * K + tid] = sinds[tid];
            a.scores_out[(size_t)l * K + tid] = f32_to_bf16_bits(sscores[tid]);
        }
        {
            const int p = warp >> 1;
            if ((warp & 1) == 0 && lane == 0 && p < nu) {
                fence_barrier_init();   // generic reads of the buffers happened before these async writes
                const int u = u0 + p, k = u / (I / 8), rb = u % (I / 8);
                const size_t row0 = (size_t)sinds[k] * I + (size_t)rb * 8;
                unsigned char *dst = ubuf + (size_t)p * S.ubytes;
                mbar_arrive_expect_tx(&ubar[p], 2 * ucb + 4 * usb);
                tma_load_1d(dst, ly.wg + row0 * (H / 16), ucb, &ubar[p]);
                tma_load_1d(dst + ucb, ly.wu + row0 * (H / 16), ucb, &ubar[p]);
                tma_load_1d(dst + 2 * ucb, ly.sg + row0 * ngH, usb, &ubar[p]);
                tma_load_1d(dst + 2 * ucb + usb, ly.bg + row0 * ngH, usb, &ubar[p]);
                tma_load_1d(dst + 2 * ucb + 2 * usb, ly.su + row0 * ngH, usb, &ubar[p]);
                tma_load_1d(dst + 2 * ucb + 3 * usb, ly.bu + row0 * ngH, usb, &ubar[p]);
            }
            if (warp == kWarps - 1 && lane == 0 && l + 1 < L && nb > 0) {
                fence_barrier_init();
                mbar_arrive_expect_tx(rbar, rsb * nb);
                for (int bi = 0; bi < nb; ++bi)
                    tma_load_1d(rbuf + (size_t)bi * rsb, a.layers[l + 1].router_t + (size_t)(b0 + bi) * 16 * E, rsb,
                                rbar);
            }
        }
        // records of h_l (written by every CTA in the previous phase B; read through L2)
        build_recs_block<true>(hcur, ngH, xrec, xscale, xsum, (float)xmul, gexp);
        {
            const int p = warp >> 1, half = warp & 1;
            float accg = 0.f, accu = 0.f;
            bool wok = false;
            if (p < nu) {
                wok = mbar_wait(&ubar[p], lphase);
                const unsigned char *base = ubuf + (size_t)p * S.ubytes;
                const uint4 *grow = reinterpret_cast<const uint4 *>(base + (size_t)g * (H / 4));
                const uint4 *urow = reinterpret_cast<const uint4 *>(base + ucb + (size_t)g * (H / 4));
                const uint16_t *sgs = reinterpret_cast<const uint16_t *>(base + 2 * ucb);
                const uint16_t *bgs = sgs + 8 * ngH, *sus = bgs + 8 * ngH, *bus = sus + 8 * ngH;
                const int nsteps = (ngH + 3) >> 2;
                const int s0 = half * nsteps / 2, s1 = (half + 1) * nsteps / 2;
                const bool bact = rec_lane_active(lane);
                const int part = rec_lane_part(lane);
                if (wok) {
                    for (int j = s0; j < s1; ++j) {
                        const int Gj = 4 * j + t;
                        const bool gok = Gj < ngH;
                        const uint4 wv = gok ? grow[Gj] : make_uint4(0, 0, 0, 0);
                        const uint4 uv = gok ? urow[Gj] : make_uint4(0, 0, 0, 0);
                        const uint2 *rec = (bact && gok) ? xrec + (size_t)Gj * 16 : zrec;
                        int dg, du;
                        mma_step_i8(wv, uv, rec, part, dg, du);
                        if (gok) {
                            const int si = g * ngH + Gj;
                            const float sc = xscale[Gj], sm = xsum[Gj];
                            accg += sb_to_f32<kFp16>(sgs[si]) * ((float)dg * sc) + sb_to_f32<kFp16>(bgs[si]) * sm;
                            accu += sb_to_f32<kFp16>(sus[si]) * ((float)du * sc) + sb_to_f32<kFp16>(bus[si]) * sm;
                        }
                    }
                }
            }
            accg += __shfl_xor_sync(0xffffffffu, accg, 1);
            accu += __shfl_xor_sync(0xffffffffu, accu, 1);
            accg += __shfl_xor_sync(0xffffffffu, accg, 2);
            accu += __shfl_xor_sync(0xffffffffu, accu, 2);
            if (p < nu && t == 0) {
                red[((p * 2 + half) * 8 + g) * 2 + 0] = accg;
                red[((p * 2 + half) * 8 + g) * 2 + 1] = accu;
            }
            __syncthreads();
            if (p < nu && half == 0 && lane < 8) {
                const float gs = red[((p * 2) * 8 + lane) * 2 + 0] + red[((p * 2 + 1) * 8 + lane) * 2 + 0];
                const float us = red[((p * 2) * 8 + lane) * 2 + 1] + red[((p * 2 + 1) * 8 + lane) * 2 + 1];
                const float gv = bf16r(gs), uv = bf16r(us);
                const float sig = bf16r(1.0f / (1.0f + expf(-gv)));
                const float av = wok ? bf16r(bf16r(gv * sig) * uv) : 0.f;
                const int u = u0 + p, k = u / (I / 8), rb = u % (I / 8);
                a.act[(size_t)k * I + rb * 8 + lane] = f32_to_bf16_bits(av);
            }
        }
        __syncthreads();
        // down rows into the freed unit buffers: one (block, expert) per warp, in parallel
        for (int task = warp; task < nb * K; task += kWarps) {
            if (lane == 0) {
                const int bi = task / K, k = task % K;
                fence_barrier_init();   // the unit buffers were read by the generic proxy above
                const size_t row0 = (size_t)sinds[k] * H + (size_t)(b0 + bi) * 16;
                unsigned char *dst = ubuf + (size_t)bi * S.dbytes + (size_t)k * dexp;
                mbar_arrive_expect_tx(&dbar[bi], dcb + 2 * dsb);
                tma_load_1d(dst, ly.wd + row0 * (I / 16), dcb, &dbar[bi]);
                tma_load_1d(dst + dcb, ly.sd + row0 * ngI, dsb, &dbar[bi]);
                tma_load_1d(dst + dcb + dsb, ly.bd + row0 * ngI, dsb, &dbar[bi]);
            }
        }
        grid_sync(a.bar, nbar++);

        // ---------------------------------------------------------- phase B
        build_recs_block<true>(a.act, K * ngI, arec, ascale, asum, 1.0f, gexp);
        for (int task = warp; task < nb * K; task += kWarps) {
            const int bi = task / K, k = task % K;
            const bool wok = mbar_wait(&dbar[bi], lphase);
            const unsigned char *base = ubuf + (size_t)bi * S.dbytes + (size_t)k * dexp;
            const uint16_t *sds = reinterpret_cast<const uint16_t *>(base + dcb);
            const uint16_t *bds = sds + 16 * ngI;
            const uint4 *rowa = reinterpret_cast<const uint4 *>(base + (size_t)g * (I / 4));
            const uint4 *rowbp = reinterpret_cast<const uint4 *>(base + (size_t)(g + 8) * (I / 4));
            const uint2 *rk = arec + (size_t)k * ngI * 16;
            const float *sck = ascale + k * ngI, *smk = asum + k * ngI;
            const bool bact = rec_lane_active(lane);
            const int part = rec_lane_part(lane);
            float acca = 0.f, accb = 0.f;
            if (wok) {
                for (int j = 0; j < (ngI + 3) >> 2; ++j) {
                    const int Gj = 4 * j + t;
                    const bool gok = Gj < ngI;
                    const uint4 qa = gok ? rowa[Gj] : make_uint4(0, 0, 0, 0);
                    const uint4 qb = gok ? rowbp[Gj] : make_uint4(0, 0, 0, 0);
                    const uint2 *rec = (bact && gok) ? rk + (size_t)Gj * 16 : zrec;
                    int da, db;
                    mma_step_i8(qa, qb, rec, part, da, db);
                    if (gok) {
                        const int sa = g * ngI + Gj, sbi = (g + 8) * ngI + Gj;
                        const float sc = sck[Gj], sm = smk[Gj];
                        acca += sb_to_f32<kFp16>(sds[sa]) * ((float)da * sc) + sb_to_f32<kFp16>(bds[sa]) * sm;
                        accb += sb_to_f32<kFp16>(sds[sbi]) * ((float)db * sc) + sb_to_f32<kFp16>(bds[sbi]) * sm;
                    }
                }
            }
            acca += __shfl_xor_sync(0xffffffffu, acca, 1);
            accb += __shfl_xor_sync(0xffffffffu, accb, 1);
            acca += __shfl_xor_sync(0xffffffffu, acca, 2);
            accb += __shfl_xor_sync(0xffffffffu, accb, 2);
            if (t == 0) {
                yk[(bi * K + k) * 16 + g] = wok ? bf16r(acca) : 0.f;
                yk[(bi * K + k) * 16 + 8 + g] = wok ? bf16r(accb) : 0.f;
            }
        }
        __syncthreads();
        double ssn = 0.0;
        for (int r = tid; r < nb * 16; r += kThreads) {
            const int bi = r >> 4, rr = r & 15, row = (b0 + bi) * 16 + rr;
            float accv = 0.f;
            for (int k = 0; k < K; ++k) {
                const float pk = bf16r(yk[(bi * K + k) * 16 + rr] * sscores[k]);
                accv = (k == 0) ? pk : bf16r(accv + pk);
            }
            accv = bf16r(bf16_bits_to_f32(__ldcg(hcur + row)) + accv);
            const uint16_t hb = f32_to_bf16_bits(accv);
            hnext[row] = hb;
            if (a.hs_out) a.hs_out[(size_t)(l + 1) * H + row] = hb;
            if (l + 1 == L) a.y_out[row] = hb;
            hnew[r] = (double)accv;
            ssn = fma(hnew[r], hnew[r], ssn);
        }
        ssn = block_sum_d(ssn, redd);
        if (tid == 0 && a.norm && nb > 0 && l + 1 < L) atomicAdd(a.ss + ((l + 1) & 1), ssn);
        __syncthreads();
        if (l + 1 < L && nb > 0) {
            const bool ok = mbar_wait(rbar, rphase);
            rphase ^= 1u;
            double *accn = a.acc + (size_t)((l + 1) & 1) * E;
            if (ok) {
                const uint16_t *rs = reinterpret_cast<const uint16_t *>(rbuf);
                for (int e = tid; e < E; e += kThreads) {
                    double p = 0.0;
                    for (int r = 0; r < nb * 16; ++r)
                        p = fma((double)bf16_bits_to_f32(rs[(size_t)r * E + e]), hnew[r], p);
                    atomicAdd(accn + e, p);
                }
            }
        }
        if (c == 0) {   // layer l's accumulators were consumed in phase A; ready them for l + 2
            double *accz = a.acc + (size_t)(l & 1) * E;
            for (int e = tid; e < E; e += kThreads) accz[e] = 0.0;
            if (tid == 0) a.ss[l & 1] = 0.0;
        }
        if (l + 1 < L) grid_sync(a.bar, nbar++);
    }
}

struct StackWs {
    double *acc, *ss;
    uint16_t *hbuf, *act;
    unsigned int *bar;
    size_t bytes;
};

StackWs carve(void *base, int H, int I, int E, int K) {
    StackWs w{};
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t n) { char *q = p ? p + off : nullptr; off += al256(n); return q; };
    w.acc = reinterpret_cast<double *>(take((size_t)(2 * E + 2) * 8));
    w.ss = w.acc + 2 * E;
    w.bar = reinterpret_cast<unsigned int *>(take(256));
    w.hbuf = reinterpret_cast<uint16_t *>(take((size_t)2 * H * 2));
    w.act = reinterpret_cast<uint16_t *>(take((size_t)K * I * 2));
    w.bytes = off;
    return w;
}

// bytes of the acc + barrier prefix that must be zero before every launch
size_t zero_prefix(int E) { return al256((size_t)(2 * E + 2) * 8) + 256; }

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
    if (L <= 0 || H % 256 || I % 64 || E <= 0 || E > kMaxE || K <= 0 || K > 32 || K > E)
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
    const int U = K * (I / 8), NB = H / 16;
    if ((U + G - 1) / G > kPairs || (NB + G - 1) / G > kMaxBlocks)
        return moe_set_error(MOE_EINVAL, "stack_decode: %d CTAs too few for %d units / %d blocks", G, U, NB);
    const SmemLayout S(H, I, E, K, G);
    if (S.total > 227 * 1024)
        return moe_set_error(MOE_EINVAL, "stack_decode: %zu bytes of shared memory needed", S.total);
    StackWs w = carve(workspace, H, I, E, K);
    auto st = as_stream(stream);
    MOE_CUDA_TRY(cudaMemsetAsync(workspace, 0, zero_prefix(E), st));
    StackArgs a{static_cast<const StackLayer *>(layers), L, H, I, E, K, static_cast<const uint16_t *>(x),
                static_cast<uint16_t *>(y), inds_out, static_cast<uint16_t *>(scores_out),
                static_cast<uint16_t *>(hs_out), w.acc, w.ss, norm, w.hbuf, w.act, w.bar};
    void *kargs[] = {&a};
    auto kern = sb_fp16 ? (const void *)stack_kernel<true> : (const void *)stack_kernel<false>;
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S.total));
    MOE_CUDA_TRY(cudaLaunchCooperativeKernel(kern, dim3(G), dim3(kThreads), kargs, S.total, st));
    return MOE_OK;
}

