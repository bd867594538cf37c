// Decode expert GEMVs over 2-bit affine (group 64) weights in MLX layout.
//
// Data movement: each CTA owns a contiguous block of weight rows (8 gate + 8 up rows of one
// routed expert, or 16 down rows of every routed expert) and pulls it -- codes, scales and
// biases -- into shared memory with 1-D TMA bulk copies (cp.async.bulk, no multicast) that
// complete on an mbarrier; the input's MMA records arrive the same way. With programmatic
// dependent launch the down kernel issues its weight copies while the gate/up kernel is
// still running.
//
// Dot products: m16n8k32 u8 x s8 integer MMAs (gemv_i8.cuh): codes masked in place as u8,
// input split exactly into int8 hi/lo parts per group, exact int32 accumulation; the
// per-group affine terms are applied in fp32:  row += s[G] * dot[G] * 2^E[G] + b[G] * sum[G].
//
//   gate/up  grid (I/8, K, T), 4 warps split the H axis of one block of 8 gate rows (MMA
//            rows 0-7) and the matching 8 up rows (rows 8-15); SwiGLU in the epilogue
//            (cpp/src/layers.cpp:349-358, cpp/src/kernels.cpp:1090-1094). The last of the 8
//            CTAs covering a 64-wide group of the activations builds that group's record
//            for the down kernel (atomic ticket per group, re-armed by the builder).
//   down     grid (H/16, T); warp k = routed expert k over all of I for 16 output rows; the
//            CTA combines the K experts with the routing scores (loader.py:914,965).
#include "common.cuh"
#include "gemv_i8.cuh"
#include "internal.h"

namespace {

constexpr int kGuWarps = 4;        // K-split warps per gate/up CTA (one 8-row block)
constexpr int kMaxK = 16;


// --------------------------------------------------------------------- gate + up

struct GuArgs {
    const uint16_t *x;
    const uint2 *xrec;           // optional pre-built records of x ([T][ngH][16])
    const float *xscale, *xsum;  // [T][pad4(ngH)]
    const uint32_t *slots;
    const uint32_t *wg, *wu;
    const uint16_t *sg, *bg, *su, *bu;
    int H, I, K, cap;
    uint16_t *act;               // [T][K][I]
    uint2 *arec;                 // optional records of act ([T][K][ngI][16])
    float *ascale, *asum;        // [T][pad4(K*ngI)]
    unsigned int *acnt;          // [T][K][ngI] tickets, zero between launches
    uint32_t slot_base;          // slot = slots[] - slot_base (expert-parallel shards); >= cap: skipped
};

struct GuLayout {
    size_t xraw, rec, scale, sum, zero, w, red, total;
    MOE_HD GuLayout(int H, bool self_stage) {
        const int ng = H / 64;
        xraw = 128;
        rec = xraw + (self_stage ? al16((size_t)H * 2) : 0);
        scale = rec + (size_t)ng * 128;
        sum = scale + al16((size_t)pad4(ng) * 4);
        zero = sum + al16((size_t)pad4(ng) * 4);
        w = al128(zero + 128);
        red = w + al16(16 * (size_t)(H / 4) + 4 * 8 * (size_t)ng * 2);
        total = red + kGuWarps * 8 * 2 * 4;
    }
};

template <bool kFp16>
__global__ void __launch_bounds__(kGuWarps * 32) gateup_kernel(GuArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int H = a.H, I = a.I, K = a.K;
    const int ng = H >> 6, rowb = H >> 2;
    const bool self_stage = (a.xrec == nullptr);
    const GuLayout L(H, self_stage);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint16_t *xraw = reinterpret_cast<uint16_t *>(smem + L.xraw);
    uint2 *xrec = reinterpret_cast<uint2 *>(smem + L.rec);
    float *xscale = reinterpret_cast<float *>(smem + L.scale);
    float *xsum = reinterpret_cast<float *>(smem + L.sum);
    uint2 *zrec = reinterpret_cast<uint2 *>(smem + L.zero);
    unsigned char *wsm = smem + L.w;
    float *red = reinterpret_cast<float *>(smem + L.red);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int k = blockIdx.y, tok = blockIdx.z;
    const int r0 = blockIdx.x * 8;

    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 32) zrec[threadIdx.x >> 1] = make_uint2(0u, 0u);
    __syncthreads();

    pdl_wait();                       // router (slots, x records) and the producer of x are done
    pdl_launch_dependents();

    const uint32_t slot_raw = a.slots[(size_t)tok * K + k] - a.slot_base;
    const bool sok = slot_raw < (uint32_t)a.cap;
    const size_t row0 = (size_t)(sok ? slot_raw : 0) * I + r0;
    const uint32_t cb = 8u * rowb, sb = 8u * ng * 2u;
    if (threadIdx.x == 0) {
        if (sok) {
            mbar_arrive_expect_tx(&bars[1], 2 * cb + 4 * sb);
            tma_load_1d(wsm, a.wg + row0 * (H >> 4), cb, &bars[1]);
            tma_load_1d(wsm + cb, a.wu + row0 * (H >> 4), cb, &bars[1]);
            tma_load_1d(wsm + 2 * cb, a.sg + row0 * ng, sb, &bars[1]);
            tma_load_1d(wsm + 2 * cb + sb, a.bg + row0 * ng, sb, &bars[1]);
            tma_load_1d(wsm + 2 * cb + 2 * sb, a.su + row0 * ng, sb, &bars[1]);
            tma_load_1d(wsm + 2 * cb + 3 * sb, a.bu + row0 * ng, sb, &bars[1]);
        }
        if (self_stage) {
            mbar_arrive_expect_tx(&bars[0], (uint32_t)H * 2);
            tma_load_1d(xraw, a.x + (size_t)tok * H, (uint32_t)H * 2, &bars[0]);
        } else {
            const uint32_t rb = (uint32_t)ng * 128, fb = (uint32_t)pad4(ng) * 4;
            mbar_arrive_expect_tx(&bars[0], rb + 2 * fb);
            tma_load_1d(xrec, a.xrec + (size_t)tok * ng * 16, rb, &bars[0]);
            tma_load_1d(xscale, a.xscale + (size_t)tok * pad4(ng), fb, &bars[0]);
            tma_load_1d(xsum, a.xsum + (size_t)tok * pad4(ng), fb, &bars[0]);
        }
    }
    const bool xok = mbar_wait(&bars[0], 0);
    if (self_stage) {
        // records of x from the raw copy: one aligned half warp per group
        for (int G0 = 0; G0 < ng; G0 += blockDim.x / 16) {
            const int G = G0 + (threadIdx.x >> 4);
            const bool v = xok && G < ng;
            build_rec_group(xraw + (size_t)(v ? G : 0) * 64, v, threadIdx.x & 15, xrec + (size_t)G * 16,
                            xscale + G, xsum + G);
        }
    }
    __syncthreads();
    // the weight copies were issued whenever the slot is valid: wait for them even when the x
    // wait failed, so no bulk copy is still writing shared memory when the CTA exits
    const bool wdone = sok && mbar_wait(&bars[1], 0);
    const bool wok = wdone && xok;

    const uint16_t *sgs = reinterpret_cast<const uint16_t *>(wsm + 2 * cb);
    const uint16_t *bgs = sgs + 8 * ng, *sus = bgs + 8 * ng, *bus = sus + 8 * ng;
    float accg = 0.f, accu = 0.f;
    if (wok) {
        const uint4 *grow = reinterpret_cast<const uint4 *>(wsm + (size_t)g * rowb);
        const uint4 *urow = reinterpret_cast<const uint4 *>(wsm + cb + (size_t)g * rowb);
        const int nsteps = (ng + 3) >> 2;
        const int s0 = (warp * nsteps) / kGuWarps, s1 = ((warp + 1) * nsteps) / kGuWarps;
        const bool bact = rec_lane_active(lane);
        const int part = rec_lane_part(lane);
        for (int j = s0; j < s1; ++j) {
            const int G = 4 * j + t;
            const bool gok = G < ng;
            const uint4 wv = gok ? grow[G] : make_uint4(0, 0, 0, 0);
            const uint4 uv = gok ? urow[G] : make_uint4(0, 0, 0, 0);
            const uint2 *rec = (bact && gok) ? xrec + (size_t)G * 16 : zrec;
            int dg, du;
            mma_step_i8(wv, uv, rec, part, dg, du);
            if (gok) {
                const int si = g * ng + G;
                const float sc = xscale[G], sm = xsum[G];
                accg += sb_to_f32<kFp16>(sgs[si]) * ((float)dg * sc) + sb_to_f32<kFp16>(bgs[si]) * sm;
                accu += sb_to_f32<kFp16>(sus[si]) * ((float)du * sc) + sb_to_f32<kFp16>(bus[si]) * sm;
            }
        }
    }
    accg += __shfl_xor_sync(0xffffffffu, accg, 1);
    accu += __shfl_xor_sync(0xffffffffu, accu, 1);
    accg += __shfl_xor_sync(0xffffffffu, accg, 2);
    accu += __shfl_xor_sync(0xffffffffu, accu, 2);
    if (t == 0) {
        red[(warp * 8 + g) * 2 + 0] = accg;
        red[(warp * 8 + g) * 2 + 1] = accu;
    }
    __syncthreads();
    if (warp == 0) {
        const int p = r0 + (lane & 7);
        if (lane < 8) {
            float sgsum = 0.f, susum = 0.f;
#pragma unroll
            for (int w = 0; w < kGuWarps; ++w) {
                sgsum += red[(w * 8 + lane) * 2 + 0];
                susum += red[(w * 8 + lane) * 2 + 1];
            }
            const float gv = bf16r(sgsum), uv = bf16r(susum);
            // SwiGLU rounded after every op, like an MLX bf16 graph
            const float sig = bf16r(1.0f / (1.0f + expf(-gv)));
            const float av = wok ? bf16r(bf16r(gv * sig) * uv) : 0.f;
            a.act[((size_t)tok * K + k) * I + p] = f32_to_bf16_bits(av);
        }
        if (a.arec) {
            // the last of the 8 CTAs of this 64-wide group builds its record
            const int ngI = I >> 6, G = r0 >> 6;
            const size_t gi = ((size_t)tok * K + k) * ngI + G;
            unsigned int last = 0;
            __threadfence();
            __syncwarp();
            if (lane == 0) last = (atomicAdd(a.acnt + gi, 1u) == 7u) ? 1u : 0u;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                const uint16_t *src = a.act + ((size_t)tok * K + k) * I + (size_t)G * 64;
                // read the group through L2 (other CTAs wrote it) into registers, then build
                __shared__ __align__(16) uint16_t grp[64];
                const uint32_t two = __ldcg(reinterpret_cast<const unsigned int *>(src) + lane);
                reinterpret_cast<uint32_t *>(grp)[lane] = two;
                __syncwarp();
                const size_t fo = (size_t)tok * pad4(K * ngI) + (size_t)k * ngI + G;
                build_rec_group(grp, lane < 16, lane & 15, a.arec + gi * 16, a.ascale + fo, a.asum + fo);
                if (lane == 0) a.acnt[gi] = 0u;
            }
        }
    }
}

// --------------------------------------------------------------------- down + combine

struct DnArgs {
    const uint16_t *act;
    const uint2 *arec;           // optional records of act (from the gate/up kernel)
    const float *ascale, *asum;  // [T][pad4(K*ngI)]
    const uint32_t *slots;
    const uint16_t *scores;
    const uint32_t *wd;
    const uint16_t *sd, *bd;
    int H, I, K, cap;
    const uint16_t *addend, *resid;
    uint16_t *y, *yk;
    uint32_t slot_base;          // as GuArgs::slot_base
};

struct DnLayout {
    size_t araw, rec, scale, sum, zero, yks, warps, warp_bytes, total;
    MOE_HD DnLayout(int I, int K, bool self_stage) {
        const int ng = I / 64;
        araw = 256;                                   // after K+1 mbarriers (K <= 16)
        rec = araw + (self_stage ? al16((size_t)K * I * 2) : 0);
        scale = rec + (size_t)K * ng * 128;
        sum = scale + al16((size_t)pad4(K * ng) * 4);
        zero = sum + al16((size_t)pad4(K * ng) * 4);
        yks = zero + 128;
        warps = al128(yks + (size_t)K * 16 * 4);
        warp_bytes = al128(16 * (size_t)(I / 4) + 2 * 16 * (size_t)ng * 2);
        total = warps + (size_t)K * warp_bytes;
    }
};

template <bool kFp16>
__global__ void __launch_bounds__(kMaxK * 32) down_kernel(DnArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int H = a.H, I = a.I, K = a.K;
    const int ng = I >> 6, rowb = I >> 2;
    const bool self_stage = (a.arec == nullptr);
    const DnLayout L(I, K, self_stage);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    uint16_t *araw = reinterpret_cast<uint16_t *>(smem + L.araw);
    uint2 *arec = reinterpret_cast<uint2 *>(smem + L.rec);
    float *ascale = reinterpret_cast<float *>(smem + L.scale);
    float *asum = reinterpret_cast<float *>(smem + L.sum);
    uint2 *zrec = reinterpret_cast<uint2 *>(smem + L.zero);
    float *yks = reinterpret_cast<float *>(smem + L.yks);

    const int lane = threadIdx.x & 31, k = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int tok = blockIdx.y;
    const int r0 = blockIdx.x * 16;
    unsigned char *my = smem + L.warps + (size_t)k * L.warp_bytes;

    if (threadIdx.x == 0) {
        for (int i = 0; i <= K; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 32) zrec[threadIdx.x >> 1] = make_uint2(0u, 0u);
    __syncthreads();

    // The routing (slots) was produced two kernels back and is complete once the gate/up
    // kernel has started (it waits on the router before triggering this launch), so the
    // weight copies go out before waiting on the activations.
    const uint32_t slot_raw = a.slots[(size_t)tok * K + k] - a.slot_base;
    const bool sok = slot_raw < (uint32_t)a.cap;
    const size_t row0 = (size_t)(sok ? slot_raw : 0) * H + r0;
    const uint32_t cb = 16u * rowb, sb = 16u * ng * 2u;
    if (lane == 0 && sok) {
        mbar_arrive_expect_tx(&bars[1 + k], cb + 2 * sb);
        tma_load_1d(my, a.wd + row0 * (I >> 4), cb, &bars[1 + k]);
        tma_load_1d(my + cb, a.sd + row0 * ng, sb, &bars[1 + k]);
        tma_load_1d(my + cb + sb, a.bd + row0 * ng, sb, &bars[1 + k]);
    }

    pdl_wait();                       // activations (gate/up kernel) are complete
    pdl_launch_dependents();

    if (threadIdx.x == 0) {
        if (self_stage) {
            const uint32_t ab = (uint32_t)K * I * 2;
            mbar_arrive_expect_tx(&bars[0], ab);
            tma_load_1d(araw, a.act + (size_t)tok * K * I, ab, &bars[0]);
        } else {
            const uint32_t rb = (uint32_t)K * ng * 128, fb = (uint32_t)pad4(K * ng) * 4;
            mbar_arrive_expect_tx(&bars[0], rb + 2 * fb);
            tma_load_1d(arec, a.arec + (size_t)tok * K * ng * 16, rb, &bars[0]);
            tma_load_1d(ascale, a.ascale + (size_t)tok * pad4(K * ng), fb, &bars[0]);
            tma_load_1d(asum, a.asum + (size_t)tok * pad4(K * ng), fb, &bars[0]);
        }
    }
    const bool aok = mbar_wait(&bars[0], 0);
    if (self_stage) {
        for (int G0 = 0; G0 < K * ng; G0 += blockDim.x / 16) {     // K vectors back to back
            const int G = G0 + (threadIdx.x >> 4);
            const bool v = aok && G < K * ng;
            build_rec_group(araw + (size_t)(v ? G : 0) * 64, v, threadIdx.x & 15, arec + (size_t)G * 16,
                            ascale + G, asum + G);
        }
    }
    __syncthreads();
    // wait for this expert's weight copies whenever they were issued (even after a failed
    // activation wait), so no bulk copy is in flight when the CTA exits
    const bool wdone = sok && mbar_wait(&bars[1 + k], 0);
    const bool wok = wdone && aok;

    const uint16_t *sds = reinterpret_cast<const uint16_t *>(my + cb);
    const uint16_t *bds = sds + 16 * ng;
    float acca = 0.f, accb = 0.f;
    if (wok) {
        const uint2 *rk = arec + (size_t)k * ng * 16;
        const float *sck = ascale + k * ng, *smk = asum + k * ng;
        const uint4 *rowa = reinterpret_cast<const uint4 *>(my + (size_t)g * rowb);
        const uint4 *rowbp = reinterpret_cast<const uint4 *>(my + (size_t)(g + 8) * rowb);
        const int nsteps = (ng + 3) >> 2;
        const bool bact = rec_lane_active(lane);
        const int part = rec_lane_part(lane);
        for (int j = 0; j < nsteps; ++j) {
            const int G = 4 * j + t;
            const bool gok = G < ng;
            const uint4 qa = gok ? rowa[G] : make_uint4(0, 0, 0, 0);
            const uint4 qb = gok ? rowbp[G] : make_uint4(0, 0, 0, 0);
            const uint2 *rec = (bact && gok) ? rk + (size_t)G * 16 : zrec;
            int da, db;
            mma_step_i8(qa, qb, rec, part, da, db);
            if (gok) {
                const int sa = g * ng + G, sbi = (g + 8) * ng + G;
                const float sc = sck[G], sm = smk[G];
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
        const float ya = wok ? bf16r(acca) : 0.f, yb = wok ? bf16r(accb) : 0.f;
        yks[k * 16 + g] = ya;
        yks[k * 16 + 8 + g] = yb;
        if (a.yk) {
            a.yk[((size_t)tok * K + k) * H + r0 + g] = f32_to_bf16_bits(ya);
            a.yk[((size_t)tok * K + k) * H + r0 + 8 + g] = f32_to_bf16_bits(yb);
        }
    }
    __syncthreads();
    if (a.y && threadIdx.x < 16) {
        const int rr = r0 + threadIdx.x;
        float acc = 0.f;
        for (int kk = 0; kk < K; ++kk) {
            const float sc = bf16_bits_to_f32(a.scores[(size_t)tok * K + kk]);
            const float pk = bf16r(yks[kk * 16 + threadIdx.x] * sc);
            acc = (kk == 0) ? pk : bf16r(acc + pk);
        }
        if (a.addend) acc = bf16r(acc + bf16_bits_to_f32(a.addend[(size_t)tok * H + rr]));
        if (a.resid) acc = bf16r(bf16_bits_to_f32(a.resid[(size_t)tok * H + rr]) + acc);
        a.y[(size_t)tok * H + rr] = f32_to_bf16_bits(acc);
    }
}

int check_common(int H, int I, int K, int T, int cap, int bits, int group_size, const char *who) {
    if (bits != 2 || group_size != 64)
        return moe_set_error(MOE_EINVAL, "%s: only bits=2, group_size=64 are implemented (got %d, %d)", who,
                             bits, group_size);
    if (T <= 0 || K <= 0 || K > kMaxK || H <= 0 || I <= 0 || H % 64 || I % 64 || cap <= 0)
        return moe_set_error(MOE_EINVAL, "%s: bad sizes T=%d H=%d I=%d K=%d cap=%d", who, T, H, I, K, cap);
    return MOE_OK;
}

bool misaligned(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }  // null is aligned

}  // namespace

__device__ unsigned int g_moe_device_error = 0;

int moe_experts_gateup_ex(const void *x, const void *xrec, const float *xscale, const float *xsum, int T,
                          int H, int I, int K, int cap, const uint32_t *slots, const uint32_t *wg,
                          const void *sg, const void *bg, const uint32_t *wu, const void *su, const void *bu,
                          int bits, int group_size, int sb_fp16, void *act, void *arec, float *ascale,
                          float *asum, unsigned int *acnt, void *stream, uint32_t slot_base) {
    int rc = check_common(H, I, K, T, cap, bits, group_size, "experts_gateup");
    if (rc) return rc;
    if (!x || !slots || !wg || !wu || !sg || !bg || !su || !bu || !act)
        return moe_set_error(MOE_EINVAL, "experts_gateup: null pointer");
    if (misaligned(x) || misaligned(wg) || misaligned(wu) || misaligned(sg) || misaligned(bg) ||
        misaligned(su) || misaligned(bu) || misaligned(xrec) || misaligned(xscale) || misaligned(xsum))
        return moe_set_error(MOE_EINVAL, "experts_gateup: tensors must be 16-byte aligned");
    if ((xrec != nullptr) != (xscale != nullptr) || (xrec != nullptr) != (xsum != nullptr) ||
        (arec != nullptr) != (ascale != nullptr) || (arec != nullptr) != (asum != nullptr) ||
        (arec != nullptr) != (acnt != nullptr))
        return moe_set_error(MOE_EINVAL, "experts_gateup: incomplete record buffers");
    const GuLayout L(H, xrec == nullptr);
    if (L.total > 227 * 1024) return moe_set_error(MOE_EINVAL, "experts_gateup: H=%d too large", H);
    GuArgs a{static_cast<const uint16_t *>(x), static_cast<const uint2 *>(xrec), xscale, xsum, slots, wg, wu,
             static_cast<const uint16_t *>(sg), static_cast<const uint16_t *>(bg),
             static_cast<const uint16_t *>(su), static_cast<const uint16_t *>(bu), H, I, K, cap,
             static_cast<uint16_t *>(act), static_cast<uint2 *>(arec), ascale, asum, acnt, slot_base};
    dim3 grid(I / 8, K, T);
    cudaError_t e = sb_fp16 ? launch_pdl(gateup_kernel<true>, grid, dim3(kGuWarps * 32), L.total, as_stream(stream), a)
                            : launch_pdl(gateup_kernel<false>, grid, dim3(kGuWarps * 32), L.total, as_stream(stream), a);
    if (e != cudaSuccess) return moe_set_cuda_error(e);
    return MOE_OK;
}

int moe_experts_down_ex(const void *act, const void *arec, const float *ascale, const float *asum, int T, int H,
                        int I, int K, int cap, const uint32_t *slots, const void *scores, const uint32_t *wd,
                        const void *sd, const void *bd, int bits, int group_size, int sb_fp16,
                        const void *addend, const void *resid, void *y, void *yk, void *stream,
                        uint32_t slot_base) {
    int rc = check_common(H, I, K, T, cap, bits, group_size, "experts_down");
    if (rc) return rc;
    if (!act || !slots || !wd || !sd || !bd) return moe_set_error(MOE_EINVAL, "experts_down: null pointer");
    if (y && !scores) return moe_set_error(MOE_EINVAL, "experts_down: y needs scores");
    if (!y && !yk) return moe_set_error(MOE_EINVAL, "experts_down: no output requested");
    if ((arec != nullptr) != (ascale != nullptr) || (arec != nullptr) != (asum != nullptr))
        return moe_set_error(MOE_EINVAL, "experts_down: incomplete record buffers");
    if (misaligned(act) || misaligned(wd) || misaligned(sd) || misaligned(bd) || misaligned(arec) ||
        misaligned(ascale) || misaligned(asum))
        return moe_set_error(MOE_EINVAL, "experts_down: tensors must be 16-byte aligned");
    const DnLayout L(I, K, arec == nullptr);
    if (L.total > 227 * 1024) return moe_set_error(MOE_EINVAL, "experts_down: K*I too large");
    DnArgs a{static_cast<const uint16_t *>(act), static_cast<const uint2 *>(arec), ascale, asum, slots,
             static_cast<const uint16_t *>(scores), wd, static_cast<const uint16_t *>(sd),
             static_cast<const uint16_t *>(bd), H, I, K, cap, static_cast<const uint16_t *>(addend),
             static_cast<const uint16_t *>(resid), static_cast<uint16_t *>(y), static_cast<uint16_t *>(yk),
             slot_base};
    dim3 grid(H / 16, T);
    cudaError_t e = sb_fp16 ? launch_pdl(down_kernel<true>, grid, dim3(K * 32), L.total, as_stream(stream), a)
                            : launch_pdl(down_kernel<false>, grid, dim3(K * 32), L.total, as_stream(stream), a);
    if (e != cudaSuccess) return moe_set_cuda_error(e);
    return MOE_OK;
}

extern "C" int moe_experts_gateup(const void *x, int T, int H, int I, int K, int cap, const uint32_t *slots,
                                  const uint32_t *wg, const void *sg, const void *bg,
                                  const uint32_t *wu, const void *su, const void *bu, int bits,
                                  int group_size, int sb_fp16, void *act, void *stream) {
    return moe_experts_gateup_ex(x, nullptr, nullptr, nullptr, T, H, I, K, cap, slots, wg, sg, bg, wu, su, bu,
                                 bits, group_size, sb_fp16, act, nullptr, nullptr, nullptr, nullptr, stream);
}

extern "C" int moe_experts_down(const void *act, int T, int H, int I, int K, int cap, const uint32_t *slots,
                                const void *scores, const uint32_t *wd, const void *sd,
                                const void *bd, int bits, int group_size, int sb_fp16,
                                const void *addend, const void *resid, void *y, void *yk,
                                void *stream) {
    return moe_experts_down_ex(act, nullptr, nullptr, nullptr, T, H, I, K, cap, slots, scores, wd, sd, bd, bits,
                               group_size, sb_fp16, addend, resid, y, yk, stream);
}

extern "C" int moe_device_error(int clear) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_moe_device_error, sizeof(v));
    if (e != cudaSuccess) return moe_set_cuda_error(e);
    if (clear) {
        unsigned int z = 0;
        e = cudaMemcpyToSymbol(g_moe_device_error, &z, sizeof(z));
        if (e != cudaSuccess) return moe_set_cuda_error(e);
    }
    return (int)v;
}
