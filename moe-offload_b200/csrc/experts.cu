// Decode expert GEMVs over 2-bit affine (group 64) weights in MLX layout.
//
// Both kernels run the dot products on the tensor cores through m16n8k16 bf16 MMAs whose
// A operand is built in registers from the packed codes (expand_word: 10 integer ops per
// 16 codes, no per-code shift or convert) and whose B operand is a pre-scaled copy of the
// input vector staged in shared memory. A GEMV has one useful column; the N dimension is
// used instead to process four different 64-code groups per MMA: lane quad t of every row
// supplies group 4j+t, and B column n holds the input of group 4j+n on the k-slots of lane
// t == n only, so D[row][n] is the row's partial dot over group 4j+n. Each lane loads a
// full 16-byte group of its row per step, which keeps the weight stream 16-byte coalesced.
//
//   gate/up  grid (I/8, K, T), kGuWarps warps split the H axis; MMA rows 0-7 are gate rows
//            r..r+7 of the routed expert, rows 8-15 the matching up rows, so SwiGLU happens
//            in the epilogue without another pass (layers.cpp:349-358, kernels.cpp:1090).
//   down     grid (H/16, T), one warp per routed expert over all of I; the CTA combines the
//            K experts' 16 output rows with the routing scores (loader.py:914,965).
#include "common.cuh"

namespace {

constexpr int kGuWarps = 4;       // K-split warps of the gate/up kernel
constexpr int kGuMaxSteps = 4;    // 4 groups per step -> H <= kGuWarps*kGuMaxSteps*256 = 4096
constexpr int kDnMaxSteps = 8;    // down: I <= 8*256 = 2048 (template instances 4 and 8)
constexpr int kMaxK = 16;         // routed experts per token handled by one down CTA

template <bool kFp16>
struct SB {
    static MOE_D float get(const uint16_t *p, size_t i) { return sb_to_f32<kFp16>(__ldg(p + i)); }
};

// --------------------------------------------------------------------- gate + up

template <bool kFp16>
__global__ void __launch_bounds__(kGuWarps * 32) gateup_kernel(
    const uint16_t *__restrict__ x, const uint32_t *__restrict__ slots,
    const uint32_t *__restrict__ wg, const uint16_t *__restrict__ sg, const uint16_t *__restrict__ bg,
    const uint32_t *__restrict__ wu, const uint16_t *__restrict__ su, const uint16_t *__restrict__ bu,
    int H, int I, int K, int cap, uint16_t *__restrict__ act) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int ngroups = H >> 6;
    uint2 *xfrag = reinterpret_cast<uint2 *>(smem);                       // [ngroups][16]
    float *corr = reinterpret_cast<float *>(smem + (size_t)ngroups * 128);  // [ngroups]
    float *xsum = corr + ngroups;                                          // [ngroups]
    float *red = xsum + ngroups;                                           // [kGuWarps][8][2]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int k = blockIdx.y, tok = blockIdx.z;
    const int r = blockIdx.x * 8 + g;
    const uint32_t slot_raw = slots[(size_t)tok * K + k];
    const bool sok = slot_raw < (uint32_t)cap;          // out-of-range slot: no loads, zero output
    const bool rok = r < I && sok;
    const size_t slot = sok ? slot_raw : 0;

    const int nsteps = (ngroups + 3) >> 2;
    const int s0 = (warp * nsteps) / kGuWarps, s1 = ((warp + 1) * nsteps) / kGuWarps;

    // 1) weight stream first: every load of this warp in flight before anything else
    const size_t row = slot * I + r;
    const uint4 *gw = reinterpret_cast<const uint4 *>(wg + row * (size_t)(H >> 4));
    const uint4 *uw = reinterpret_cast<const uint4 *>(wu + row * (size_t)(H >> 4));
    uint4 ag[kGuMaxSteps], au[kGuMaxSteps];
#pragma unroll
    for (int i = 0; i < kGuMaxSteps; ++i) {
        const int G = 4 * (s0 + i) + t;
        const bool ok = rok && (s0 + i < s1) && (G < ngroups);
        ag[i] = ok ? ldg_stream16(gw + G) : make_uint4(0, 0, 0, 0);
        au[i] = ok ? ldg_stream16(uw + G) : make_uint4(0, 0, 0, 0);
    }
    // scales / biases of the two groups this lane finalises per step (lanes t < 2)
    float sgv[kGuMaxSteps][2], bgv[kGuMaxSteps][2], suv[kGuMaxSteps][2], buv[kGuMaxSteps][2];
#pragma unroll
    for (int i = 0; i < kGuMaxSteps; ++i)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int G = 4 * (s0 + i) + 2 * t + c;
            const bool ok = rok && t < 2 && (s0 + i < s1) && (G < ngroups);
            const size_t si = row * ngroups + G;
            sgv[i][c] = ok ? SB<kFp16>::get(sg, si) : 0.f;
            bgv[i][c] = ok ? SB<kFp16>::get(bg, si) : 0.f;
            suv[i][c] = ok ? SB<kFp16>::get(su, si) : 0.f;
            buv[i][c] = ok ? SB<kFp16>::get(bu, si) : 0.f;
        }

    // 2) stage the token's input as MMA B records while the weights are in flight
    stage_bfrag(x + (size_t)tok * H, H, ngroups, xfrag, corr, xsum);
    __syncthreads();

    float accg = 0.f, accu = 0.f;
    const bool bl = (g == t);   // lanes holding B column n == t
#pragma unroll
    for (int i = 0; i < kGuMaxSteps; ++i) {
        if (s0 + i >= s1) break;
        const int Gb = 4 * (s0 + i);
        const bool bok = bl && (Gb + t < ngroups);
        const uint2 *xf = xfrag + (size_t)(Gb + t) * 16;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t gwd[4] = {ag[i].x, ag[i].y, ag[i].z, ag[i].w};
        const uint32_t uwd[4] = {au[i].x, au[i].y, au[i].z, au[i].w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            uint32_t gp[8], up[8];
            expand_word(gwd[m], gp);
            expand_word(uwd[m], up);
#pragma unroll
            for (int mi = 0; mi < 4; ++mi) {
                const uint2 b = bok ? xf[m * 4 + mi] : make_uint2(0u, 0u);
                mma_bf16_16816(d, gp[2 * mi], up[2 * mi], gp[2 * mi + 1], up[2 * mi + 1], b.x, b.y);
            }
        }
        if (t < 2) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int G = Gb + 2 * t + c;
                if (G < ngroups) {
                    accg += sgv[i][c] * (d[c] - corr[G]) + bgv[i][c] * xsum[G];
                    accu += suv[i][c] * (d[2 + c] - corr[G]) + buv[i][c] * xsum[G];
                }
            }
        }
    }
    accg += __shfl_xor_sync(0xffffffffu, accg, 1);
    accu += __shfl_xor_sync(0xffffffffu, accu, 1);
    if (t == 0) {
        red[(warp * 8 + g) * 2 + 0] = accg;
        red[(warp * 8 + g) * 2 + 1] = accu;
    }
    __syncthreads();
    if (warp == 0 && lane < 8) {
        const int rr = blockIdx.x * 8 + lane;
        if (rr < I) {
            float sgsum = 0.f, susum = 0.f;
#pragma unroll
            for (int w = 0; w < kGuWarps; ++w) {
                sgsum += red[(w * 8 + lane) * 2 + 0];
                susum += red[(w * 8 + lane) * 2 + 1];
            }
            const float gv = bf16r(sgsum), uv = bf16r(susum);
            // SwiGLU rounded after every op, like an MLX bf16 graph
            const float sig = bf16r(1.0f / (1.0f + expf(-gv)));
            const float a = sok ? bf16r(bf16r(gv * sig) * uv) : 0.f;
            act[((size_t)tok * K + k) * I + rr] = f32_to_bf16_bits(a);
        }
    }
}

// --------------------------------------------------------------------- down + combine

template <bool kFp16, int kSteps>
__global__ void __launch_bounds__(kMaxK * 32) down_kernel(
    const uint16_t *__restrict__ act, const uint32_t *__restrict__ slots,
    const uint16_t *__restrict__ scores, const uint32_t *__restrict__ wd,
    const uint16_t *__restrict__ sd, const uint16_t *__restrict__ bd, int H, int I, int K, int cap,
    const uint16_t *__restrict__ addend, const uint16_t *__restrict__ resid,
    uint16_t *__restrict__ y, uint16_t *__restrict__ yk) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int ngroups = I >> 6;
    uint2 *afrag = reinterpret_cast<uint2 *>(smem);                                 // [K][ngroups][16]
    float *corr = reinterpret_cast<float *>(smem + (size_t)K * ngroups * 128);      // [K][ngroups]
    float *xsum = corr + K * ngroups;                                               // [K][ngroups]
    float *yks = xsum + K * ngroups;                                                // [K][16]

    const int lane = threadIdx.x & 31, k = threadIdx.x >> 5;   // warp k <-> routed expert k
    const int g = lane >> 2, t = lane & 3;
    const int tok = blockIdx.y;
    const int r0 = blockIdx.x * 16;
    const uint32_t slot_raw = slots[(size_t)tok * K + k];
    const bool sok = slot_raw < (uint32_t)cap;          // out-of-range slot: rows read as absent
    const int ra = sok ? r0 + g : H, rb = sok ? r0 + 8 + g : H;
    const size_t slot = sok ? slot_raw : 0;
    const int nsteps = (ngroups + 3) >> 2;

    const size_t rowa = slot * H + ra, rowb = slot * H + rb;
    const uint4 *wa = reinterpret_cast<const uint4 *>(wd + rowa * (size_t)(I >> 4));
    const uint4 *wb = reinterpret_cast<const uint4 *>(wd + rowb * (size_t)(I >> 4));
    uint4 qa[kSteps], qb[kSteps];
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
        const int G = 4 * i + t;
        const bool ok = (i < nsteps) && (G < ngroups);
        qa[i] = (ok && ra < H) ? ldg_stream16(wa + G) : make_uint4(0, 0, 0, 0);
        qb[i] = (ok && rb < H) ? ldg_stream16(wb + G) : make_uint4(0, 0, 0, 0);
    }
    // scale / bias of the two groups this lane finalises per step (lanes t < 2)
    float sa[kSteps][2], ba[kSteps][2], sbv[kSteps][2], bbv[kSteps][2];
#pragma unroll
    for (int i = 0; i < kSteps; ++i)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int G = 4 * i + 2 * t + c;
            const bool ok = t < 2 && (i < nsteps) && (G < ngroups);
            sa[i][c] = (ok && ra < H) ? SB<kFp16>::get(sd, rowa * ngroups + G) : 0.f;
            ba[i][c] = (ok && ra < H) ? SB<kFp16>::get(bd, rowa * ngroups + G) : 0.f;
            sbv[i][c] = (ok && rb < H) ? SB<kFp16>::get(sd, rowb * ngroups + G) : 0.f;
            bbv[i][c] = (ok && rb < H) ? SB<kFp16>::get(bd, rowb * ngroups + G) : 0.f;
        }

    // stage every routed expert's activation vector (one warp-segment group at a time)
    for (int kk = 0; kk < K; ++kk)
        stage_bfrag(act + ((size_t)tok * K + kk) * I, I, ngroups, afrag + (size_t)kk * ngroups * 16,
                    corr + kk * ngroups, xsum + kk * ngroups);
    __syncthreads();

    const uint2 *xf0 = afrag + (size_t)k * ngroups * 16;
    const float *ck = corr + k * ngroups, *xk = xsum + k * ngroups;
    const bool bl = (g == t);
    float acca = 0.f, accb = 0.f;
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
        if (i >= nsteps) break;
        const int Gb = 4 * i;
        const bool bok = bl && (Gb + t < ngroups);
        const uint2 *xf = xf0 + (size_t)(Gb + t) * 16;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t awd[4] = {qa[i].x, qa[i].y, qa[i].z, qa[i].w};
        const uint32_t bwd[4] = {qb[i].x, qb[i].y, qb[i].z, qb[i].w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            uint32_t pa[8], pb[8];
            expand_word(awd[m], pa);
            expand_word(bwd[m], pb);
#pragma unroll
            for (int mi = 0; mi < 4; ++mi) {
                const uint2 b = bok ? xf[m * 4 + mi] : make_uint2(0u, 0u);
                mma_bf16_16816(d, pa[2 * mi], pb[2 * mi], pa[2 * mi + 1], pb[2 * mi + 1], b.x, b.y);
            }
        }
        if (t < 2) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int G = Gb + 2 * t + c;
                if (G < ngroups) {
                    acca += sa[i][c] * (d[c] - ck[G]) + ba[i][c] * xk[G];
                    accb += sbv[i][c] * (d[2 + c] - ck[G]) + bbv[i][c] * xk[G];
                }
            }
        }
    }
    acca += __shfl_xor_sync(0xffffffffu, acca, 1);
    accb += __shfl_xor_sync(0xffffffffu, accb, 1);
    if (t == 0) {
        const float ya = bf16r(acca), yb = bf16r(accb);
        yks[k * 16 + g] = ya;
        yks[k * 16 + 8 + g] = yb;
        if (yk) {
            const int oa = r0 + g, ob = r0 + 8 + g;
            if (oa < H) yk[((size_t)tok * K + k) * H + oa] = f32_to_bf16_bits(ya);
            if (ob < H) yk[((size_t)tok * K + k) * H + ob] = f32_to_bf16_bits(yb);
        }
    }
    __syncthreads();
    if (y && scores && threadIdx.x < 16) {
        const int rr = r0 + threadIdx.x;
        if (rr < H) {
            float acc = 0.f;
            for (int kk = 0; kk < K; ++kk) {
                const float sc = bf16_bits_to_f32(__ldg(scores + (size_t)tok * K + kk));
                const float pk = bf16r(yks[kk * 16 + threadIdx.x] * sc);
                acc = (kk == 0) ? pk : bf16r(acc + pk);
            }
            if (addend) acc = bf16r(acc + bf16_bits_to_f32(addend[(size_t)tok * H + rr]));
            if (resid) acc = bf16r(bf16_bits_to_f32(resid[(size_t)tok * H + rr]) + acc);
            y[(size_t)tok * H + rr] = f32_to_bf16_bits(acc);
        }
    }
}

int check_common(int H, int I, int K, int T, int bits, int group_size, const void *p0,
                 const void *p1, const char *who) {
    if (bits != 2 || group_size != 64)
        return moe_set_error(MOE_EINVAL, "%s: only bits=2, group_size=64 are implemented (got %d, %d)", who,
                             bits, group_size);
    if (T <= 0 || K <= 0 || K > kMaxK || H <= 0 || I <= 0 || H % 64 || I % 64)
        return moe_set_error(MOE_EINVAL, "%s: bad sizes T=%d H=%d I=%d K=%d", who, T, H, I, K);
    if ((reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1)) & 15)
        return moe_set_error(MOE_EINVAL, "%s: weight codes must be 16-byte aligned", who);
    return MOE_OK;
}

}  // namespace

extern "C" int moe_experts_gateup(const void *x, int T, int H, int I, int K, int cap, const uint32_t *slots,
                                  const uint32_t *wg, const void *sg, const void *bg,
                                  const uint32_t *wu, const void *su, const void *bu, int bits,
                                  int group_size, int sb_fp16, void *act, void *stream) {
    int rc = check_common(H, I, K, T, bits, group_size, wg, wu, "experts_gateup");
    if (rc) return rc;
    if (!x || !slots || !sg || !bg || !su || !bu || !act)
        return moe_set_error(MOE_EINVAL, "experts_gateup: null pointer");
    if (cap <= 0) return moe_set_error(MOE_EINVAL, "experts_gateup: cap=%d", cap);
    const int ngroups = H / 64, nsteps = (ngroups + 3) / 4;
    if ((nsteps + kGuWarps - 1) / kGuWarps > kGuMaxSteps)
        return moe_set_error(MOE_EINVAL, "experts_gateup: H=%d exceeds %d", H, kGuWarps * kGuMaxSteps * 256);
    const size_t smem = (size_t)ngroups * 128 + (size_t)ngroups * 8 + kGuWarps * 8 * 2 * sizeof(float);
    dim3 grid((I + 7) / 8, K, T);
    auto st = as_stream(stream);
    const auto *xs = static_cast<const uint16_t *>(x);
    if (sb_fp16)
        gateup_kernel<true><<<grid, kGuWarps * 32, smem, st>>>(
            xs, slots, wg, static_cast<const uint16_t *>(sg), static_cast<const uint16_t *>(bg), wu,
            static_cast<const uint16_t *>(su), static_cast<const uint16_t *>(bu), H, I, K, cap, static_cast<uint16_t *>(act));
    else
        gateup_kernel<false><<<grid, kGuWarps * 32, smem, st>>>(
            xs, slots, wg, static_cast<const uint16_t *>(sg), static_cast<const uint16_t *>(bg), wu,
            static_cast<const uint16_t *>(su), static_cast<const uint16_t *>(bu), H, I, K, cap, static_cast<uint16_t *>(act));
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" int moe_experts_down(const void *act, int T, int H, int I, int K, int cap, const uint32_t *slots,
                                const void *scores, const uint32_t *wd, const void *sd,
                                const void *bd, int bits, int group_size, int sb_fp16,
                                const void *addend, const void *resid, void *y, void *yk,
                                void *stream) {
    int rc = check_common(H, I, K, T, bits, group_size, wd, wd, "experts_down");
    if (rc) return rc;
    if (!act || !slots || !sd || !bd) return moe_set_error(MOE_EINVAL, "experts_down: null pointer");
    if (cap <= 0) return moe_set_error(MOE_EINVAL, "experts_down: cap=%d", cap);
    if (y && !scores) return moe_set_error(MOE_EINVAL, "experts_down: y needs scores");
    if (!y && !yk) return moe_set_error(MOE_EINVAL, "experts_down: no output requested");
    const int ngroups = I / 64;
    if ((ngroups + 3) / 4 > kDnMaxSteps)
        return moe_set_error(MOE_EINVAL, "experts_down: I=%d exceeds %d", I, kDnMaxSteps * 256);
    const size_t smem = (size_t)K * ngroups * 128 + (size_t)K * ngroups * 8 + (size_t)K * 16 * sizeof(float);
    if (smem > 227 * 1024) return moe_set_error(MOE_EINVAL, "experts_down: K*I too large");
    dim3 grid((H + 15) / 16, T);
    auto st = as_stream(stream);
    const int nsteps = (ngroups + 3) / 4;
    const auto *as = static_cast<const uint16_t *>(act);
    const auto *sc = static_cast<const uint16_t *>(scores);
    const auto *sdp = static_cast<const uint16_t *>(sd);
    const auto *bdp = static_cast<const uint16_t *>(bd);
    const auto *adp = static_cast<const uint16_t *>(addend);
    const auto *rsp = static_cast<const uint16_t *>(resid);
    auto *yp = static_cast<uint16_t *>(y);
    auto *ykp = static_cast<uint16_t *>(yk);
    auto go = [&](auto kern) -> int {
        if (smem > 48 * 1024)
            MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        kern<<<grid, K * 32, smem, st>>>(as, slots, sc, wd, sdp, bdp, H, I, K, cap, adp, rsp, yp, ykp);
        return MOE_OK;
    };
    if (sb_fp16) rc = (nsteps <= 4) ? go(down_kernel<true, 4>) : go(down_kernel<true, 8>);
    else rc = (nsteps <= 4) ? go(down_kernel<false, 4>) : go(down_kernel<false, 8>);
    if (rc) return rc;
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}
