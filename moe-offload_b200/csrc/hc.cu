// The hyper-connection mixer in front of each MoE block (Qwen38Engine::run_hc,
// mlx-qwen38/cpp/src/kernels.cpp:1363-1560) for affine-quantised mixer matrices:
//   written = h (+ bf16(branch[t] * gate[t][c]) added to stream c)        (the write)
//   normed  = per-stream RMS norm of written, times (1 + norm_w)
//   mix     = silu(down(normed) / HC)                                    [T, R]
//   mixed   = mean over streams c of sigmoid(up(mix))[c] * normed[c]     [T, H], the block input
//   inj     = 2 * sigmoid(inject(normed) / HC)                           [T, HC]
// with the reference's two rounding regimes: T <= 16 (its fused decode kernels) keeps the
// down / up / inject dot products unrounded and rounds mix, mixed and inj once; T > 16 (its
// prefill path and tail/inject kernel, kernels.cpp:788-846) rounds the dot products to bf16 and
// rounds after every op of silu and of the stream sum. Dot products follow the quantised-linear
// arithmetic of qlinear.cuh; the RMS statistic is a double sum of squares with
// rs = float(1 / sqrt(ss / H + eps)).
//
// Launches: norm (one block per row and stream) -> down and inject rows (float totals) ->
// activation (silu, inject sigmoid) -> up rows of the four streams of one hidden index in one
// warp, with the stream sum in its epilogue.
#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

#include "common.cuh"
#include "qlinear.cuh"
#include "../../include/moe_b200.h"

namespace {

using namespace moe_qlin;

constexpr int kHc = 4;                           // streams (hc_count of the reference's models)
constexpr int kNormThreads = 256;
constexpr int kPrefillRows = 16;                 // run_hc: rows <= 16 take the fused decode kernels

MOE_D uint16_t ldu16(const uint16_t *p) { return __ldg(p); }

// one block per (stream c, row t): written and normed for H values
__global__ void __launch_bounds__(kNormThreads) hc_norm_kernel(const uint16_t *__restrict__ h,
                                                               const uint16_t *__restrict__ branch,
                                                               const uint16_t *__restrict__ gate,
                                                               const uint16_t *__restrict__ norm_w, float eps, int H,
                                                               uint16_t *__restrict__ written,
                                                               uint16_t *__restrict__ normed) {
    extern __shared__ float sxv[];               // [H] the written values
    __shared__ double spart[kNormThreads / 32];
    __shared__ float srs;
    const int c = blockIdx.x, t = blockIdx.y, W = kHc * H;
    const size_t base = (size_t)t * W + (size_t)c * H;
    const float gv = branch ? bf16_bits_to_f32(ldu16(gate + (size_t)t * kHc + c)) : 0.f;
    double ss = 0.0;
    for (int i = threadIdx.x; i < H; i += kNormThreads) {
        float v = bf16_bits_to_f32(ldu16(h + base + i));
        if (branch) {
            const float p = bf16r(__fmul_rn(bf16_bits_to_f32(ldu16(branch + (size_t)t * H + i)), gv));
            v = bf16r(__fadd_rn(v, p));
            written[base + i] = f32_to_bf16_bits(v);
        }
        sxv[i] = v;
        ss += (double)v * (double)v;             // exact square; double sum
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) spart[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < kNormThreads / 32; ++w) tot += spart[w];
        srs = (float)(1.0 / sqrt(tot / H + (double)eps));
    }
    __syncthreads();
    const float rs = srs;
    for (int i = threadIdx.x; i < H; i += kNormThreads) {
        const float y = __fmul_rn(sxv[i], rs);
        const float sc = __fadd_rn(1.0f, bf16_bits_to_f32(ldu16(norm_w + (size_t)c * H + i)));
        normed[base + i] = f32_to_bf16_bits(__fmul_rn(y, sc));
    }
}

// mix = silu(d / HC) [T, R] and inj = 2 * sigmoid(iv / HC) [T, HC] in the row count's regime
__global__ void hc_act_kernel(const float *__restrict__ dv, const float *__restrict__ iv, int T, int R, int prefill,
                              uint16_t *__restrict__ mix, uint16_t *__restrict__ inj) {
    const int n = T * R, ni = T * kHc;
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < n + ni; k += gridDim.x * blockDim.x) {
        if (k < n) {
            const float d = dv[k];
            float o;
            if (prefill) {
                const float v = bf16r(__fdiv_rn(bf16r(d), (float)kHc));
                o = __fmul_rn(v, sigmoid_bf16(v));
            } else {
                const float v = __fdiv_rn(d, (float)kHc);
                o = __fmul_rn(v, sigmoidf(v));
            }
            mix[k] = f32_to_bf16_bits(o);
        } else if (inj) {
            const int q = k - n;
            float o = 0.f;
            if (iv) {
                if (prefill) o = __fmul_rn(2.0f, sigmoid_bf16(bf16r(__fdiv_rn(bf16r(iv[q]), (float)kHc))));
                else o = __fmul_rn(2.0f, sigmoidf(__fdiv_rn(iv[q], (float)kHc)));
            }
            inj[q] = f32_to_bf16_bits(o);
        }
    }
}

// mixed[t][h] = mean_c sigmoid(u[t][c*H + h]) * normed[t][c*H + h], u = mix . Wu^T; one warp
// per hidden index h takes the four up rows c*H + h
template <int kBits, int kGs, bool kFp16>
__global__ void __launch_bounds__(kLinThreads) hc_up_tail_kernel(const uint16_t *__restrict__ mix, int T, int R,
                                                                 int H, const uint32_t *__restrict__ wu,
                                                                 const uint16_t *__restrict__ su,
                                                                 const uint16_t *__restrict__ bu,
                                                                 const uint16_t *__restrict__ normed, int prefill,
                                                                 uint16_t *__restrict__ mixed, int stage) {
    extern __shared__ __align__(16) unsigned char lin_smem_raw[];
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hi = blockIdx.x * kLinWarps + wib;
    const bool active = hi < H;
    const int ng = R / kGs, W = kHc * H;
    const LinSmem L = lin_smem(kHc, ng, T, R);
    double *sv = reinterpret_cast<double *>(lin_smem_raw) + (size_t)wib * kHc * kLinTok * ng;
    uint16_t *sx = reinterpret_cast<uint16_t *>(lin_smem_raw + L.grp);
    constexpr int per = Group<kBits, kGs>::kPer;
    const int hr = active ? hi : 0;
    const uint32_t *wr[kHc];
    const uint16_t *sr[kHc], *br[kHc];
#pragma unroll
    for (int c = 0; c < kHc; ++c) {
        const size_t row = (size_t)c * H + hr;
        wr[c] = wu + row * (R / per);
        sr[c] = su + row * ng;
        br[c] = bu + row * ng;
    }
    const uint32_t *const(&wrc)[kHc] = wr;
    const uint16_t *const(&src)[kHc] = sr;
    const uint16_t *const(&brc)[kHc] = br;
#pragma unroll 1
    for (int t0 = 0; t0 < T; t0 += kLinTok) {
        const int nt = min(kLinTok, T - t0);
        const uint16_t *xs = mix + (size_t)t0 * R;
        if (stage) {
            __syncthreads();
            stage_x(sx, mix, R, t0, nt);
            __syncthreads();
            xs = sx;
        }
        if (active) {
            stage_rows_spread<kBits, kGs, kFp16, kHc>(xs, R, nt, wrc, src, brc, ng, lane, sv);
            __syncwarp();
            const int j = lane & (kLinTok - 1), m = lane / kLinTok;     // lane = m * kLinTok + j
            float u = 0.f;
            if (m < kHc && j < nt) {
                u = (float)sum_in_order(sv + (m * kLinTok + j) * ng, ng);
                if (prefill) u = bf16r(u);
            }
            float uc[kHc];
#pragma unroll
            for (int c = 0; c < kHc; ++c) uc[c] = __shfl_sync(0xffffffffu, u, c * kLinTok + j);
            if (lane < nt) {
                const size_t t = (size_t)(t0 + lane);
                float acc = 0.f;
#pragma unroll
                for (int c = 0; c < kHc; ++c) {
                    const float nv = bf16_bits_to_f32(ldu16(normed + t * W + (size_t)c * H + hi));
                    if (prefill) {
                        const float p = bf16r(__fmul_rn(sigmoid_bf16(uc[c]), nv));
                        acc = c == 0 ? p : bf16r(__fadd_rn(acc, p));
                    } else {
                        const float p = __fmul_rn(sigmoidf(uc[c]), nv);
                        acc = c == 0 ? p : __fadd_rn(acc, p);
                    }
                }
                mixed[t * H + hi] =
                    f32_to_bf16_bits(prefill ? __fmul_rn(acc, 1.0f / (float)kHc) : __fdiv_rn(acc, (float)kHc));
            }
            __syncwarp();
        }
    }
}

template <typename K>
int prepare_smem(K kern, size_t bytes) {
    if (bytes > 48 * 1024)
        MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return MOE_OK;
}

template <int kBits, int kGs, bool kFp16>
int launch_up_tail(const void *mix, int T, int R, int H, const void *wu, const void *su, const void *bu,
                   const void *normed, int prefill, void *mixed, cudaStream_t st) {
    auto kern = hc_up_tail_kernel<kBits, kGs, kFp16>;
    const LinSmem L = lin_smem(kHc, R / kGs, T, R);
    int rc = prepare_smem(kern, L.total());
    if (rc) return rc;
    kern<<<(H + kLinWarps - 1) / kLinWarps, kLinThreads, L.total(), st>>>(
        static_cast<const uint16_t *>(mix), T, R, H, static_cast<const uint32_t *>(wu),
        static_cast<const uint16_t *>(su), static_cast<const uint16_t *>(bu), static_cast<const uint16_t *>(normed),
        prefill, static_cast<uint16_t *>(mixed), L.xbytes > 0);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

int dispatch_up_tail(int bits, int gs, int sb_fp16, const void *mix, int T, int R, int H, const void *wu,
                     const void *su, const void *bu, const void *normed, int prefill, void *mixed, cudaStream_t st) {
#define MOE_HC_CASE(B, G)                                                                                    \
    if (bits == B && gs == G)                                                                                \
        return sb_fp16 ? launch_up_tail<B, G, true>(mix, T, R, H, wu, su, bu, normed, prefill, mixed, st)   \
                       : launch_up_tail<B, G, false>(mix, T, R, H, wu, su, bu, normed, prefill, mixed, st);
    MOE_HC_CASE(2, 32) MOE_HC_CASE(2, 64) MOE_HC_CASE(2, 128)
    MOE_HC_CASE(4, 32) MOE_HC_CASE(4, 64) MOE_HC_CASE(4, 128)
    MOE_HC_CASE(8, 32) MOE_HC_CASE(8, 64) MOE_HC_CASE(8, 128)
#undef MOE_HC_CASE
    return moe_set_error(MOE_EINVAL, "hc_mix: no up kernel for bits=%d group_size=%d", bits, gs);
}

struct HcWs {
    size_t normed, dv, iv, mix, total;
};

HcWs hc_ws(int T, int HC, int H, int R) {
    HcWs w;
    w.normed = 0;
    w.dv = al256((size_t)T * HC * H * 2);
    w.iv = w.dv + al256((size_t)T * R * 4);
    w.mix = w.iv + al256((size_t)T * HC * 4);
    w.total = w.mix + al256((size_t)T * R * 2);
    return w;
}

}  // namespace

extern "C" size_t moe_hc_workspace_bytes(int T, int HC, int H, int R) {
    if (T <= 0 || HC <= 0 || H <= 0 || R <= 0) return 0;
    return hc_ws(T, HC, H, R).total;
}

extern "C" int moe_hc_mix(const void *h, int T, int HC, int H, int R, const void *branch, const void *gate,
                          const void *norm_w, float eps, const void *wd, const void *sd, const void *bd, int dbits,
                          int dgs, const void *wu, const void *su, const void *bu, int ubits, int ugs, const void *wi,
                          const void *si, const void *bi, int ibits, int igs, int sb_fp16, void *written,
                          void *mixed, void *inj, void *workspace, size_t workspace_bytes, void *stream) {
    if (HC != kHc) return moe_set_error(MOE_EINVAL, "hc_mix: %d streams (the quantised path supports %d)", HC, kHc);
    if (!h || !norm_w || !mixed || !workspace) return moe_set_error(MOE_EINVAL, "hc_mix: null pointer");
    if (T <= 0 || H <= 0 || R <= 0 || H % 8) return moe_set_error(MOE_EINVAL, "hc_mix: bad sizes T=%d H=%d R=%d", T, H, R);
    if ((branch == nullptr) != (gate == nullptr) || (branch && !written))
        return moe_set_error(MOE_EINVAL, "hc_mix: a write needs branch, gate and written");
    if (!(eps >= 0.f)) return moe_set_error(MOE_EINVAL, "hc_mix: eps must be >= 0");
    const HcWs L = hc_ws(T, HC, H, R);
    if (workspace_bytes < L.total)
        return moe_set_error(MOE_EINVAL, "hc_mix: workspace of %zu bytes needed, %zu given", L.total, workspace_bytes);
    char *p = static_cast<char *>(workspace);
    uint16_t *normed = reinterpret_cast<uint16_t *>(p + L.normed);
    float *dv = reinterpret_cast<float *>(p + L.dv), *iv = reinterpret_cast<float *>(p + L.iv);
    uint16_t *mix = reinterpret_cast<uint16_t *>(p + L.mix);
    const int W = HC * H;
    int rc = moe_qlin_check("hc_mix down", normed, T, W, R, wd, sd, bd, dbits, dgs, mixed);
    if (!rc) rc = moe_qlin_check("hc_mix up", mix, T, R, W, wu, su, bu, ubits, ugs, mixed);
    if (!rc && wi) rc = moe_qlin_check("hc_mix inject", normed, T, W, HC, wi, si, bi, ibits, igs, mixed);
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(h) % 2 || (written && reinterpret_cast<uintptr_t>(written) % 2))
        return moe_set_error(MOE_EINVAL, "hc_mix: misaligned bf16 buffers");
    cudaStream_t st = as_stream(stream);
    const int prefill = T > kPrefillRows;
    if ((rc = prepare_smem(hc_norm_kernel, (size_t)H * sizeof(float)))) return rc;
    hc_norm_kernel<<<dim3(HC, T), kNormThreads, (size_t)H * sizeof(float), st>>>(
        static_cast<const uint16_t *>(h), static_cast<const uint16_t *>(branch), static_cast<const uint16_t *>(gate),
        static_cast<const uint16_t *>(norm_w), eps, H, static_cast<uint16_t *>(written), normed);
    MOE_CUDA_TRY(cudaGetLastError());
    if ((rc = moe_qlin_linear(normed, T, W, R, wd, sd, bd, dbits, dgs, sb_fp16, nullptr, nullptr, dv, st))) return rc;
    if (wi && (rc = moe_qlin_linear(normed, T, W, HC, wi, si, bi, ibits, igs, sb_fp16, nullptr, nullptr, iv, st)))
        return rc;
    const int nact = T * (R + HC);
    hc_act_kernel<<<(nact + 255) / 256, 256, 0, st>>>(dv, wi ? iv : nullptr, T, R, prefill, mix,
                                                      static_cast<uint16_t *>(inj));
    MOE_CUDA_TRY(cudaGetLastError());
    return dispatch_up_tail(ubits, ugs, sb_fp16, mix, T, R, H, wu, su, bu, normed, prefill, mixed, st);
}
