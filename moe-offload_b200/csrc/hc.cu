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
// Launches (programmatic dependent launch, each kernel loading its weights before it waits on
// the previous one): norm (one block per row and stream) -> down and inject rows in one launch
// (float totals) -> up rows of the four streams of each hidden index, the silu of the down
// totals formed while staging them and the stream sum and inject sigmoid in the epilogue.
#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

#include "common.cuh"
#include "qlinear.cuh"
#include "hcmath.cuh"
#include "../../include/moe_b200.h"

namespace {

using namespace moe_qlin;

constexpr int kHc = 4;                           // streams (hc_count of the reference's models)
constexpr int kNormThreads = 1024;                  // few values per thread: the norm has only HC x T blocks
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
    pdl_launch_dependents();
    pdl_wait();                                  // h, branch and gate come from earlier kernels
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

// mixed[t][h] = mean_c sigmoid(u[t][c*H + h]) * normed[t][c*H + h], u = mix . Wu^T: a block
// takes `rows` hidden indices h with the four up rows c*H + h each, items (h, c, group) one per
// thread; the mix rows (silu of the down totals dv) are formed while staging them; block 0 also
// writes inj from the inject totals iv
template <int kBits, int kGs, bool kFp16>
__global__ void __launch_bounds__(max_block(kGs)) hc_up_tail_kernel(const float *__restrict__ dv,
                                                                    const float *__restrict__ iv, int T, int R, int H,
                                                                    const uint32_t *__restrict__ wu,
                                                                    const uint16_t *__restrict__ su,
                                                                    const uint16_t *__restrict__ bu,
                                                                    const uint16_t *__restrict__ normed, int prefill,
                                                                    uint16_t *__restrict__ mixed,
                                                                    uint16_t *__restrict__ inj) {
    extern __shared__ __align__(16) unsigned char lin_smem_raw[];
    using GI = GroupItem<kBits, kGs, kFp16>;
    const int ng = R / kGs, W = kHc * H;
    const FlatShape F = flat_shape(kHc, ng, T, R);
    double *sv = reinterpret_cast<double *>(lin_smem_raw);              // [rows][kHc][kLinTok][ng]
    uint16_t *sx = reinterpret_cast<uint16_t *>(lin_smem_raw + F.grp);
    const int c = (threadIdx.x / ng) % kHc, r = threadIdx.x / (kHc * ng), g = threadIdx.x % ng;
    const int hi = blockIdx.x * F.rows + r;
    const bool item = r < F.rows && hi < H;
    GI it;
    if (item) {
        const size_t row = (size_t)c * H + hi;
        it.load(wu + row * (R / GI::kPer), su + row * ng, bu + row * ng, g);
    }
    pdl_launch_dependents();
    pdl_wait();                                  // dv, iv and normed come from earlier kernels
    if (blockIdx.x == 0 && inj)
        for (int q = threadIdx.x; q < T * kHc; q += blockDim.x)
            inj[q] = f32_to_bf16_bits(iv ? hc_inj_value(iv[q], prefill) : 0.f);
#pragma unroll 1
    for (int t0 = 0; t0 < T; t0 += kLinTok) {
        const int nt = min(kLinTok, T - t0);
        __syncthreads();                         // the previous pass is done with sx and sv
        for (int k = threadIdx.x; k < nt * R; k += blockDim.x)   // mix rows t0 .. t0+nt-1
            sx[k] = f32_to_bf16_bits(hc_mix_value(dv[(size_t)t0 * R + k], prefill));
        __syncthreads();
        if (item)
            for (int j = 0; j < nt; ++j)
                sv[((r * kHc + c) * kLinTok + j) * ng + g] = it.value(sx + (size_t)j * R + (size_t)g * kGs);
        __syncthreads();
        for (int q = threadIdx.x; q < F.rows * nt; q += blockDim.x) {
            const int rr = q / nt, j = q - rr * nt, hh = blockIdx.x * F.rows + rr;
            if (hh >= H) continue;
            const size_t t = (size_t)(t0 + j);
            float acc = 0.f;
#pragma unroll
            for (int cc = 0; cc < kHc; ++cc) {
                float u = (float)sum_in_order(sv + ((rr * kHc + cc) * kLinTok + j) * ng, ng);
                const float nv = bf16_bits_to_f32(ldu16(normed + t * W + (size_t)cc * H + hh));
                if (prefill) {
                    u = bf16r(u);
                    const float p = bf16r(__fmul_rn(sigmoid_bf16(u), nv));
                    acc = cc == 0 ? p : bf16r(__fadd_rn(acc, p));
                } else {
                    const float p = __fmul_rn(sigmoidf(u), nv);
                    acc = cc == 0 ? p : __fadd_rn(acc, p);
                }
            }
            mixed[t * H + hh] = f32_to_bf16_bits(prefill ? __fmul_rn(acc, 1.0f / (float)kHc) : __fdiv_rn(acc, (float)kHc));
        }
    }
}

struct UpTailArgs {
    const float *dv, *iv;
    int T, R, H;
    const void *wu, *su, *bu, *normed;
    int prefill;
    void *mixed, *inj;
};

template <int kBits, int kGs, bool kFp16>
int launch_up_tail(const UpTailArgs &a, cudaStream_t st) {
    const FlatShape F = flat_shape(kHc, a.R / kGs, a.T, a.R);   // the mix rows always fit: R <= kMaxHcRank
    MOE_CUDA_TRY(launch_pdl_v(hc_up_tail_kernel<kBits, kGs, kFp16>, dim3((a.H + F.rows - 1) / F.rows),
                              dim3(F.threads), F.smem(), st, a.dv, a.iv, a.T, a.R, a.H,
                              static_cast<const uint32_t *>(a.wu), static_cast<const uint16_t *>(a.su),
                              static_cast<const uint16_t *>(a.bu), static_cast<const uint16_t *>(a.normed), a.prefill,
                              static_cast<uint16_t *>(a.mixed), static_cast<uint16_t *>(a.inj)));
    return MOE_OK;
}

int dispatch_up_tail(int bits, int gs, int sb_fp16, const UpTailArgs &a, cudaStream_t st) {
#define MOE_HC_CASE(B, G)                                                                          \
    if (bits == B && gs == G)                                                                      \
        return sb_fp16 ? launch_up_tail<B, G, true>(a, st) : launch_up_tail<B, G, false>(a, st);
    MOE_HC_CASE(2, 32) MOE_HC_CASE(2, 64) MOE_HC_CASE(2, 128)
    MOE_HC_CASE(4, 32) MOE_HC_CASE(4, 64) MOE_HC_CASE(4, 128)
    MOE_HC_CASE(8, 32) MOE_HC_CASE(8, 64) MOE_HC_CASE(8, 128)
#undef MOE_HC_CASE
    return moe_set_error(MOE_EINVAL, "hc_mix: no up kernel for bits=%d group_size=%d", bits, gs);
}

constexpr int kMaxHcRank = 8192;                 // the up pass stages kLinTok rows of R mix values

struct HcWs {
    size_t normed, dv, iv, total;
};

HcWs hc_ws(int T, int HC, int H, int R) {
    HcWs w;
    w.normed = 0;
    w.dv = al256((size_t)T * HC * H * 2);
    w.iv = w.dv + al256((size_t)T * R * 4);
    w.total = w.iv + al256((size_t)T * HC * 4);
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
    const int W = HC * H;
    if (R > kMaxHcRank) return moe_set_error(MOE_EINVAL, "hc_mix: rank %d above %d", R, kMaxHcRank);
    int rc = moe_qlin_check("hc_mix down", normed, T, W, R, wd, sd, bd, dbits, dgs, mixed);
    if (!rc) rc = moe_qlin_check("hc_mix up", normed, T, R, W, wu, su, bu, ubits, ugs, mixed);
    if (!rc && wi) rc = moe_qlin_check("hc_mix inject", normed, T, W, HC, wi, si, bi, ibits, igs, mixed);
    if (rc) return rc;
    if (kHc * (R / ugs) > max_block(ugs))
        return moe_set_error(MOE_EINVAL, "hc_mix: %d up groups per row (at most %d)", R / ugs, max_block(ugs) / kHc);
    if (reinterpret_cast<uintptr_t>(h) % 2 || (written && reinterpret_cast<uintptr_t>(written) % 2))
        return moe_set_error(MOE_EINVAL, "hc_mix: misaligned bf16 buffers");
    cudaStream_t st = as_stream(stream);
    const int prefill = T > kPrefillRows;
    MOE_CUDA_TRY(launch_pdl_v(hc_norm_kernel, dim3(HC, T), dim3(kNormThreads), (size_t)H * sizeof(float), st,
                              static_cast<const uint16_t *>(h), static_cast<const uint16_t *>(branch),
                              static_cast<const uint16_t *>(gate), static_cast<const uint16_t *>(norm_w), eps, H,
                              static_cast<uint16_t *>(written), normed));
    if (wi && ibits == dbits && igs == dgs) {    // down and inject rows in one launch
        rc = moe_qlin_linear(normed, T, W, R, wd, sd, bd, dbits, dgs, sb_fp16, nullptr, nullptr, dv, st, wi, si, bi,
                             HC, iv);
    } else {
        rc = moe_qlin_linear(normed, T, W, R, wd, sd, bd, dbits, dgs, sb_fp16, nullptr, nullptr, dv, st);
        if (!rc && wi) rc = moe_qlin_linear(normed, T, W, HC, wi, si, bi, ibits, igs, sb_fp16, nullptr, nullptr, iv, st);
    }
    if (rc) return rc;
    const UpTailArgs a{dv, wi ? iv : nullptr, T, R, H, wu, su, bu, normed, prefill, mixed, inj};
    return dispatch_up_tail(ubits, ugs, sb_fp16, a, st);
}
