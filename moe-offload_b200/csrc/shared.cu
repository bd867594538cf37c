// Affine-quantised linear layers and the shared expert of the reference's MoE layer
// (mlx-qwen38/cpp/src/engine.cpp:394-400: shared_gate_proj / shared_up_proj, SwiGLU,
// shared_down_proj, sigmoid(shared_expert_gate(x)) * out; QLinear::forward
// cpp/src/kernels.cpp:997-1019). Weights in MLX's affine format: w = scale * q + bias per group
// of `group_size` inputs, `bits`-bit codes packed 32/bits per little-endian uint32, code j in
// bits [bits*j, bits*j + bits) of its word.
//
// Arithmetic (the routed-expert GEMVs' qmv form, scale * sum(q x) + bias * sum(x) per group):
// within a group, sum(q x) and sum(x) are float sums in input order (each q x is exact in
// float); the group's value scale * sum(q x) + bias * sum(x) is formed in double (both products
// exact); the row total is the double sum of the group values in group order, rounded to float
// and then to bf16. With that order fixed the output does not depend on the launch shape.
// SwiGLU and the gate product round to bf16 after every op.
//
// Kernels: one warp per output row, lane l on groups l, l + 32, ... (the words of the next
// group are loaded before the current one is used); group values are staged in shared memory
// and lane j adds token j's in group order. The shared expert is two launches: gate + up +
// SwiGLU (+ one extra warp for the scalar expert gate), then down with the sigmoid(gate) scale
// in its epilogue.
#include <algorithm>
#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

#include "common.cuh"
#include "qlinear.cuh"
#include "../../include/moe_b200.h"

namespace {

using namespace moe_qlin;

// y[t][n] = bf16(float(row total)) (gl == nullptr), or bf16(bf16(sigmoid(gl[t])) * that), or,
// with yf != nullptr, float(row total) to yf
template <int kBits, int kGs, bool kFp16>
__global__ void __launch_bounds__(kLinThreads) affine_linear_kernel(const uint16_t *__restrict__ x, int T, int Kin,
                                                                    int N, const uint32_t *__restrict__ w,
                                                                    const uint16_t *__restrict__ s,
                                                                    const uint16_t *__restrict__ b,
                                                                    const uint16_t *__restrict__ gl,
                                                                    uint16_t *__restrict__ y, float *__restrict__ yf,
                                                                    int stage) {
    extern __shared__ __align__(16) unsigned char lin_smem_raw[];
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * kLinWarps + wib;
    const bool active = n < N;                   // idle warps still take part in the x staging
    const int ng = Kin / kGs;
    const LinSmem L = lin_smem(1, ng, T, Kin);
    double *sv = reinterpret_cast<double *>(lin_smem_raw) + (size_t)wib * kLinTok * ng;
    uint16_t *sx = reinterpret_cast<uint16_t *>(lin_smem_raw + L.grp);
    const int nrow = active ? n : 0;
    const uint32_t *const wr[1] = {w + (size_t)nrow * (Kin / Group<kBits, kGs>::kPer)};
    const uint16_t *const sr[1] = {s + (size_t)nrow * ng};
    const uint16_t *const br[1] = {b + (size_t)nrow * ng};
#pragma unroll 1
    for (int t0 = 0; t0 < T; t0 += kLinTok) {
        const int nt = min(kLinTok, T - t0);
        const uint16_t *xs = x + (size_t)t0 * Kin;
        if (stage) {
            __syncthreads();                     // the previous pass is done with sx
            stage_x(sx, x, Kin, t0, nt);
            __syncthreads();
            xs = sx;
        }
        if (active) {
            stage_rows<kBits, kGs, kFp16, 1>(xs, Kin, nt, wr, sr, br, ng, lane, sv);
            __syncwarp();
            if (lane < nt) {
                const int t = t0 + lane;
                const double total = sum_in_order(sv + lane * ng, ng);
                if (yf) {
                    yf[(size_t)t * N + n] = (float)total;
                } else {
                    uint16_t o = row_out(total);
                    if (gl) o = f32_to_bf16_bits(__fmul_rn(sigmoid_bf16(bf16_bits_to_f32(gl[t])), bf16_bits_to_f32(o)));
                    y[(size_t)t * N + n] = o;
                }
            }
            __syncwarp();
        }
    }
}

// act[t][i] = bf16(bf16(g * bf16(sigmoid(g))) * u) with g, u rows i of the gate / up
// projections; the warp of row I computes gl[t] = x[t] . We (runtime bits / group size).
template <int kBits, int kGs, bool kFp16>
__global__ void __launch_bounds__(kLinThreads) gateup_swiglu_kernel(
    const uint16_t *__restrict__ x, int T, int H, int I, const uint32_t *__restrict__ wg,
    const uint16_t *__restrict__ sg, const uint16_t *__restrict__ bg, const uint32_t *__restrict__ wu,
    const uint16_t *__restrict__ su, const uint16_t *__restrict__ bu, const uint32_t *__restrict__ we,
    const uint16_t *__restrict__ se, const uint16_t *__restrict__ be, int ebits, int egs,
    uint16_t *__restrict__ act, uint16_t *__restrict__ gl, int stage) {
    extern __shared__ __align__(16) unsigned char lin_smem_raw[];
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * kLinWarps + wib;
    const int ng = H / kGs, nge = H / egs;
    const LinSmem L = lin_smem(2, max(ng, (nge + 1) / 2), T, H);
    double *sv = reinterpret_cast<double *>(lin_smem_raw) + (size_t)wib * 2 * kLinTok * max(ng, (nge + 1) / 2);
    uint16_t *sx = reinterpret_cast<uint16_t *>(lin_smem_raw + L.grp);
    constexpr int per = Group<kBits, kGs>::kPer;
    const int irow = i < I ? i : 0;
    const uint32_t *const wr[2] = {wg + (size_t)irow * (H / per), wu + (size_t)irow * (H / per)};
    const uint16_t *const sr[2] = {sg + (size_t)irow * ng, su + (size_t)irow * ng};
    const uint16_t *const br[2] = {bg + (size_t)irow * ng, bu + (size_t)irow * ng};
#pragma unroll 1
    for (int t0 = 0; t0 < T; t0 += kLinTok) {
        const int nt = min(kLinTok, T - t0);
        const uint16_t *xs = x + (size_t)t0 * H;
        if (stage) {
            __syncthreads();
            stage_x(sx, x, H, t0, nt);
            __syncthreads();
            xs = sx;
        }
        if (i == I) {                            // the scalar expert gate
            stage_row_generic<kFp16>(xs, H, nt, we, se, be, ebits, egs, lane, sv);
            __syncwarp();
            if (lane < nt) gl[t0 + lane] = row_out(sum_in_order(sv + lane * nge, nge));
            __syncwarp();
        } else if (i < I) {
            stage_rows<kBits, kGs, kFp16, 2>(xs, H, nt, wr, sr, br, ng, lane, sv);
            __syncwarp();
            // lanes 0..nt-1 add the gate rows, lanes kLinTok..kLinTok+nt-1 the up rows
            const int j = lane & (kLinTok - 1), m = lane / kLinTok;
            float v = 0.f;
            if (m < 2 && j < nt) v = bf16_bits_to_f32(row_out(sum_in_order(sv + (m * kLinTok + j) * ng, ng)));
            const float uv = __shfl_down_sync(0xffffffffu, v, kLinTok);
            if (lane < nt)
                act[(size_t)(t0 + lane) * I + i] =
                    f32_to_bf16_bits(bf16r(__fmul_rn(bf16r(__fmul_rn(v, sigmoid_bf16(v))), uv)));
            __syncwarp();
        }
    }
}

int check_lin(const char *who, const void *x, int T, int Kin, int N, const void *w, const void *s, const void *b,
              int bits, int gs, const void *y) {
    if (!x || !w || !s || !b || !y) return moe_set_error(MOE_EINVAL, "%s: null pointer", who);
    if (T <= 0 || Kin <= 0 || N <= 0)
        return moe_set_error(MOE_EINVAL, "%s: bad sizes T=%d K=%d N=%d", who, T, Kin, N);
    if (bits != 2 && bits != 4 && bits != 8)
        return moe_set_error(MOE_EINVAL, "%s: bits=%d (2, 4 or 8 supported)", who, bits);
    if (gs != 32 && gs != 64 && gs != 128)
        return moe_set_error(MOE_EINVAL, "%s: group_size=%d (32, 64 or 128 supported)", who, gs);
    if (Kin % gs) return moe_set_error(MOE_EINVAL, "%s: group_size %d does not divide K=%d", who, gs, Kin);
    if (Kin / gs > kMaxGroups)
        return moe_set_error(MOE_EINVAL, "%s: %d groups per row (at most %d)", who, Kin / gs, kMaxGroups);
    const uintptr_t wa = (gs * bits / 8) % 16 ? 8 : 16;      // the group's word loads
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % wa)
        return moe_set_error(MOE_EINVAL, "%s: x must be 16-byte and codes %d-byte aligned", who, (int)wa);
    return MOE_OK;
}

// the dynamic shared memory of one block; above the 48 KB default the kernel is opted in
template <typename K>
int prepare_smem(K kern, size_t bytes) {
    if (bytes > 48 * 1024)
        MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return MOE_OK;
}

template <int kBits, int kGs, bool kFp16>
int launch_lin_t(const void *x, int T, int Kin, int N, const void *w, const void *s, const void *b, const void *gl,
                 void *y, float *yf, cudaStream_t st) {
    auto kern = affine_linear_kernel<kBits, kGs, kFp16>;
    const LinSmem L = lin_smem(1, Kin / kGs, T, Kin);
    int rc = prepare_smem(kern, L.total());
    if (rc) return rc;
    kern<<<(N + kLinWarps - 1) / kLinWarps, kLinThreads, L.total(), st>>>(
        static_cast<const uint16_t *>(x), T, Kin, N, static_cast<const uint32_t *>(w),
        static_cast<const uint16_t *>(s), static_cast<const uint16_t *>(b), static_cast<const uint16_t *>(gl),
        static_cast<uint16_t *>(y), yf, L.xbytes > 0);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

struct GateUpArgs {
    const void *x;
    int T, H, I;
    const void *wg, *sg, *bg, *wu, *su, *bu, *we, *se, *be;
    int ebits, egs;
    void *act, *gl;
};

template <int kBits, int kGs, bool kFp16>
int launch_gateup_t(const GateUpArgs &a, cudaStream_t st) {
    auto kern = gateup_swiglu_kernel<kBits, kGs, kFp16>;
    const LinSmem L = lin_smem(2, std::max(a.H / kGs, (a.H / a.egs + 1) / 2), a.T, a.H);
    int rc = prepare_smem(kern, L.total());
    if (rc) return rc;
    auto u16 = [](const void *p) { return static_cast<const uint16_t *>(p); };
    auto u32 = [](const void *p) { return static_cast<const uint32_t *>(p); };
    kern<<<(a.I + 1 + kLinWarps - 1) / kLinWarps, kLinThreads, L.total(), st>>>(
        u16(a.x), a.T, a.H, a.I, u32(a.wg), u16(a.sg), u16(a.bg), u32(a.wu), u16(a.su), u16(a.bu), u32(a.we),
        u16(a.se), u16(a.be), a.ebits, a.egs, static_cast<uint16_t *>(a.act), static_cast<uint16_t *>(a.gl),
        L.xbytes > 0);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

// (bits, group_size, scale type) -> one instantiation of F
template <template <int, int, bool> class F, typename... A>
int dispatch(int bits, int gs, int sb_fp16, A &&...args) {
#define MOE_SH_CASE(B, G)                                                               \
    if (bits == B && gs == G)                                                           \
        return sb_fp16 ? F<B, G, true>::run(std::forward<A>(args)...)                   \
                       : F<B, G, false>::run(std::forward<A>(args)...);
    MOE_SH_CASE(2, 32) MOE_SH_CASE(2, 64) MOE_SH_CASE(2, 128)
    MOE_SH_CASE(4, 32) MOE_SH_CASE(4, 64) MOE_SH_CASE(4, 128)
    MOE_SH_CASE(8, 32) MOE_SH_CASE(8, 64) MOE_SH_CASE(8, 128)
#undef MOE_SH_CASE
    return moe_set_error(MOE_EINVAL, "affine linear: no kernel for bits=%d group_size=%d", bits, gs);
}

template <int kBits, int kGs, bool kFp16>
struct LinRun {
    static int run(const void *x, int T, int Kin, int N, const void *w, const void *s, const void *b, const void *gl,
                   void *y, float *yf, cudaStream_t st) {
        return launch_lin_t<kBits, kGs, kFp16>(x, T, Kin, N, w, s, b, gl, y, yf, st);
    }
};

template <int kBits, int kGs, bool kFp16>
struct GateUpRun {
    static int run(const GateUpArgs &a, cudaStream_t st) { return launch_gateup_t<kBits, kGs, kFp16>(a, st); }
};

}  // namespace

int moe_qlin_check(const char *who, const void *x, int T, int Kin, int N, const void *w, const void *s,
                   const void *b, int bits, int gs, const void *y) {
    return check_lin(who, x, T, Kin, N, w, s, b, bits, gs, y);
}

int moe_qlin_linear(const void *x, int T, int Kin, int N, const void *w, const void *s, const void *b, int bits,
                    int gs, int sb_fp16, const void *gl, void *y, float *yf, cudaStream_t st) {
    return dispatch<LinRun>(bits, gs, sb_fp16, x, T, Kin, N, w, s, b, gl, y, yf, st);
}

extern "C" int moe_affine_linear(const void *x, int T, int Kin, int N, const void *w, const void *scales,
                                 const void *biases, int bits, int group_size, int sb_fp16, void *y, void *stream) {
    int rc = check_lin("affine_linear", x, T, Kin, N, w, scales, biases, bits, group_size, y);
    if (rc) return rc;
    return dispatch<LinRun>(bits, group_size, sb_fp16, x, T, Kin, N, w, scales, biases, nullptr, y,
                            static_cast<float *>(nullptr), as_stream(stream));
}

extern "C" size_t moe_shared_expert_workspace_bytes(int T, int H, int I) {
    if (T <= 0 || H <= 0 || I <= 0) return 0;
    return al256((size_t)T * I * 2) + al256((size_t)T * 2);
}

extern "C" int moe_shared_expert(const void *x, int T, int H, int I, const void *wg, const void *sg, const void *bg,
                                 const void *wu, const void *su, const void *bu, const void *wd, const void *sd,
                                 const void *bd, int bits, int group_size, const void *weg, const void *seg,
                                 const void *beg, int gate_bits, int gate_group_size, int sb_fp16, void *y,
                                 void *workspace, size_t workspace_bytes, void *stream) {
    if (!workspace) return moe_set_error(MOE_EINVAL, "shared_expert: null workspace");
    const size_t need = moe_shared_expert_workspace_bytes(T, H, I);
    if (need == 0 || workspace_bytes < need)
        return moe_set_error(MOE_EINVAL, "shared_expert: workspace of %zu bytes needed, %zu given", need,
                             workspace_bytes);
    int rc = check_lin("shared_expert gate_proj", x, T, H, I, wg, sg, bg, bits, group_size, y);
    if (!rc) rc = check_lin("shared_expert up_proj", x, T, H, I, wu, su, bu, bits, group_size, y);
    if (!rc) rc = check_lin("shared_expert down_proj", workspace, T, I, H, wd, sd, bd, bits, group_size, y);
    if (!rc) rc = check_lin("shared_expert gate", x, T, H, 1, weg, seg, beg, gate_bits, gate_group_size, y);
    if (rc) return rc;
    char *p = static_cast<char *>(workspace);
    void *act = p, *gl = p + al256((size_t)T * I * 2);
    cudaStream_t st = as_stream(stream);
    const GateUpArgs a{x, T, H, I, wg, sg, bg, wu, su, bu, weg, seg, beg, gate_bits, gate_group_size, act, gl};
    if ((rc = dispatch<GateUpRun>(bits, group_size, sb_fp16, a, st))) return rc;
    return dispatch<LinRun>(bits, group_size, sb_fp16, act, T, I, H, wd, sd, bd, gl, y, static_cast<float *>(nullptr),
                            st);
}
