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
// Kernels (qlinear.cuh): one thread per (matrix, row, group) item, its codes loaded before the
// kernel waits on its predecessor (programmatic dependent launch); group values in shared
// memory, added in group order by one thread per (row, token). The shared expert is two
// launches: gate + up + SwiGLU (+ one block for the scalar expert gate), then down with the
// sigmoid(gate) scale in its epilogue.
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
// with yf != nullptr, float(row total) to yf; rows N .. N+N2-1 are the rows of a second matrix
// (w2, s2, b2), written as float totals to yf2. Block: `rows` rows x ng groups, one per thread.
template <int kBits, int kGs, bool kFp16>
__global__ void __launch_bounds__(max_block(kGs)) affine_linear_kernel(
    const uint16_t *__restrict__ x, int T, int Kin, int N, const uint32_t *__restrict__ w,
    const uint16_t *__restrict__ s, const uint16_t *__restrict__ b, const uint16_t *__restrict__ gl,
    uint16_t *__restrict__ y, float *__restrict__ yf, const uint32_t *__restrict__ w2, const uint16_t *__restrict__ s2,
    const uint16_t *__restrict__ b2, int N2, float *__restrict__ yf2) {
    extern __shared__ __align__(16) unsigned char lin_smem_raw[];
    using GI = GroupItem<kBits, kGs, kFp16>;
    const int ng = Kin / kGs;
    const FlatShape F = flat_shape(1, ng, T, Kin);
    double *sv = reinterpret_cast<double *>(lin_smem_raw);              // [rows][kLinTok][ng]
    uint16_t *sx = reinterpret_cast<uint16_t *>(lin_smem_raw + F.grp);
    const int r = threadIdx.x / ng, g = threadIdx.x - r * ng;
    const int n = blockIdx.x * F.rows + r;
    const bool item = r < F.rows && n < N + N2;
    GI it;
    if (item) {
        const bool second = n >= N;
        const size_t row = second ? n - N : n;
        it.load((second ? w2 : w) + row * (Kin / GI::kPer), (second ? s2 : s) + row * ng,
                (second ? b2 : b) + row * ng, g);
    }
    pdl_launch_dependents();
    pdl_wait();                                  // x (and gl) come from earlier kernels
#pragma unroll 1
    for (int t0 = 0; t0 < T; t0 += kLinTok) {
        const int nt = min(kLinTok, T - t0);
        const uint16_t *xs = x + (size_t)t0 * Kin;
        __syncthreads();                         // the previous pass is done with sx and sv
        if (F.xbytes) {
            stage_x(sx, x, Kin, t0, nt);
            __syncthreads();
            xs = sx;
        }
        if (item)
            for (int j = 0; j < nt; ++j) sv[(r * kLinTok + j) * ng + g] = it.value(xs + (size_t)j * Kin + (size_t)g * kGs);
        __syncthreads();
        for (int q = threadIdx.x; q < F.rows * nt; q += blockDim.x) {
            const int rr = q / nt, j = q - rr * nt, nn = blockIdx.x * F.rows + rr, t = t0 + j;
            if (nn >= N + N2) continue;
            const double total = sum_in_order(sv + (rr * kLinTok + j) * ng, ng);
            if (nn >= N) {
                yf2[(size_t)t * N2 + (nn - N)] = (float)total;
            } else if (yf) {
                yf[(size_t)t * N + nn] = (float)total;
            } else {
                uint16_t o = row_out(total);
                if (gl) o = f32_to_bf16_bits(__fmul_rn(sigmoid_bf16(bf16_bits_to_f32(gl[t])), bf16_bits_to_f32(o)));
                y[(size_t)t * N + nn] = o;
            }
        }
    }
}

// act[t][i] = bf16(bf16(g * bf16(sigmoid(g))) * u) with g, u rows i of the gate / up
// projections: items (row, matrix, group). The last block computes gl[t] = x[t] . We (the
// scalar expert gate, runtime bits / group size).
template <int kBits, int kGs, bool kFp16>
__global__ void __launch_bounds__(max_block(kGs)) gateup_swiglu_kernel(
    const uint16_t *__restrict__ x, int T, int H, int I, const uint32_t *__restrict__ wg,
    const uint16_t *__restrict__ sg, const uint16_t *__restrict__ bg, const uint32_t *__restrict__ wu,
    const uint16_t *__restrict__ su, const uint16_t *__restrict__ bu, const uint32_t *__restrict__ we,
    const uint16_t *__restrict__ se, const uint16_t *__restrict__ be, int ebits, int egs,
    uint16_t *__restrict__ act, uint16_t *__restrict__ gl) {
    extern __shared__ __align__(16) unsigned char lin_smem_raw[];
    using GI = GroupItem<kBits, kGs, kFp16>;
    const int ng = H / kGs, nge = H / egs;
    FlatShape F = flat_shape(2, ng, T, H);
    const size_t gate_grp = (size_t)kLinTok * nge * sizeof(double);   // the gate block's values
    if (gate_grp > F.grp) F.grp = gate_grp;
    double *sv = reinterpret_cast<double *>(lin_smem_raw);              // [rows][2][kLinTok][ng]
    uint16_t *sx = reinterpret_cast<uint16_t *>(lin_smem_raw + F.grp);
    const bool gate_block = blockIdx.x == gridDim.x - 1;
    // the gate block's copy of the scalar gate row: codes, then scales, then biases
    uint32_t *gw = reinterpret_cast<uint32_t *>(lin_smem_raw + F.grp + F.xbytes);
    const int gwords = H * ebits / 32;
    uint16_t *gsc = reinterpret_cast<uint16_t *>(gw + gwords), *gbi = gsc + nge;
    if (gate_block) {                            // weights only: copied before the wait
        for (int k = threadIdx.x; k < gwords; k += blockDim.x) gw[k] = __ldg(we + k);
        for (int k = threadIdx.x; k < nge; k += blockDim.x) gsc[k] = __ldg(se + k), gbi[k] = __ldg(be + k);
    }
    const int m = (threadIdx.x / ng) & 1, r = threadIdx.x / (2 * ng), g = threadIdx.x % ng;
    const int i = blockIdx.x * F.rows + r;
    const bool item = !gate_block && r < F.rows && i < I;
    GI it;
    if (item) {
        const size_t row = i;
        it.load((m ? wu : wg) + row * (H / GI::kPer), (m ? su : sg) + row * ng, (m ? bu : bg) + row * ng, g);
    }
    pdl_launch_dependents();
    pdl_wait();                                  // x comes from earlier kernels
#pragma unroll 1
    for (int t0 = 0; t0 < T; t0 += kLinTok) {
        const int nt = min(kLinTok, T - t0);
        const uint16_t *xs = x + (size_t)t0 * H;
        __syncthreads();
        if (F.xbytes) {
            stage_x(sx, x, H, t0, nt);
            __syncthreads();
            xs = sx;
        }
        if (gate_block) {                        // [kLinTok][nge] values of the scalar gate
            for (int q = threadIdx.x; q < nge * nt; q += blockDim.x) {
                const int j = q / nge, ge = q - j * nge;
                sv[j * nge + ge] = generic_group_value<kFp16>(xs + (size_t)j * H + (size_t)ge * egs, gw, gsc, gbi,
                                                              ebits, egs, ge);
            }
            __syncthreads();
            if ((int)threadIdx.x < nt) gl[t0 + threadIdx.x] = row_out(sum_in_order(sv + threadIdx.x * nge, nge));
            continue;
        }
        if (item)
            for (int j = 0; j < nt; ++j)
                sv[((r * 2 + m) * kLinTok + j) * ng + g] = it.value(xs + (size_t)j * H + (size_t)g * kGs);
        __syncthreads();
        for (int q = threadIdx.x; q < F.rows * nt; q += blockDim.x) {
            const int rr = q / nt, j = q - rr * nt, ii = blockIdx.x * F.rows + rr;
            if (ii >= I) continue;
            const float gv = bf16_bits_to_f32(row_out(sum_in_order(sv + ((rr * 2) * kLinTok + j) * ng, ng)));
            const float uv = bf16_bits_to_f32(row_out(sum_in_order(sv + ((rr * 2 + 1) * kLinTok + j) * ng, ng)));
            act[(size_t)(t0 + j) * I + ii] =
                f32_to_bf16_bits(bf16r(__fmul_rn(bf16r(__fmul_rn(gv, sigmoid_bf16(gv))), uv)));
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
    const int gmax = kMaxGroups < max_block(gs) ? kMaxGroups : max_block(gs);
    if (Kin / gs > gmax) return moe_set_error(MOE_EINVAL, "%s: %d groups per row (at most %d)", who, Kin / gs, gmax);
    const uintptr_t wa = (gs * bits / 8) % 16 ? 8 : 16;      // the group's word loads
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % wa)
        return moe_set_error(MOE_EINVAL, "%s: x must be 16-byte and codes %d-byte aligned", who, (int)wa);
    return MOE_OK;
}

template <int kBits, int kGs, bool kFp16>
int launch_lin_t(const void *x, int T, int Kin, int N, const void *w, const void *s, const void *b, const void *gl,
                 void *y, float *yf, const void *w2, const void *s2, const void *b2, int N2, float *yf2,
                 cudaStream_t st) {
    const FlatShape F = flat_shape(1, Kin / kGs, T, Kin);
    const int rows = N + N2;
    MOE_CUDA_TRY(launch_pdl_v(affine_linear_kernel<kBits, kGs, kFp16>, dim3((rows + F.rows - 1) / F.rows),
                              dim3(F.threads), F.smem(), st, static_cast<const uint16_t *>(x), T, Kin, N,
                              static_cast<const uint32_t *>(w), static_cast<const uint16_t *>(s),
                              static_cast<const uint16_t *>(b), static_cast<const uint16_t *>(gl),
                              static_cast<uint16_t *>(y), yf, static_cast<const uint32_t *>(w2),
                              static_cast<const uint16_t *>(s2), static_cast<const uint16_t *>(b2), N2, yf2));
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
    FlatShape F = flat_shape(2, a.H / kGs, a.T, a.H);
    // the gate block keeps [kLinTok][H / egs] values in the same region (as the kernel computes)
    F.grp = std::max(F.grp, (size_t)kLinTok * (a.H / a.egs) * sizeof(double));
    // plus the gate block's copy of the scalar gate row (codes, scales, biases)
    const size_t gate_row = (size_t)a.H * a.ebits / 8 + (size_t)(a.H / a.egs) * 4;
    auto u16 = [](const void *p) { return static_cast<const uint16_t *>(p); };
    auto u32 = [](const void *p) { return static_cast<const uint32_t *>(p); };
    MOE_CUDA_TRY(launch_pdl_v(gateup_swiglu_kernel<kBits, kGs, kFp16>, dim3((a.I + F.rows - 1) / F.rows + 1),
                              dim3(F.threads), F.smem() + gate_row, st, u16(a.x), a.T, a.H, a.I, u32(a.wg), u16(a.sg), u16(a.bg),
                              u32(a.wu), u16(a.su), u16(a.bu), u32(a.we), u16(a.se), u16(a.be), a.ebits, a.egs,
                              static_cast<uint16_t *>(a.act), static_cast<uint16_t *>(a.gl)));
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
                   void *y, float *yf, const void *w2, const void *s2, const void *b2, int N2, float *yf2,
                   cudaStream_t st) {
        return launch_lin_t<kBits, kGs, kFp16>(x, T, Kin, N, w, s, b, gl, y, yf, w2, s2, b2, N2, yf2, st);
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
                    int gs, int sb_fp16, const void *gl, void *y, float *yf, cudaStream_t st, const void *w2,
                    const void *s2, const void *b2, int N2, float *yf2) {
    if (N2 > 0 && !(w2 && s2 && b2 && yf2)) return moe_set_error(MOE_EINVAL, "affine linear: second matrix incomplete");
    return dispatch<LinRun>(bits, gs, sb_fp16, x, T, Kin, N, w, s, b, gl, y, yf, w2, s2, b2, N2 > 0 ? N2 : 0, yf2, st);
}

extern "C" int moe_affine_linear(const void *x, int T, int Kin, int N, const void *w, const void *scales,
                                 const void *biases, int bits, int group_size, int sb_fp16, void *y, void *stream) {
    int rc = check_lin("affine_linear", x, T, Kin, N, w, scales, biases, bits, group_size, y);
    if (rc) return rc;
    return moe_qlin_linear(x, T, Kin, N, w, scales, biases, bits, group_size, sb_fp16, nullptr, y, nullptr,
                           as_stream(stream));
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
    if (2 * (H / group_size) > max_block(group_size))
        return moe_set_error(MOE_EINVAL, "shared_expert: %d groups per row (at most %d)", H / group_size,
                             max_block(group_size) / 2);
    char *p = static_cast<char *>(workspace);
    void *act = p, *gl = p + al256((size_t)T * I * 2);
    cudaStream_t st = as_stream(stream);
    const GateUpArgs a{x, T, H, I, wg, sg, bg, wu, su, bu, weg, seg, beg, gate_bits, gate_group_size, act, gl};
    if ((rc = dispatch<GateUpRun>(bits, group_size, sb_fp16, a, st))) return rc;
    return moe_qlin_linear(act, T, I, H, wd, sd, bd, bits, group_size, sb_fp16, gl, y, nullptr, st);
}
