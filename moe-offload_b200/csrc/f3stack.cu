// Persistent decode of the step in front of every MoE block, all layers in ONE cooperative
// launch per token: per layer the hyper-connection mixer with the previous block's write
// (Qwen38Engine::run_hc, mlx-qwen38/cpp/src/kernels.cpp:1363-1560) and the shared expert on its
// output (engine.cpp:394-400), the shared expert's output being the block output that the
// next layer's mixer writes (the routed experts are the persistent MoE stack's part,
// csrc/stack.cu). Replaces, per token, the five launches per layer of moe_hc_mix +
// moe_shared_expert with the same arithmetic, bit for bit (one token: the decode regime).
//
// Per layer, with G >= 128 CTAs of 512 threads (one per SM) and five grid barriers:
//   P0a the write (stream c of the state gets bf16(branch * gate_c) added) and the sums of the
//       per-stream RMS norm, split exactly as hc_norm_kernel's reduction tree: CTA 32c + w
//       takes virtual warp w of stream c (virtual thread v sums its values v, v + 1024, ... in
//       order, a xor-shuffle tree per 32) and stores the written state    | barrier
//   P0b every CTA: the 32 warp sums in order, and the normed values of all 4 streams into its
//       shared memory (its loads issued together)
//   P1  mixer down (R rows) and inject (4 rows) over the 4H normed values: CTA j owns rows
//       j, j+G, ...; one thread per (row, group) item, group values in double, row totals in
//       group order (float totals)                                             | barrier
//   P2  mix = silu(down / 4) of all R totals (every CTA), mixer up for the hidden indices the
//       CTA owns (their four stream rows), mixed = mean_c sigmoid(up_c) * normed_c; CTA 0
//       forms inj = 2 sigmoid(inject / 4)                                       | barrier
//   P3  shared gate + up rows the CTA owns, SwiGLU with MLX's bf16 roundings; the scalar
//       expert gate's group values, spread over the CTAs with the fewest rows  | barrier
//   P4  the gate (its group values summed in order), shared down rows the CTA owns scaled by
//       bf16(sigmoid(gate)): the block output                                   | barrier
// The first weight item of every phase is loaded before the barrier in front of it. After the
// last layer CTA 0 applies the last block's write to the state. Every item's group value and
// every row total is formed exactly as in the per-kernel path (qlinear.cuh), so the result does
// not depend on G. Grid barriers are bounded: a timeout sets the device error word.
#include <cstdint>

#include <cuda_runtime.h>

#include "common.cuh"
#include "hcmath.cuh"
#include "qlinear.cuh"
#include "../../include/moe_b200.h"

namespace {

using namespace moe_qlin;

constexpr int kF3Threads = 512;
constexpr int kVirt = 1024;                      // hc_norm_kernel's block size (its reduction tree)
constexpr int kNormK = 4;                        // values per virtual thread and stream: H <= 4096
constexpr int kNormVec = kHcStreams * kNormK * kVirt / (8 * kF3Threads);   // 16-byte vectors per thread (4)
constexpr uint32_t kF3SpinLimit = 1u << 24;

struct F3Args {
    const moe_f3_layer *layers;
    int L, H, R, I;
    float eps;
    const uint16_t *h0, *branch0, *gate0;
    uint16_t *state_out, *branch_out, *inj_out, *branch_all;
    float *dv, *iv;
    double *ssum;                                // [4 streams][32 virtual warps] of the norm's tree
    double *gsum;                                // the scalar expert gate's group values
    uint16_t *mixed, *act, *state, *branch, *inj;
    unsigned int *bar;
};

MOE_D unsigned int ld_acquire_u32(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// barrier n of the launch: waits for (n + 1) * gridDim.x arrivals (the counter only grows)
MOE_D void f3_grid_sync(unsigned int *bar, unsigned int n) {
    __syncthreads();
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const unsigned int target = (n + 1) * gridDim.x;
        uint32_t it = 0;
#pragma unroll 1
        while (ld_acquire_u32(bar) < target) {
            if (++it > kF3SpinLimit) {
                atomicOr(&g_moe_device_error, MOE_DEVERR_MBAR_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

// Phase timestamps for profiling builds (-DMOE_STACK_TRACE, build.py --trace):
// g_f3_trace[cta][layer][slot], read back with moe_f3_trace_read. Slots: 0 layer start, 1 norm
// done, 2 mixer-down items done, 3 barrier 1 passed, 4 mixer up + tail done, 5 barrier 2,
// 6 shared gate / up done, 7 barrier 3, 8 shared down done, 9 barrier 4. The library build
// compiles them out.
#ifdef MOE_STACK_TRACE
constexpr int kF3TraceCtas = 160, kF3TraceLayers = 64, kF3TraceSlots = 16;
__device__ unsigned long long g_f3_trace[kF3TraceCtas * kF3TraceLayers * kF3TraceSlots];
MOE_D void f3_stamp(int layer, int slot) {
    if (threadIdx.x == 0 && blockIdx.x < kF3TraceCtas && layer < kF3TraceLayers) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_f3_trace[((size_t)blockIdx.x * kF3TraceLayers + layer) * kF3TraceSlots + slot] = t;
    }
}
#define F3_STAMP(l, s) f3_stamp(l, s)
#else
#define F3_STAMP(l, s) ((void)0)
#endif

MOE_D const uint16_t *u16(const void *p) { return static_cast<const uint16_t *>(p); }
MOE_D const uint32_t *u32(const void *p) { return static_cast<const uint32_t *>(p); }

// bf16 values (global, possibly written earlier in this launch) -> shared memory, 16 bytes a copy
MOE_D void stage_l2(uint16_t *dst, const uint16_t *src, int n) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int i = threadIdx.x; i < n / 8; i += blockDim.x) d[i] = __ldcg(s + i);
}

struct Smem {
    size_t normed, sx, sv, spart, total;
    MOE_HD Smem(int H, int R, int I, int G) {
        const int W = kHcStreams * H;
        const int rpc1 = (R + kHcStreams + G - 1) / G, rpc2 = (H + G - 1) / G, rpc3 = (I + G - 1) / G;
        size_t items = (size_t)rpc1 * (W / 64);
        const size_t i2 = (size_t)rpc2 * kHcStreams * (R / 64), i3 = (size_t)rpc3 * 2 * (H / 64),
                     i4 = (size_t)rpc2 * (I / 64);
        items = items > i2 ? items : i2;
        items = items > i3 ? items : i3;
        items = items > i4 ? items : i4;
        const int xmax = R > H ? (R > I ? R : I) : (H > I ? H : I);
        normed = 0;
        sx = al128((size_t)W * 2);
        sv = sx + al128((size_t)xmax * 2);
        spart = sv + al128(items * 8);
        total = spart + al128((size_t)(kHcStreams * 32 > H / 64 ? kHcStreams * 32 : H / 64) * 8);
    }
};

template <bool kFp16>
__global__ void __launch_bounds__(kF3Threads, 1) f3_stack_kernel(F3Args a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int H = a.H, R = a.R, I = a.I, W = kHcStreams * H, G = gridDim.x, j = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Smem S(H, R, I, G);
    uint16_t *normed = reinterpret_cast<uint16_t *>(smem + S.normed);
    uint16_t *sx = reinterpret_cast<uint16_t *>(smem + S.sx);
    double *sv = reinterpret_cast<double *>(smem + S.sv);
    double *spart = reinterpret_cast<double *>(smem + S.spart);   // [4 streams][32 virtual warps]
    __shared__ float srs[kHcStreams];
    unsigned int nbar = 0;
    using G8 = GroupItem<8, 64, kFp16>;
    using G4 = GroupItem<4, 64, kFp16>;
    const int ng1 = W / 64, ng2 = R / 64, ng3 = H / 64, ng4 = I / 64;
    // items each CTA owns in every phase (rows j, j + G, ...)
    const int nh = H > j ? (H - 1 - j) / G + 1 : 0;          // P2 hidden indices, P4 rows
    const int ni = I > j ? (I - 1 - j) / G + 1 : 0;          // P3 rows
    // the scalar expert gate's groups: group g on CTA G - 1 - (g mod G), whose row items leave room
    const int ngate = ng3 > G - 1 - j ? (ng3 - 1 - (G - 1 - j)) / G + 1 : 0;

    // item loaders (weights only: they never depend on an earlier phase, so the first item of
    // a phase is loaded before the barrier that precedes it)
    auto load1 = [&](const moe_f3_layer &Ly, int it, G8 &gi) {
        const int k = it / ng1, g = it - k * ng1, row = j + k * G;
        const bool inj = row >= R;
        const int rr = inj ? row - R : row;
        gi.load(u32(inj ? Ly.wi : Ly.wd) + (size_t)rr * (W / 4), u16(inj ? Ly.si : Ly.sd) + (size_t)rr * ng1,
                u16(inj ? Ly.bi : Ly.bd) + (size_t)rr * ng1, g);
    };
    auto load2 = [&](const moe_f3_layer &Ly, int it, G8 &gi) {
        const int per = kHcStreams * ng2;
        const int k = it / per, c = (it / ng2) % kHcStreams, g = it % ng2;
        const size_t row = (size_t)c * H + (j + k * G);
        gi.load(u32(Ly.wu) + row * (R / 4), u16(Ly.su) + row * ng2, u16(Ly.bu) + row * ng2, g);
    };
    auto load3 = [&](const moe_f3_layer &Ly, int it, G4 &gi) {
        const int per = 2 * ng3;
        const int k = it / per, m = (it / ng3) & 1, g = it % ng3;
        const size_t row = (size_t)(j + k * G);
        gi.load(u32(m ? Ly.wsu : Ly.wsg) + row * (H / 8), u16(m ? Ly.ssu : Ly.ssg) + row * ng3,
                u16(m ? Ly.bsu : Ly.bsg) + row * ng3, g);
    };
    auto load4 = [&](const moe_f3_layer &Ly, int it, G4 &gi) {
        const int k = it / ng4, g = it - k * ng4;
        const size_t row = (size_t)(j + k * G);
        gi.load(u32(Ly.wsd) + row * (I / 8), u16(Ly.ssd) + row * ng4, u16(Ly.bsd) + row * ng4, g);
    };
    auto nrows1 = [&](const moe_f3_layer &Ly) {
        const int N1 = R + (Ly.wi ? kHcStreams : 0);
        return N1 > j ? (N1 - 1 - j) / G + 1 : 0;
    };

    G8 pf1, pf2;
    G4 pf3, pf4;
    if (tid < nrows1(a.layers[0]) * ng1) load1(a.layers[0], tid, pf1);

#pragma unroll 1
    for (int l = 0; l < a.L; ++l) {
        const moe_f3_layer &Ly = a.layers[l];
        const uint16_t *hin = l == 0 ? a.h0 : a.state + (size_t)(l & 1) * W;
        const uint16_t *br = l == 0 ? a.branch0 : a.branch + (size_t)((l - 1) & 1) * H;
        const uint16_t *gt = l == 0 ? a.gate0 : a.inj + (size_t)((l - 1) & 1) * kHcStreams;
        uint16_t *wout = a.state + (size_t)((l + 1) & 1) * W;
        const int nrows = nrows1(Ly);
        F3_STAMP(l, 0);

        // ---------------------------------------------------------------- P0a: write + sums
        // hc_norm_kernel's tree per stream c: virtual thread v (of 1024) sums its values v,
        // v + 1024, ... in order, a xor-shuffle tree per 32 virtual threads, then the 32 warp
        // sums in order. CTA 32 c + w (w < 32) takes virtual warp w of stream c: it forms the
        // written values of its elements (stored as the next state) and the warp's sum.
        if (j < kHcStreams * 32 && warp == 0) {
            const int c = j >> 5, w = j & 31, v = 32 * w + lane;
            const float gv = br ? bf16_bits_to_f32(__ldcg(gt + c)) : 0.f;
            uint16_t hv[kNormK], bv[kNormK];
#pragma unroll
            for (int k = 0; k < kNormK; ++k) {
                const int i = v + kVirt * k;
                hv[k] = i < H ? __ldcg(hin + (size_t)c * H + i) : (uint16_t)0;
                bv[k] = (i < H && br) ? __ldcg(br + i) : (uint16_t)0;
            }
            double ss = 0.0;
#pragma unroll
            for (int k = 0; k < kNormK; ++k) {
                const int i = v + kVirt * k;
                if (i >= H) continue;
                float x = bf16_bits_to_f32(hv[k]);
                if (br) x = bf16r(__fadd_rn(x, bf16r(__fmul_rn(bf16_bits_to_f32(bv[k]), gv))));
                wout[(size_t)c * H + i] = f32_to_bf16_bits(x);
                ss += (double)x * (double)x;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            if (lane == 0) a.ssum[c * 32 + w] = ss;
        }
        F3_STAMP(l, 12);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 10);

        // ---------------------------------------------------------------- P0b: norm (every CTA)
        {
            if (tid < kHcStreams * 32) spart[tid] = __ldcg(a.ssum + tid);
            const uint16_t *nw = u16(Ly.norm_w);
            // every load of the thread's elements first (the pass is latency-bound otherwise):
            // 8 consecutive values per 16-byte load
            uint4 xv[kNormVec], wv[kNormVec];
#pragma unroll
            for (int m = 0; m < kNormVec; ++m) {
                const int q = 8 * (tid + kF3Threads * m);
                xv[m] = q < W ? __ldcg(reinterpret_cast<const uint4 *>(wout + q)) : make_uint4(0u, 0u, 0u, 0u);
                wv[m] = q < W ? __ldg(reinterpret_cast<const uint4 *>(nw + q)) : make_uint4(0u, 0u, 0u, 0u);
            }
            __syncthreads();
            if (tid < kHcStreams) {
                double tot = 0.0;
                for (int w = 0; w < kVirt / 32; ++w) tot += spart[tid * 32 + w];
                srs[tid] = (float)(1.0 / sqrt(tot / H + (double)a.eps));
            }
            __syncthreads();
#pragma unroll
            for (int m = 0; m < kNormVec; ++m) {
                const int q = 8 * (tid + kF3Threads * m);
                if (q >= W) continue;
                const float rs = srs[q / H];
                const uint32_t xw[4] = {xv[m].x, xv[m].y, xv[m].z, xv[m].w}, ww[4] = {wv[m].x, wv[m].y, wv[m].z, wv[m].w};
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float y0 = __fmul_rn(bf16_lo(xw[e]), rs), y1 = __fmul_rn(bf16_hi(xw[e]), rs);
                    const float s0 = __fadd_rn(1.0f, bf16_lo(ww[e])), s1 = __fadd_rn(1.0f, bf16_hi(ww[e]));
                    o[e] = (uint32_t)f32_to_bf16_bits(__fmul_rn(y0, s0)) | ((uint32_t)f32_to_bf16_bits(__fmul_rn(y1, s1)) << 16);
                }
                *reinterpret_cast<uint4 *>(normed + q) = make_uint4(o[0], o[1], o[2], o[3]);
            }
            __syncthreads();
        }
        F3_STAMP(l, 1);

        // ---------------------------------------------------------------- P1: mixer down + inject
        for (int it = tid; it < nrows * ng1; it += kF3Threads) {
            if (it != tid) load1(Ly, it, pf1);
            sv[it] = pf1.value(normed + (size_t)(it % ng1) * 64);
        }
        if (tid < nh * kHcStreams * ng2) load2(Ly, tid, pf2);
        __syncthreads();
        for (int q = tid; q < nrows; q += kF3Threads) {
            const int row = j + q * G;
            const float tot = (float)sum_in_order(sv + (size_t)q * ng1, ng1);
            if (row < R) a.dv[row] = tot;
            else a.iv[row - R] = tot;
        }
        F3_STAMP(l, 2);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 3);

        // ---------------------------------------------------------------- P2: mixer up + tail
        {
            for (int k = tid; k < R; k += kF3Threads) sx[k] = f32_to_bf16_bits(hc_mix_value(__ldcg(a.dv + k), 0));
            uint16_t *injo = a.inj + (size_t)(l & 1) * kHcStreams;
            if (j == 0 && tid < kHcStreams)
                injo[tid] = f32_to_bf16_bits(Ly.wi ? hc_inj_value(__ldcg(a.iv + tid), 0) : 0.f);
            __syncthreads();
            for (int it = tid; it < nh * kHcStreams * ng2; it += kF3Threads) {
                if (it != tid) load2(Ly, it, pf2);
                sv[it] = pf2.value(sx + (size_t)(it % ng2) * 64);
            }
            if (tid < ni * 2 * ng3) load3(Ly, tid, pf3);
            __syncthreads();
            for (int q = tid; q < nh; q += kF3Threads) {
                const int hh = j + q * G;
                float acc = 0.f;
#pragma unroll
                for (int c = 0; c < kHcStreams; ++c) {
                    const float u = (float)sum_in_order(sv + (size_t)(q * kHcStreams + c) * ng2, ng2);
                    const float nv = bf16_bits_to_f32(normed[(size_t)c * H + hh]);
                    const float p = __fmul_rn(sigmoidf(u), nv);
                    acc = c == 0 ? p : __fadd_rn(acc, p);
                }
                a.mixed[hh] = f32_to_bf16_bits(__fdiv_rn(acc, (float)kHcStreams));
            }
        }
        F3_STAMP(l, 4);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 5);

        // ---------------------------------------------------------------- P3: shared gate / up
        {
            stage_l2(sx, a.mixed, H);
            __syncthreads();
            const int per = 2 * ng3;
            for (int it = tid; it < ni * per; it += kF3Threads) {
                if (it != tid) load3(Ly, it, pf3);
                sv[it] = pf3.value(sx + (size_t)(it % ng3) * 64);
            }
            for (int q = tid; q < ngate; q += kF3Threads) {   // the scalar expert gate's groups (8-bit g64)
                const int g = (G - 1 - j) + q * G;
                G8 gi;
                gi.load(u32(Ly.wse), u16(Ly.sse), u16(Ly.bse), g);
                a.gsum[g] = gi.value(sx + (size_t)g * 64);
            }
            if (tid < nh * ng4) load4(Ly, tid, pf4);
            __syncthreads();
            for (int q = tid; q < ni; q += kF3Threads) {
                const int i = j + q * G;
                const float gv = bf16_bits_to_f32(row_out(sum_in_order(sv + (size_t)(q * 2) * ng3, ng3)));
                const float uv = bf16_bits_to_f32(row_out(sum_in_order(sv + (size_t)(q * 2 + 1) * ng3, ng3)));
                a.act[i] = f32_to_bf16_bits(bf16r(__fmul_rn(bf16r(__fmul_rn(gv, sigmoid_bf16(gv))), uv)));
            }
        }
        F3_STAMP(l, 6);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 7);

        // ---------------------------------------------------------------- P4: shared down
        {
            stage_l2(sx, a.act, I);
            if (tid < ng3) spart[tid] = __ldcg(a.gsum + tid);
            __syncthreads();
            if (tid == 0) srs[0] = sigmoid_bf16(bf16_bits_to_f32(row_out(sum_in_order(spart, ng3))));
            __syncthreads();
            const float gsig = srs[0];
            uint16_t *bro = a.branch + (size_t)(l & 1) * H;
            for (int it = tid; it < nh * ng4; it += kF3Threads) {
                if (it != tid) load4(Ly, it, pf4);
                sv[it] = pf4.value(sx + (size_t)(it % ng4) * 64);
            }
            if (l + 1 < a.L && tid < nrows1(a.layers[l + 1]) * ng1) load1(a.layers[l + 1], tid, pf1);
            __syncthreads();
            for (int q = tid; q < nh; q += kF3Threads) {
                const int n = j + q * G;
                const uint16_t o = row_out(sum_in_order(sv + (size_t)q * ng4, ng4));
                const uint16_t y = f32_to_bf16_bits(__fmul_rn(gsig, bf16_bits_to_f32(o)));
                bro[n] = y;
                if (a.branch_all) a.branch_all[(size_t)l * H + n] = y;
            }
        }
        F3_STAMP(l, 8);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 9);
    }

    // the last block's write into the state, and the last block output and gate
    if (j == 0) {
        const int l = a.L - 1;
        const uint16_t *st = a.state + (size_t)((l + 1) & 1) * W;
        const uint16_t *br = a.branch + (size_t)(l & 1) * H;
        const uint16_t *gt = a.inj + (size_t)(l & 1) * kHcStreams;
        for (int q = tid; q < W; q += kF3Threads) {
            const int c = q / H, i = q - c * H;
            const float gv = bf16_bits_to_f32(__ldcg(gt + c));
            const float p = bf16r(__fmul_rn(bf16_bits_to_f32(__ldcg(br + i)), gv));
            a.state_out[q] = f32_to_bf16_bits(bf16r(__fadd_rn(bf16_bits_to_f32(__ldcg(st + q)), p)));
        }
        for (int q = tid; q < H; q += kF3Threads) a.branch_out[q] = __ldcg(br + q);
        if (tid < kHcStreams && a.inj_out) a.inj_out[tid] = __ldcg(gt + tid);
    }
}

struct F3Ws {
    size_t dv, iv, ssum, gsum, mixed, act, state, branch, inj, bar, total;
    F3Ws(int H, int R, int I) {
        const size_t W = (size_t)kHcStreams * H;
        dv = 0;
        iv = dv + al256((size_t)R * 4);
        ssum = iv + al256(kHcStreams * 4);
        gsum = ssum + al256(kHcStreams * 32 * 8);
        mixed = gsum + al256((size_t)(H / 64) * 8);
        act = mixed + al256((size_t)H * 2);
        state = act + al256((size_t)I * 2);
        branch = state + al256(2 * W * 2);
        inj = branch + al256(2 * (size_t)H * 2);
        bar = inj + 256;
        total = bar + 256;
    }
};

}  // namespace

extern "C" size_t moe_f3_stack_workspace_bytes(int H, int R, int I) {
    if (H <= 0 || R <= 0 || I <= 0) return 0;
    return F3Ws(H, R, I).total;
}

extern "C" int moe_f3_stack_decode(const void *layers, int L, int H, int R, int I, int sb_fp16, float eps,
                                   const void *h, const void *branch0, const void *gate0, void *state_out,
                                   void *branch_out, void *inj_out, void *branch_all, void *workspace,
                                   size_t workspace_bytes, int num_ctas, void *stream) {
    if (!layers || !h || !state_out || !branch_out || !workspace)
        return moe_set_error(MOE_EINVAL, "f3_stack_decode: null pointer");
    if (L <= 0 || H <= 0 || R <= 0 || I <= 0 || H % 64 || R % 64 || I % 64 || H > kVirt * kNormK)
        return moe_set_error(MOE_EINVAL, "f3_stack_decode: bad sizes L=%d H=%d R=%d I=%d (multiples of 64, H <= %d)", L,
                             H, R, I, kVirt * kNormK);
    if ((branch0 == nullptr) != (gate0 == nullptr))
        return moe_set_error(MOE_EINVAL, "f3_stack_decode: the first write needs both branch and gate");
    if (!(eps >= 0.f)) return moe_set_error(MOE_EINVAL, "f3_stack_decode: eps must be >= 0");
    const F3Ws w(H, R, I);
    if (workspace_bytes < w.total)
        return moe_set_error(MOE_EINVAL, "f3_stack_decode: workspace of %zu bytes needed, %zu given", w.total,
                             workspace_bytes);
    const void *bufs[] = {h, branch0, state_out, branch_out, workspace, branch_all};
    for (const void *p : bufs)
        if (reinterpret_cast<uintptr_t>(p) % 16)
            return moe_set_error(MOE_EINVAL, "f3_stack_decode: buffers must be 16-byte aligned");
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int G = num_ctas > 0 ? (num_ctas < sms ? num_ctas : sms) : sms;
    if (G < kHcStreams * 32)
        return moe_set_error(MOE_EINVAL, "f3_stack_decode: %d CTAs (the norm takes %d)", G, kHcStreams * 32);
    const Smem S(H, R, I, G);
    if (S.total > 200 * 1024) return moe_set_error(MOE_EINVAL, "f3_stack_decode: shapes need %zu bytes of shared memory", S.total);
    char *p = static_cast<char *>(workspace);
    F3Args a{};
    a.layers = static_cast<const moe_f3_layer *>(layers);
    a.L = L, a.H = H, a.R = R, a.I = I, a.eps = eps;
    a.h0 = static_cast<const uint16_t *>(h);
    a.branch0 = static_cast<const uint16_t *>(branch0);
    a.gate0 = static_cast<const uint16_t *>(gate0);
    a.state_out = static_cast<uint16_t *>(state_out);
    a.branch_out = static_cast<uint16_t *>(branch_out);
    a.inj_out = static_cast<uint16_t *>(inj_out);
    a.branch_all = static_cast<uint16_t *>(branch_all);
    a.dv = reinterpret_cast<float *>(p + w.dv);
    a.iv = reinterpret_cast<float *>(p + w.iv);
    a.ssum = reinterpret_cast<double *>(p + w.ssum);
    a.gsum = reinterpret_cast<double *>(p + w.gsum);
    a.mixed = reinterpret_cast<uint16_t *>(p + w.mixed);
    a.act = reinterpret_cast<uint16_t *>(p + w.act);
    a.state = reinterpret_cast<uint16_t *>(p + w.state);
    a.branch = reinterpret_cast<uint16_t *>(p + w.branch);
    a.inj = reinterpret_cast<uint16_t *>(p + w.inj);
    a.bar = reinterpret_cast<unsigned int *>(p + w.bar);
    cudaStream_t st = as_stream(stream);
    MOE_CUDA_TRY(cudaMemsetAsync(a.bar, 0, sizeof(unsigned int), st));
    void *kern = sb_fp16 ? (void *)f3_stack_kernel<true> : (void *)f3_stack_kernel<false>;
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S.total));
    void *kargs[] = {&a};
    MOE_CUDA_TRY(cudaLaunchCooperativeKernel(kern, dim3(G), dim3(kF3Threads), kargs, S.total, st));
    return MOE_OK;
}

#ifdef MOE_STACK_TRACE
extern "C" int moe_f3_trace_read(unsigned long long *host, size_t n) {
    const size_t total = (size_t)kF3TraceCtas * kF3TraceLayers * kF3TraceSlots;
    MOE_CUDA_TRY(cudaMemcpyFromSymbol(host, g_f3_trace, (n < total ? n : total) * sizeof(unsigned long long)));
    return MOE_OK;
}
#endif
