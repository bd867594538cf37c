// The phases of the step in front of every MoE block at decode (one token): the
// hyper-connection mixer with the previous block's write (Qwen38Engine::run_hc,
// mlx-qwen38/cpp/src/kernels.cpp:1363-1560) and the shared expert on its output
// (engine.cpp:394-400), as device code for persistent cooperative kernels of 512 threads per
// CTA: csrc/f3stack.cu runs them alone, csrc/stack.cu fused with the routed block.
//
// Every item's group value and every row total is formed exactly as in the per-launch path
// (moe_hc_mix + moe_shared_expert, qlinear.cuh), so the results do not depend on the CTA count.
// The phase functions run between grid barriers; each loads the first weight item of the next
// phase before returning, so that load overlaps the barrier in front of that phase.
#pragma once

#include <cstdint>

#include "common.cuh"
#include "hcmath.cuh"
#include "qlinear.cuh"
#include "../../include/moe_b200.h"

namespace moe_f3 {

using namespace moe_qlin;

constexpr int kF3Threads = 512;
constexpr int kVirt = 1024;                      // hc_norm_kernel's block size (its reduction tree)
constexpr int kNormK = 4;                        // values per virtual thread and stream: H <= 4096
constexpr int kNormVec = kHcStreams * kNormK * kVirt / (8 * kF3Threads);   // 16-byte vectors per thread (4)

MOE_D const uint16_t *u16(const void *p) { return static_cast<const uint16_t *>(p); }
MOE_D const uint32_t *u32(const void *p) { return static_cast<const uint32_t *>(p); }

// bf16 values (global, possibly written earlier in this launch) -> shared memory, 16 bytes a copy
MOE_D void stage_l2(uint16_t *dst, const uint16_t *src, int n) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *d = reinterpret_cast<uint4 *>(dst);
    for (int i = threadIdx.x; i < n / 8; i += blockDim.x) d[i] = __ldcg(s + i);
}

// global scratch of the phases (written and read within a layer, through L2)
struct F3Bufs {
    float *dv, *iv;          // mixer down row totals [R], inject totals [4]
    double *ssum;            // [4 streams][32 virtual warps] of the norm's tree
    double *gsum;            // the scalar expert gate's group values [H / 64]
    uint16_t *mixed, *act;   // the mixer output [H], the shared expert's SwiGLU [I]
};

// shared memory of the phases; extra_items: group values a caller's own phase keeps in sv
struct F3Smem {
    size_t normed, sx, sv, spart, total;
    MOE_HD F3Smem(int H, int R, int I, int G, size_t extra_items = 0) {
        const int W = kHcStreams * H;
        const int rpc1 = (R + kHcStreams + G - 1) / G, rpc2 = (H + G - 1) / G, rpc3 = (I + G - 1) / G;
        size_t items = (size_t)rpc1 * (W / 64);
        const size_t i2 = (size_t)rpc2 * kHcStreams * (R / 64), i3 = (size_t)rpc3 * 2 * (H / 64),
                     i4 = (size_t)rpc2 * (I / 64);
        items = items > i2 ? items : i2;
        items = items > i3 ? items : i3;
        items = items > i4 ? items : i4;
        items = items > extra_items ? items : extra_items;
        const int xmax = R > H ? (R > I ? R : I) : (H > I ? H : I);
        normed = 0;
        sx = al128((size_t)W * 2);
        sv = sx + al128((size_t)xmax * 2);
        spart = sv + al128(items * 8);
        total = spart + al128((size_t)(kHcStreams * 32 > H / 64 ? kHcStreams * 32 : H / 64) * 8);
    }
};

// One CTA's view of the phases. Rows are owned round-robin: CTA j takes rows j, j + G, ...
// of every phase's matrix (and hidden indices j, j + G, ... of the mixer's tail).
template <bool kFp16>
struct F3Phases {
    using G8 = GroupItem<8, 64, kFp16>;
    using G4 = GroupItem<4, 64, kFp16>;

    int H, R, I, W, G, j, tid, lane, warp;
    int ng1, ng2, ng3, ng4;
    int nh, ni, ngate;       // hidden indices (mixer tail, shared down rows), shared gate/up rows, gate groups
    F3Bufs b;
    uint16_t *normed, *sx;   // shared: the normed streams [4H]; staged inputs
    double *sv, *spart;      // shared: group values; the norm's warp sums / the gate's group values
    float *srs;              // shared: per-stream 1 / rms, then the expert gate's sigmoid
    G8 pf1, pf2;             // first items of the mixer down / up phases, loaded ahead
    G4 pf3, pf4;             // first items of the shared gate/up / down phases

    // normed_ / sx_ / sv_ / spart_: shared buffers sized as F3Smem's; srs_: 4 floats
    MOE_D F3Phases(int H_, int R_, int I_, const F3Bufs &b_, unsigned char *normed_, unsigned char *sx_,
                   unsigned char *sv_, unsigned char *spart_, float *srs_)
        : H(H_), R(R_), I(I_), W(kHcStreams * H_), G(gridDim.x), j(blockIdx.x), tid(threadIdx.x),
          lane(threadIdx.x & 31), warp(threadIdx.x >> 5), b(b_) {
        ng1 = W / 64, ng2 = R / 64, ng3 = H / 64, ng4 = I / 64;
        nh = H > j ? (H - 1 - j) / G + 1 : 0;
        ni = I > j ? (I - 1 - j) / G + 1 : 0;
        // the scalar expert gate's groups: group g on CTA G - 1 - (g mod G), whose row items leave room
        ngate = ng3 > G - 1 - j ? (ng3 - 1 - (G - 1 - j)) / G + 1 : 0;
        normed = reinterpret_cast<uint16_t *>(normed_);
        sx = reinterpret_cast<uint16_t *>(sx_);
        sv = reinterpret_cast<double *>(sv_);
        spart = reinterpret_cast<double *>(spart_);
        srs = srs_;
    }

    // ---- item loaders (weights only: they never depend on an earlier phase)
    MOE_D int nrows1(const moe_f3_layer &Ly) const {
        const int N1 = R + (Ly.wi ? kHcStreams : 0);
        return N1 > j ? (N1 - 1 - j) / G + 1 : 0;
    }
    MOE_D void load1(const moe_f3_layer &Ly, int it, G8 &gi) const {
        const int k = it / ng1, g = it - k * ng1, row = j + k * G;
        const bool inj = row >= R;
        const int rr = inj ? row - R : row;
        gi.load(u32(inj ? Ly.wi : Ly.wd) + (size_t)rr * (W / 4), u16(inj ? Ly.si : Ly.sd) + (size_t)rr * ng1,
                u16(inj ? Ly.bi : Ly.bd) + (size_t)rr * ng1, g);
    }
    MOE_D void load2(const moe_f3_layer &Ly, int it, G8 &gi) const {
        const int per = kHcStreams * ng2;
        const int k = it / per, c = (it / ng2) % kHcStreams, g = it % ng2;
        const size_t row = (size_t)c * H + (j + k * G);
        gi.load(u32(Ly.wu) + row * (R / 4), u16(Ly.su) + row * ng2, u16(Ly.bu) + row * ng2, g);
    }
    MOE_D void load3(const moe_f3_layer &Ly, int it, G4 &gi) const {
        const int per = 2 * ng3;
        const int k = it / per, m = (it / ng3) & 1, g = it % ng3;
        const size_t row = (size_t)(j + k * G);
        gi.load(u32(m ? Ly.wsu : Ly.wsg) + row * (H / 8), u16(m ? Ly.ssu : Ly.ssg) + row * ng3,
                u16(m ? Ly.bsu : Ly.bsg) + row * ng3, g);
    }
    // shared down item it of the rows row0 + it / ng4 (row0 = j, step G: the round-robin rows)
    MOE_D void load4(const moe_f3_layer &Ly, int it, G4 &gi, int row0, int step) const {
        const int k = it / ng4, g = it - k * ng4;
        const size_t row = (size_t)(row0 + k * step);
        gi.load(u32(Ly.wsd) + row * (I / 8), u16(Ly.ssd) + row * ng4, u16(Ly.bsd) + row * ng4, g);
    }

    MOE_D void prefetch_mixer_down(const moe_f3_layer &Ly) {
        if (tid < nrows1(Ly) * ng1) load1(Ly, tid, pf1);
    }

    // P0a: the write (stream c of the state gets bf16(branch * gate_c) added) and the sums of
    // the per-stream RMS norm, split as hc_norm_kernel's tree: virtual thread v (of 1024) sums its
    // values v, v + 1024, ... in order, a xor-shuffle tree per 32 virtual threads. CTA 32 c + w
    // (w < 32) takes virtual warp w of stream c: it stores the written values of its elements as
    // the next state and the warp's sum.                            -> grid barrier
    MOE_D void write_and_sums(const uint16_t *hin, const uint16_t *br, const uint16_t *gt, uint16_t *wout) {
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
            if (lane == 0) b.ssum[c * 32 + w] = ss;
        }
    }

    // P0b (every CTA): the 32 warp sums of each stream in order, and the normed values of all
    // four streams into shared memory (all loads of a thread issued together)
    MOE_D void norm(const moe_f3_layer &Ly, const uint16_t *wout, float eps) {
        if (tid < kHcStreams * 32) spart[tid] = __ldcg(b.ssum + tid);
        const uint16_t *nw = u16(Ly.norm_w);
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
            srs[tid] = (float)(1.0 / sqrt(tot / H + (double)eps));
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

    // P1: mixer down (R rows) and inject (4 rows) over the 4H normed values, one thread per
    // (row, group) item, row totals in group order (float totals)         -> grid barrier
    MOE_D void mixer_down(const moe_f3_layer &Ly) {
        const int nrows = nrows1(Ly);
        for (int it = tid; it < nrows * ng1; it += kF3Threads) {
            if (it != tid) load1(Ly, it, pf1);
            sv[it] = pf1.value(normed + (size_t)(it % ng1) * 64);
        }
        if (tid < nh * kHcStreams * ng2) load2(Ly, tid, pf2);
        __syncthreads();
        for (int q = tid; q < nrows; q += kF3Threads) {
            const int row = j + q * G;
            const float tot = (float)sum_in_order(sv + (size_t)q * ng1, ng1);
            if (row < R) b.dv[row] = tot;
            else b.iv[row - R] = tot;
        }
    }

    // P2: mix = silu(down / 4) of all R totals (every CTA), mixer up for the hidden indices
    // this CTA owns (their four stream rows), mixed = mean_c sigmoid(up_c) * normed_c; CTA 0
    // forms inj = 2 sigmoid(inject / 4). own_mixed (shared, nh floats) receives this CTA's
    // mixed values (bf16-rounded) when given; prefetch_gate_up: load the first shared gate /
    // up item (P3).                                                      -> grid barrier
    MOE_D void mixer_up(const moe_f3_layer &Ly, uint16_t *injo, float *own_mixed, bool prefetch_gate_up = true) {
        for (int k = tid; k < R; k += kF3Threads) sx[k] = f32_to_bf16_bits(hc_mix_value(__ldcg(b.dv + k), 0));
        if (j == 0 && tid < kHcStreams) injo[tid] = f32_to_bf16_bits(Ly.wi ? hc_inj_value(__ldcg(b.iv + tid), 0) : 0.f);
        __syncthreads();
        for (int it = tid; it < nh * kHcStreams * ng2; it += kF3Threads) {
            if (it != tid) load2(Ly, it, pf2);
            sv[it] = pf2.value(sx + (size_t)(it % ng2) * 64);
        }
        if (prefetch_gate_up && tid < ni * 2 * ng3) load3(Ly, tid, pf3);
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
            const uint16_t mv = f32_to_bf16_bits(__fdiv_rn(acc, (float)kHcStreams));
            b.mixed[hh] = mv;
            if (own_mixed) own_mixed[q] = bf16_bits_to_f32(mv);
        }
    }

    // P3: shared gate + up rows this CTA owns, SwiGLU with MLX's bf16 roundings; the scalar
    // expert gate's group values (8-bit g64) on the CTAs with the fewest rows. mixed must be
    // staged in sx. prefetched: mixer_up loaded the first item; prefetch_down: load the first
    // round-robin shared down item (P4).                                  -> grid barrier
    MOE_D void shared_gate_up(const moe_f3_layer &Ly, bool prefetch_down, bool prefetched = true) {
        const int per = 2 * ng3;
        for (int it = tid; it < ni * per; it += kF3Threads) {
            if (it != tid || !prefetched) load3(Ly, it, pf3);
            sv[it] = pf3.value(sx + (size_t)(it % ng3) * 64);
        }
        for (int q = tid; q < ngate; q += kF3Threads) {
            const int g = (G - 1 - j) + q * G;
            G8 gi;
            gi.load(u32(Ly.wse), u16(Ly.sse), u16(Ly.bse), g);
            b.gsum[g] = gi.value(sx + (size_t)g * 64);
        }
        if (prefetch_down && tid < nh * ng4) load4(Ly, tid, pf4, j, G);
        __syncthreads();
        for (int q = tid; q < ni; q += kF3Threads) {
            const int i = j + q * G;
            const float gv = bf16_bits_to_f32(row_out(sum_in_order(sv + (size_t)(q * 2) * ng3, ng3)));
            const float uv = bf16_bits_to_f32(row_out(sum_in_order(sv + (size_t)(q * 2 + 1) * ng3, ng3)));
            b.act[i] = f32_to_bf16_bits(bf16r(__fmul_rn(bf16r(__fmul_rn(gv, sigmoid_bf16(gv))), uv)));
        }
    }

    // P4 prologue: the shared SwiGLU staged in sx and the expert gate's sigmoid (its group
    // values summed in order); returns bf16(sigmoid(gate))
    MOE_D float stage_down(void) {
        stage_l2(sx, b.act, I);
        if (tid < ng3) spart[tid] = __ldcg(b.gsum + tid);
        __syncthreads();
        if (tid == 0) srs[0] = sigmoid_bf16(bf16_bits_to_f32(row_out(sum_in_order(spart, ng3))));
        __syncthreads();
        return srs[0];
    }

    // P4 items: the group values of shared down rows row0, row0 + step, ... (nrows of them) into
    // sv[row index * ng4 + group]; the first item of each thread may have been prefetched (pf4)
    MOE_D void shared_down_items(const moe_f3_layer &Ly, int row0, int step, int nrows, bool prefetched) {
        for (int it = tid; it < nrows * ng4; it += kF3Threads) {
            if (it != tid || !prefetched) load4(Ly, it, pf4, row0, step);
            sv[it] = pf4.value(sx + (size_t)(it % ng4) * 64);
        }
    }

    // the shared expert's output of row index q (after shared_down_items and a block barrier)
    MOE_D uint16_t shared_down_out(int q, float gsig) const {
        const uint16_t o = row_out(sum_in_order(sv + (size_t)q * ng4, ng4));
        return f32_to_bf16_bits(__fmul_rn(gsig, bf16_bits_to_f32(o)));
    }
};

}  // namespace moe_f3
