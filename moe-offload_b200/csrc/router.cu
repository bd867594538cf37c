// Router: gate GEMV (exact double accumulation, one bf16 rounding) fused with the
// precise softmax, MLX-order top-k, renormalisation and the optional next-layer top-M
// prediction. One launch per layer step:
//
//   grid (ceil(R / 8), T), 256 threads; R = E rows of this layer's router plus, when a
//   prediction is requested, E rows of the next layer's router (same input x, the way
//   loader.py:950-958 evaluates inds and pred_next in one sync). Each warp produces one
//   logit; the last CTA to finish a token (atomic ticket in the workspace) runs the
//   softmax / selection tail for that token and re-arms the ticket.
//
// For batches of 256 tokens or more (bf16 router, no fused normalisation / records) the GEMV
// becomes a tiled double-precision GEMM plus one softmax / selection block per token (at the
// c3 shape the GEMM takes ~0.3 ms for 256 .. 2048 tokens; the per-token kernel 0.3 ms at 256
// tokens and 1.16 ms at 1023).
//
// Reference semantics: mlx-qwen38/loader.py:903-908 (router), loader.py:237-242
// (topk_sorted_indices); cpp/src/layers.cpp:311-341.
#include "common.cuh"
#include "gemv_i8.cuh"
#include "topk.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxE = 2048;              // experts per layer supported by the tail

struct RouterArgs {
    const uint16_t *x;
    int T, H, E, K, M, gs;
    const void *w;
    const uint16_t *ws, *wb;
    const void *wn;
    const uint16_t *wns, *wnb;
    const float *pred_bias;
    uint16_t *logits;     // [T, E]
    uint16_t *plogits;    // [T, E] (prediction rows), may be null when M == 0
    uint16_t *probs;      // [T, E] or null
    uint32_t *inds;       // [T, K]
    uint16_t *scores;     // [T, K]
    uint32_t *pred;       // [T, M] or null
    unsigned int *tickets;  // [T], zero between launches
    uint2 *xrec;          // [T, H/64, 16] int8 MMA records of x (gemv_i8.cuh), or null
    float *xscale, *xsum; // [T, pad4(H/64)] each
    int norm;             // 1: the router input is x * 2^-k (pow2_rms_shift of x), else x
};

// ---------------------------------------------------------------- row dot products

// bf16 weights: lanes stride over 16-byte chunks (8 values). A bf16 x bf16 product is exact
// in fp32 (16 significant bits), so each product is formed in fp32 and accumulated in double.
constexpr int kPre = 16;              // chunks per lane held in registers (H <= 4096)

MOE_D void preload_row_bf16(const uint16_t *__restrict__ w, int H, int lane, uint4 (&wv)[kPre]) {
    const int nchunk = H >> 3;
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
        const int c = lane + 32 * j;
        wv[j] = (c < nchunk) ? ldg_stream16(w + 8 * c) : make_uint4(0, 0, 0, 0);
    }
}

MOE_D double dot8_bf16(uint4 xv, uint4 wv, double acc) {
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t ws[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        acc += (double)(__uint_as_float(xs[q] << 16) * __uint_as_float(ws[q] << 16));
        acc += (double)(__uint_as_float(xs[q] & 0xffff0000u) * __uint_as_float(ws[q] & 0xffff0000u));
    }
    return acc;
}

MOE_D double row_dot_bf16(const uint16_t *__restrict__ x, const uint16_t *__restrict__ w, int H, int lane,
                          const uint4 (&wv)[kPre]) {
    const int nchunk = H >> 3;
    double acc[4] = {0.0, 0.0, 0.0, 0.0};        // independent chains
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunk) acc[j & 3] = dot8_bf16(__ldg(reinterpret_cast<const uint4 *>(x) + c), wv[j], acc[j & 3]);
    }
    for (int c = lane + 32 * kPre; c < nchunk; c += 32)   // H > 4096
        acc[0] = dot8_bf16(__ldg(reinterpret_cast<const uint4 *>(x) + c), ldg_stream16(w + 8 * c), acc[0]);
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// affine-quantised weights (MLX layout), any bits in {2,4,8}: per 64-code group
// s * sum(q x) + b * sum(x), every term exact or double-rounded.
template <bool kFp16>
MOE_D double row_dot_affine(const uint16_t *__restrict__ x, const uint32_t *__restrict__ w,
                            const uint16_t *__restrict__ s, const uint16_t *__restrict__ b, int H,
                            int bits, int gs, int lane) {
    const int per = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int ngroups = H / gs;
    double acc = 0.0;
    for (int G = lane; G < ngroups; G += 32) {
        double dq = 0.0, dx = 0.0;
        for (int j = 0; j < gs; ++j) {
            const int h = G * gs + j;
            const double xv = (double)bf16_bits_to_f32(x[h]);
            const uint32_t q = (__ldg(w + h / per) >> ((h % per) * bits)) & mask;
            dq = fma((double)q, xv, dq);
            dx += xv;
        }
        acc += (double)sb_to_f32<kFp16>(s[G]) * dq + (double)sb_to_f32<kFp16>(b[G]) * dx;
    }
    return acc;
}

MOE_D double warp_sum_d(double v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// order-preserving 16-bit key of a bf16 value
MOE_D uint32_t bf16_order_key(uint16_t v) {
    return (v & 0x8000) ? (uint32_t)(~v & 0xffff) : (uint32_t)(v | 0x8000);
}

// Softmax (double, fixed reduction order), bf16 probabilities, MLX-order top-k, renorm and the
// optional sorted top-M prediction of token t, from its bf16 logits (whole block).
MOE_D void router_tail(const RouterArgs &a, int t) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    __shared__ uint32_t s_keys[kMaxE];
    __shared__ double s_ex[kMaxE];
    __shared__ float s_red[kWarps];
    __shared__ double s_redd[kWarps];
    __shared__ uint32_t s_sel[64];
    const int E = a.E;
    const uint16_t *lg = a.logits + (size_t)t * E;

    // max of the bf16 logits
    float mx = -INFINITY;
    for (int e = threadIdx.x; e < E; e += kThreads) {
        const float v = bf16_bits_to_f32(__ldcg(lg + e));
        s_ex[e] = (double)v;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
#pragma unroll
    for (int i = 1; i < kWarps; ++i) mx = fmaxf(mx, s_red[i]);

    // sum of exp in double (fixed reduction order -> deterministic)
    double sum = 0.0;
    for (int e = threadIdx.x; e < E; e += kThreads) {
        const double ev = exp(s_ex[e] - (double)mx);
        s_ex[e] = ev;
        sum += ev;
    }
    sum = warp_sum_d(sum);
    if (lane == 0) s_redd[warp] = sum;
    __syncthreads();
    sum = 0.0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) sum += s_redd[i];

    // bf16 probabilities and selection keys ((p << 16) | e) + 1, all distinct and > 0
    for (int e = threadIdx.x; e < E; e += kThreads) {
        const uint16_t p = f64_to_bf16_bits(s_ex[e] / sum);
        if (a.probs) a.probs[(size_t)t * E + e] = p;
        s_keys[e] = (((uint32_t)p << 16) | (uint32_t)e) + 1u;
    }
    __syncthreads();

    if (warp == 0) {
        warp_select_desc(s_keys, E, a.K, s_sel);
        if (lane == 0) {
            // MLX order: ascending (p, index)
            float S = 0.f;
            for (int k = 0; k < a.K; ++k) {
                const uint32_t key = s_sel[a.K - 1 - k] - 1u;
                const float p = bf16_bits_to_f32((uint16_t)(key >> 16));
                S = (k == 0) ? p : bf16r(S + p);
            }
            for (int k = 0; k < a.K; ++k) {
                const uint32_t key = s_sel[a.K - 1 - k] - 1u;
                a.inds[(size_t)t * a.K + k] = key & 0xffffu;
                const float p = bf16_bits_to_f32((uint16_t)(key >> 16));
                a.scores[(size_t)t * a.K + k] = f32_to_bf16_bits(__fdiv_rn(p, S));
            }
        }
    }
    __syncthreads();

    if (a.M > 0) {
        const uint16_t *pl = a.plogits + (size_t)t * E;
        for (int e = threadIdx.x; e < E; e += kThreads)
            s_keys[e] = ((bf16_order_key(__ldcg(pl + e)) << 16) | (uint32_t)e) + 1u;
        __syncthreads();
        if (warp == 0) {
            warp_select_desc(s_keys, E, a.M, s_sel);
            if (lane == 0) {
                // descending value; equal values in ascending index order
                int o = 0, i = 0;
                while (i < a.M) {
                    const uint32_t v = (s_sel[i] - 1u) >> 16;
                    int j = i;
                    while (j + 1 < a.M && ((s_sel[j + 1] - 1u) >> 16) == v) ++j;
                    for (int q = j; q >= i; --q) a.pred[(size_t)t * a.M + o++] = (s_sel[q] - 1u) & 0xffffu;
                    i = j + 1;
                }
            }
        }
    }
}

template <bool kFp16, int kRbits>
__global__ void __launch_bounds__(kThreads) router_kernel(RouterArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.y;
    const int rows = a.E * (a.M > 0 ? 2 : 1);
    const int row = blockIdx.x * kWarps + warp;
    const uint16_t *x = a.x + (size_t)t * a.H;

    const bool next = row >= a.E;
    const int e = next ? row - a.E : row;
    uint4 wv[kPre];
    if constexpr (kRbits == 16) {
        if (row < rows) {
            const uint16_t *w = reinterpret_cast<const uint16_t *>(next ? a.wn : a.w) + (size_t)e * a.H;
            preload_row_bf16(w, a.H, lane, wv);   // weights do not depend on earlier kernels
        }
    }
    pdl_wait();                                   // x is complete
    pdl_launch_dependents();

    // optional power-of-two RMS normalisation of the layer input (exact rescale)
    double xmul = 1.0;
    if (a.norm) {
        __shared__ double s_ss[kWarps];
        double ss = 0.0;
        for (int i = threadIdx.x; i < a.H; i += kThreads) {
            const double v = (double)bf16_bits_to_f32(x[i]);
            ss = fma(v, v, ss);
        }
        ss = warp_sum_d(ss);
        if (lane == 0) s_ss[warp] = ss;
        __syncthreads();
        ss = 0.0;
#pragma unroll
        for (int i = 0; i < kWarps; ++i) ss += s_ss[i];
        xmul = ldexp(1.0, -pow2_rms_shift(ss, a.H));
    }

    if (a.xrec) {
        // int8 MMA records of x for the expert kernels (gemv_i8.cuh): 16 threads per group
        const int ng = a.H >> 6;
        for (int G0 = blockIdx.x * (kThreads / 16); G0 < ng; G0 += gridDim.x * (kThreads / 16)) {
            const int G = G0 + (threadIdx.x >> 4);
            const bool v = G < ng;
            const size_t fo = (size_t)t * pad4(ng) + G;
            build_rec_group(x + (size_t)(v ? G : 0) * 64, v, threadIdx.x & 15, a.xrec + ((size_t)t * ng + G) * 16,
                            a.xscale + fo, a.xsum + fo, (float)xmul);
        }
    }

    if (row < rows) {
        double acc;
        if constexpr (kRbits == 16) {
            const uint16_t *w = reinterpret_cast<const uint16_t *>(next ? a.wn : a.w) + (size_t)e * a.H;
            acc = row_dot_bf16(x, w, a.H, lane, wv);
        } else {
            const int words = a.H * kRbits / 32, ng = a.H / a.gs;
            const uint32_t *w = reinterpret_cast<const uint32_t *>(next ? a.wn : a.w) + (size_t)e * words;
            const uint16_t *s = (next ? a.wns : a.ws) + (size_t)e * ng;
            const uint16_t *b = (next ? a.wnb : a.wb) + (size_t)e * ng;
            acc = row_dot_affine<kFp16>(x, w, s, b, a.H, kRbits, a.gs, lane);
        }
        acc = warp_sum_d(acc) * xmul;
        if (lane == 0) {
            uint16_t l = f64_to_bf16_bits(acc);
            if (next) {
                if (a.pred_bias) l = f32_to_bf16_bits(bf16_bits_to_f32(l) + a.pred_bias[e]);
                a.plogits[(size_t)t * a.E + e] = l;
            } else {
                a.logits[(size_t)t * a.E + e] = l;
            }
        }
    }

    // ------------------------------------------------------------ last CTA of token t
    __shared__ unsigned int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int prev = atomicAdd(a.tickets + t, 1u);
        s_last = (prev == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    router_tail(a, t);
    if (threadIdx.x == 0) a.tickets[t] = 0u;   // re-arm for the next launch
}

// ---------------------------------------------------------------- batched path (T >= 256)
//
// For many tokens the router is a GEMM: logits[T][E] = x . W^T. Tiles of 64 tokens x 128
// rows per CTA on the fp64 tensor cores (mma.sync m8n8k4 .f64); the operands are converted
// exactly to double once when staged in shared memory, so each term is an exact product and
// the sum is a double sum (the same arithmetic as the per-token kernel, in another order:
// the bf16 rounding of the result differs only for a value within ~2^-45 of a rounding
// midpoint). Then one block per token runs router_tail.
constexpr int kGT = 64, kGE = 128, kGK = 32;      // tokens, rows, K per stage
constexpr int kGemmMinT = 256;                     // batches from this size use the GEMM
constexpr size_t kGemmStage = (size_t)kGK * (kGT + kGE);            // doubles per stage
constexpr size_t kGemmSmem = 2 * kGemmStage * sizeof(double);      // two stages

// fp64 tensor-core MMA: D(8x8) += A(8x4, row) * B(4x8, col); lane (g = lane >> 2, q = lane & 3)
// holds A[g][q], B[q][g] and D[g][2q], D[g][2q+1]
__device__ __forceinline__ void dmma_884(double &d0, double &d1, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                 : "+d"(d0), "+d"(d1)
                 : "d"(a), "d"(b));
}

// Tile: 64 tokens x 128 router rows per CTA, K in stages of 32. Operands are converted exactly
// to double when staged, as [k-block of 4][token or row][4] so that every fragment load of a
// warp touches each bank pair exactly twice (conflict-free), into one of two stage buffers:
// one block barrier per stage (stage s+1 is written while another warp may still read stage s;
// nobody writes stage s+2 = s before every warp has passed the barrier after stage s+1's
// writes). Warp w computes tokens (w & 1) * 32 .. +32 and rows (w >> 1) * 32 .. +32 as 4 x 4
// tiles of fp64 MMAs: exact products of bf16 values summed in double, as in the per-token kernel.
__global__ void __launch_bounds__(256) router_gemm_kernel(RouterArgs a) {
    extern __shared__ double gsm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int t0 = blockIdx.y * kGT, r0 = blockIdx.x * kGE;
    const int wt0 = (warp & 1) * 32, wr0 = (warp >> 1) * 32;
    const int rows = a.E * (a.M > 0 ? 2 : 1);
    const uint16_t *w = static_cast<const uint16_t *>(a.w);
    const uint16_t *wn = static_cast<const uint16_t *>(a.wn);
    pdl_wait();
    pdl_launch_dependents();
    double acc[4][4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;
    // global -> registers for stage k0 (x: 8 values of one token, w: 8 values of two rows per
    // thread), issued one stage ahead so the loads overlap the previous stage's MMAs
    const int ltok = tid >> 2, lrow = tid >> 2, lc = (tid & 3) * 8;
    auto load_stage = [&](int k0, uint4 &vx, uint4 (&vw)[2]) {
        const int gt = t0 + ltok;
        vx = make_uint4(0u, 0u, 0u, 0u);
        if (gt < a.T && k0 + lc < a.H) vx = *reinterpret_cast<const uint4 *>(a.x + (size_t)gt * a.H + k0 + lc);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int gr = r0 + lrow + 64 * hh;
            vw[hh] = make_uint4(0u, 0u, 0u, 0u);
            if (gr < rows && k0 + lc < a.H) {
                const uint16_t *src = (gr < a.E) ? w + (size_t)gr * a.H : wn + (size_t)(gr - a.E) * a.H;
                vw[hh] = *reinterpret_cast<const uint4 *>(src + k0 + lc);
            }
        }
    };
    // 8 bf16 values (k = lc .. lc + 7) -> two [4] groups of doubles at k-blocks lc/4, lc/4 + 1
    auto stage_vals = [&](double *base, int nrow, int row, const uint4 &v) {
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            double *d = base + ((size_t)((lc >> 2) + h) * nrow + row) * 4;
            d[0] = (double)__uint_as_float(vv[2 * h] << 16);
            d[1] = (double)__uint_as_float(vv[2 * h] & 0xffff0000u);
            d[2] = (double)__uint_as_float(vv[2 * h + 1] << 16);
            d[3] = (double)__uint_as_float(vv[2 * h + 1] & 0xffff0000u);
        }
    };
    uint4 nx, nw[2];
    load_stage(0, nx, nw);
    for (int k0 = 0, sb = 0; k0 < a.H; k0 += kGK, sb ^= 1) {
        double *xs = gsm + sb * kGemmStage;     // [kGK / 4][kGT][4]
        double *ws = xs + kGK * kGT;            // [kGK / 4][kGE][4]
        stage_vals(xs, kGT, ltok, nx);
        stage_vals(ws, kGE, lrow, nw[0]);
        stage_vals(ws, kGE, lrow + 64, nw[1]);
        if (k0 + kGK < a.H) load_stage(k0 + kGK, nx, nw);
        __syncthreads();
#pragma unroll 2
        for (int kb = 0; kb < kGK / 4; ++kb) {
            double af[4], bfr[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) af[i] = xs[((size_t)kb * kGT + wt0 + i * 8 + g) * 4 + q];
#pragma unroll
            for (int j = 0; j < 4; ++j) bfr[j] = ws[((size_t)kb * kGE + wr0 + j * 8 + g) * 4 + q];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_884(acc[i][j][0], acc[i][j][1], af[i], bfr[j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gt = t0 + wt0 + i * 8 + g;
        if (gt >= a.T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int gr = r0 + wr0 + j * 8 + 2 * q + h;
                if (gr >= rows) continue;
                uint16_t l = f64_to_bf16_bits(acc[i][j][h]);
                if (gr >= a.E) {
                    if (a.pred_bias) l = f32_to_bf16_bits(bf16_bits_to_f32(l) + a.pred_bias[gr - a.E]);
                    a.plogits[(size_t)gt * a.E + gr - a.E] = l;
                } else {
                    a.logits[(size_t)gt * a.E + gr] = l;
                }
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) router_select_kernel(RouterArgs a) {
    pdl_wait();
    pdl_launch_dependents();
    router_tail(a, blockIdx.x);
}

template <bool kFp16>
cudaError_t launch_router(const RouterArgs &a, int rbits, cudaStream_t st) {
    // the tiled GEMM pays from a few tiles of 64 tokens x 128 rows on; smaller batches keep one
    // warp per (row, token)
    if (rbits == 16 && a.T >= kGemmMinT && !a.xrec && !a.norm && (a.H % 8) == 0) {
        const int rows = a.E * (a.M > 0 ? 2 : 1);
        dim3 grid((rows + kGE - 1) / kGE, (a.T + kGT - 1) / kGT);
        cudaError_t e = launch_pdl(router_gemm_kernel, grid, dim3(256), kGemmSmem, st, a);
        if (e != cudaSuccess) return e;
        return launch_pdl(router_select_kernel, dim3(a.T), dim3(kThreads), 0, st, a);
    }
    const int rows = a.E * (a.M > 0 ? 2 : 1);
    dim3 grid((rows + kWarps - 1) / kWarps, a.T);
    switch (rbits) {
        case 16: return launch_pdl(router_kernel<kFp16, 16>, grid, dim3(kThreads), 0, st, a);
        case 8: return launch_pdl(router_kernel<kFp16, 8>, grid, dim3(kThreads), 0, st, a);
        case 4: return launch_pdl(router_kernel<kFp16, 4>, grid, dim3(kThreads), 0, st, a);
        case 2: return launch_pdl(router_kernel<kFp16, 2>, grid, dim3(kThreads), 0, st, a);
        default: return cudaErrorInvalidValue;
    }
}


inline size_t al_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

extern "C" size_t moe_router_workspace_bytes(int T, int E, int M) {
    if (T <= 0 || E <= 0) return 0;
    size_t b = al_up((size_t)T * sizeof(unsigned int), 256);        // tickets
    b += al_up((size_t)T * E * sizeof(uint16_t), 256);               // logits
    if (M > 0) b += al_up((size_t)T * E * sizeof(uint16_t), 256);    // prediction logits
    return b;
}

// Validates arguments and launches with the given ticket/logit buffers; shared by the
// workspace entry point and any caller that supplies its own scratch.
int moe_router_launch(const void *x, int T, int H, int E, int K, const void *w,
                      const void *w_scales, const void *w_biases, int rbits, int group_size,
                      int sb_fp16, const void *wn, const void *wn_scales, const void *wn_biases,
                      int M, const float *pred_bias, void *out_logits, void *out_probs,
                      uint32_t *out_inds, void *out_scores, uint32_t *out_pred,
                      unsigned int *tickets, uint16_t *logits_buf, uint16_t *plogits_buf,
                      void *xrec, float *xscale, float *xsum, int norm, void *stream) {
    if (!x || !w || !out_inds || !out_scores || !tickets)
        return moe_set_error(MOE_EINVAL, "router: null required pointer");
    if (T <= 0 || H <= 0 || E <= 0 || E > kMaxE || K <= 0 || K > E || K > 64)
        return moe_set_error(MOE_EINVAL, "router: bad sizes T=%d H=%d E=%d K=%d", T, H, E, K);
    if (M < 0 || M > E || M > 64 || (M > 0 && (!wn || !out_pred)))
        return moe_set_error(MOE_EINVAL, "router: bad prediction arguments M=%d", M);
    if (rbits == 16) {
        if (H % 8) return moe_set_error(MOE_EINVAL, "router: H=%d must be a multiple of 8", H);
        // both routers are read in one format: an affine next-layer router (scales / biases
        // given) behind a bf16 one would be read as bf16 past its codes
        if (M > 0 && (wn_scales || wn_biases))
            return moe_set_error(MOE_EINVAL, "router: the next-layer router must have this router's format");
        if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
             reinterpret_cast<uintptr_t>(wn)) & 15)
            return moe_set_error(MOE_EINVAL, "router: x/w must be 16-byte aligned");
    } else if (rbits == 8 || rbits == 4 || rbits == 2) {
        if (group_size <= 0 || H % group_size || group_size % (32 / rbits))
            return moe_set_error(MOE_EINVAL, "router: bad group_size %d", group_size);
        if (!w_scales || !w_biases || (M > 0 && (!wn_scales || !wn_biases)))
            return moe_set_error(MOE_EINVAL, "router: affine router needs scales and biases");
    } else {
        return moe_set_error(MOE_EINVAL, "router: rbits=%d unsupported", rbits);
    }
    RouterArgs a{};
    a.x = static_cast<const uint16_t *>(x);
    a.T = T; a.H = H; a.E = E; a.K = K; a.M = M; a.gs = group_size;
    a.w = w; a.ws = static_cast<const uint16_t *>(w_scales); a.wb = static_cast<const uint16_t *>(w_biases);
    a.wn = wn; a.wns = static_cast<const uint16_t *>(wn_scales); a.wnb = static_cast<const uint16_t *>(wn_biases);
    a.pred_bias = pred_bias;
    a.logits = out_logits ? static_cast<uint16_t *>(out_logits) : logits_buf;
    a.plogits = plogits_buf;
    a.probs = static_cast<uint16_t *>(out_probs);
    a.inds = out_inds;
    a.scores = static_cast<uint16_t *>(out_scores);
    a.pred = out_pred;
    a.tickets = tickets;
    a.xrec = static_cast<uint2 *>(xrec);
    a.xscale = xscale;
    a.xsum = xsum;
    a.norm = norm;
    if (xrec && (H % 64 || !xscale || !xsum))
        return moe_set_error(MOE_EINVAL, "router: x records need H %% 64 == 0 and scale/sum buffers");
    if (!a.logits || (M > 0 && !a.plogits))
        return moe_set_error(MOE_EINVAL, "router: missing logit scratch");
    cudaError_t e = sb_fp16 ? launch_router<true>(a, rbits, as_stream(stream))
                            : launch_router<false>(a, rbits, as_stream(stream));
    if (e != cudaSuccess) return moe_set_cuda_error(e);
    return MOE_OK;
}

extern "C" int moe_router_topk(const void *x, int T, int H, int E, int K, const void *w,
                               const void *w_scales, const void *w_biases, int rbits,
                               int group_size, int sb_fp16, const void *wn, const void *wn_scales,
                               const void *wn_biases, int M, const float *pred_bias,
                               void *out_logits, void *out_probs, uint32_t *out_inds,
                               void *out_scores, uint32_t *out_pred, void *workspace,
                               size_t workspace_bytes, void *stream) {
    if (T <= 0 || E <= 0) return moe_set_error(MOE_EINVAL, "router: bad sizes T=%d E=%d", T, E);
    const size_t need = moe_router_workspace_bytes(T, E, M);
    if (!workspace || workspace_bytes < need)
        return moe_set_error(MOE_EINVAL, "router: workspace of %zu bytes needed, %zu given", need,
                             workspace_bytes);
    char *ws = static_cast<char *>(workspace);
    unsigned int *tickets = reinterpret_cast<unsigned int *>(ws);
    ws += al_up((size_t)T * sizeof(unsigned int), 256);
    uint16_t *logits = reinterpret_cast<uint16_t *>(ws);
    ws += al_up((size_t)T * E * sizeof(uint16_t), 256);
    uint16_t *plogits = M > 0 ? reinterpret_cast<uint16_t *>(ws) : nullptr;
    return moe_router_launch(x, T, H, E, K, w, w_scales, w_biases, rbits, group_size, sb_fp16, wn,
                             wn_scales, wn_biases, M, pred_bias, out_logits, out_probs, out_inds,
                             out_scores, out_pred, tickets, logits, plogits, nullptr, nullptr, nullptr, 0,
                             stream);
}
