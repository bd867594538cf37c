/*
 * moe_oracle.c -- CPU restatement of the routed-expert MoE block (TEST INFRASTRUCTURE ONLY).
 *
 * This file is the checker for the CUDA path, never the product. Only tests/, the
 * smoke() check in __graft_entry__.py and the cpu_baseline / --impl reference legs of
 * bench.py may load it. The product library (libmoe_b200.so) never links or calls it.
 *
 * What it restates (citations are paths inside the Jakevin/moe-offload project):
 *   - MLX affine dequantisation, `transpose=True` layout: w = scale * q + bias per
 *     `group_size` consecutive inputs, `32/bits` codes per little-endian uint32, code j at
 *     bits [bits*j, bits*j+bits) (the layout loader.py:332-368 allocates and
 *     cpp/src/kernels.cpp:1027-1040 feeds to gather_qmm).
 *   - Router: logits = x . W^T rounded once to bf16 (loader.py:903, cpp/src/layers.cpp:315),
 *     softmax over experts rounded to bf16 (loader.py:904, layers.cpp:316), top-k in MLX
 *     argpartition order (loader.py:906, layers.cpp:317-320), gather + renormalisation
 *     (loader.py:907-908, layers.cpp:321-324).
 *   - Next-layer prediction topk_sorted_indices (loader.py:237-242, layers.cpp:327-341).
 *   - SwitchGLU expert math: up/gate gather_qmm, SwiGLU, down gather_qmm
 *     (layers.cpp:343-362, kernels.cpp:1090-1094) and the routing-weighted combine
 *     `(y * scores[..., None]).sum(-2) + shared_y` (loader.py:914,965, layers.cpp:400,599).
 *
 * Arithmetic model (fixed so the CUDA path can be held to it bit-for-bit where the
 * gates demand bit-exactness):
 *   - router dot products are accumulated in double and rounded ONCE to bf16, so the
 *     result does not depend on summation order; softmax is exp/sum/divide in double,
 *     rounded once to bf16;
 *   - top-k order = stable ascending argsort of the bf16 probabilities, last k entries
 *     (ties resolved toward the higher expert index); pinned by the reference fixture
 *     cpp/tests/fixtures.safetensors keys moe.inds_dec / moe.inds_pre;
 *   - renormalisation: S = sequential bf16 sum of the selected probabilities in index
 *     order, score = bf16(float(p) / float(S)); pinned by moe.scores_*;
 *   - expert GEMVs accumulate in float within a 64-group and in double across groups,
 *     outputs rounded to bf16 (gather_qmm returns bf16);
 *   - SwiGLU rounds after every op like an MLX bf16 graph: bf16(bf16(g*bf16(sig(g)))*u);
 *   - combine: prod_k = bf16(y_k * s_k); acc = sequential bf16 sum over k in index
 *     order; then optional bf16 addend (shared expert) and optional bf16 residual.
 *
 * Build: see oracle/Makefile (gcc -O3 -fopenmp -shared -fPIC).
 */
#include <alloca.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------ */
/* scalar conversions                                                                    */
/* ------------------------------------------------------------------------------------ */

static inline float bf16_to_f32(uint16_t h) {
    union { uint32_t u; float f; } v;
    v.u = ((uint32_t)h) << 16;
    return v.f;
}

/* float -> bf16, round to nearest even, NaN kept quiet */
static inline uint16_t f32_to_bf16(float f) {
    union { uint32_t u; float f; } v;
    v.f = f;
    uint32_t u = v.u;
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/* double -> bf16 with a single round-to-nearest-even (no double rounding through float) */
static inline uint16_t f64_to_bf16(double d) {
    if (isnan(d)) return 0x7fc0;
    if (d == 0.0) return signbit(d) ? 0x8000 : 0x0000;
    double a = fabs(d);
    int e;
    frexp(a, &e);                       /* a = m * 2^e, 0.5 <= m < 1 */
    int q = e - 8;                      /* quantum for 8 significant bits */
    if (q < -133) q = -133;             /* bf16 subnormal quantum 2^-133 */
    double scaled = ldexp(a, -q);
    double r = nearbyint(scaled);       /* default rounding mode: nearest-even */
    double res = ldexp(r, q);
    if (res > 3.3895313892515355e38) { /* beyond bf16 max finite -> inf */
        return (uint16_t)(signbit(d) ? 0xff80 : 0x7f80);
    }
    float rf = (float)res;              /* exact: res has <= 8 significant bits */
    uint16_t out = f32_to_bf16(rf);
    return (uint16_t)(signbit(d) ? (out | 0x8000) : out);
}

static inline float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ff;
    union { uint32_t u; float f; } v;
    if (e == 0) {
        float r = ldexpf((float)m, -24);
        return s ? -r : r;
    } else if (e == 31) {
        v.u = s | 0x7f800000u | (m << 13);
        return v.f;
    }
    v.u = s | ((e + 112) << 23) | (m << 13);
    return v.f;
}

static inline float sb_to_f32(uint16_t v, int fp16) { return fp16 ? f16_to_f32(v) : bf16_to_f32(v); }

static inline float bf(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* ------------------------------------------------------------------------------------ */
/* affine dequantised dot products                                                       */
/* ------------------------------------------------------------------------------------ */

/* one row of an affine-quantised matrix dotted with x (float), double result */
static double qdot_row(const uint32_t *w, const uint16_t *s, const uint16_t *b, int sb_fp16,
                       const float *x, int n, int bits, int gs) {
    const int per = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    double total = 0.0;
    for (int g0 = 0; g0 < n; g0 += gs) {
        float acc = 0.f, xs = 0.f;
        for (int j = g0; j < g0 + gs; ++j) {
            uint32_t word = w[j / per];
            float q = (float)((word >> ((j % per) * bits)) & mask);
            acc += q * x[j];
            xs += x[j];
        }
        int g = g0 / gs;
        total += (double)sb_to_f32(s[g], sb_fp16) * (double)acc + (double)sb_to_f32(b[g], sb_fp16) * (double)xs;
    }
    return total;
}

/* exact router row: x (bf16) . w (bf16 or affine) in double */
static double router_row(const uint16_t *x, int H, int rbits, const void *rw, const uint16_t *rs,
                         const uint16_t *rb, int gs, int sb_fp16, int e) {
    double acc = 0.0;
    if (rbits == 16) {
        const uint16_t *w = (const uint16_t *)rw + (size_t)e * H;
        for (int h = 0; h < H; ++h) acc += (double)bf16_to_f32(x[h]) * (double)bf16_to_f32(w[h]);
        return acc;
    }
    const int per = 32 / rbits;
    const uint32_t mask = (1u << rbits) - 1u;
    const uint32_t *w = (const uint32_t *)rw + (size_t)e * (H / per);
    const uint16_t *s = rs + (size_t)e * (H / gs);
    const uint16_t *b = rb + (size_t)e * (H / gs);
    for (int h = 0; h < H; ++h) {
        uint32_t q = (w[h / per] >> ((h % per) * rbits)) & mask;
        double wv = (double)sb_to_f32(s[h / gs], sb_fp16) * (double)q + (double)sb_to_f32(b[h / gs], sb_fp16);
        acc += (double)bf16_to_f32(x[h]) * wv;
    }
    return acc;
}

/* ------------------------------------------------------------------------------------ */
/* router                                                                                */
/* ------------------------------------------------------------------------------------ */

/* logits[t,e] = bf16(sum_h x[t,h] * W[e,h]) (+ optional float bias, rounded again) */
int orc_router_logits(const uint16_t *x, int T, int H, int E, int rbits, const void *rw,
                      const uint16_t *rs, const uint16_t *rb, int gs, int sb_fp16,
                      const float *bias, uint16_t *logits) {
    if (T < 0 || H <= 0 || E <= 0) return -22;
    if (rbits != 16 && rbits != 8 && rbits != 4 && rbits != 2) return -22;
    if (rbits != 16 && (gs <= 0 || H % gs)) return -22;
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e) {
            double v = router_row(x + (size_t)t * H, H, rbits, rw, rs, rb, gs, sb_fp16, e);
            uint16_t l = f64_to_bf16(v);
            if (bias) l = f32_to_bf16(bf16_to_f32(l) + bias[e]);
            logits[(size_t)t * E + e] = l;
        }
    return 0;
}

/* order-preserving 16-bit key of a bf16 value (larger value -> larger key) */
static inline uint32_t bf16_order_key(uint16_t v) {
    return (v & 0x8000) ? (uint32_t)(~v & 0xffff) : (uint32_t)(v | 0x8000);
}

/* softmax (double, one rounding) + top-k in MLX argpartition order + renormalisation */
int orc_softmax_topk(const uint16_t *logits, int T, int E, int K, uint16_t *probs,
                     uint32_t *inds, uint16_t *scores) {
    if (K <= 0 || K > E || E > 65535) return -22;
    uint16_t *p = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)E);
    uint32_t *key = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)E);
    if (!p || !key) { free(p); free(key); return -12; }
    for (int t = 0; t < T; ++t) {
        const uint16_t *l = logits + (size_t)t * E;
        double mx = -INFINITY;
        for (int e = 0; e < E; ++e) { double v = bf16_to_f32(l[e]); if (v > mx) mx = v; }
        double sum = 0.0;
        for (int e = 0; e < E; ++e) sum += exp((double)bf16_to_f32(l[e]) - mx);
        for (int e = 0; e < E; ++e) {
            p[e] = f64_to_bf16(exp((double)bf16_to_f32(l[e]) - mx) / sum);
            key[e] = ((uint32_t)p[e] << 16) | (uint32_t)e;   /* p >= 0: raw bits are ordered */
            if (probs) probs[(size_t)t * E + e] = p[e];
        }
        /* the K largest keys, output in ascending key order */
        uint32_t *sel = (uint32_t *)alloca(sizeof(uint32_t) * (size_t)K);
        int n = 0;
        for (int e = 0; e < E; ++e) {
            uint32_t k = key[e];
            if (n < K) {
                int j = n++;
                while (j > 0 && sel[j - 1] > k) { sel[j] = sel[j - 1]; --j; }
                sel[j] = k;
            } else if (k > sel[0]) {
                int j = 0;
                while (j + 1 < K && sel[j + 1] < k) { sel[j] = sel[j + 1]; ++j; }
                sel[j] = k;
            }
        }
        float S = bf16_to_f32((uint16_t)(sel[0] >> 16));
        for (int k = 1; k < K; ++k) S = bf(S + bf16_to_f32((uint16_t)(sel[k] >> 16)));
        for (int k = 0; k < K; ++k) {
            uint32_t e = sel[k] & 0xffffu;
            inds[(size_t)t * K + k] = e;
            if (scores) scores[(size_t)t * K + k] = f32_to_bf16(bf16_to_f32(p[e]) / S);
        }
    }
    free(p);
    free(key);
    return 0;
}

/* topk_sorted_indices: M largest logits (ties -> higher index selected), output sorted by
 * value descending with ties in ascending index order (stable argsort of -vals over the
 * argpartition order). */
int orc_topm_sorted(const uint16_t *logits, int T, int E, int M, uint32_t *pred) {
    if (M <= 0 || M > E || E > 65535) return -22;
    uint32_t *sel = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)M);
    if (!sel) return -12;
    for (int t = 0; t < T; ++t) {
        const uint16_t *l = logits + (size_t)t * E;
        int n = 0;
        for (int e = 0; e < E; ++e) {
            uint32_t k = (bf16_order_key(l[e]) << 16) | (uint32_t)e;
            if (n < M) {
                int j = n++;
                while (j > 0 && sel[j - 1] > k) { sel[j] = sel[j - 1]; --j; }
                sel[j] = k;
            } else if (k > sel[0]) {
                int j = 0;
                while (j + 1 < M && sel[j + 1] < k) { sel[j] = sel[j + 1]; ++j; }
                sel[j] = k;
            }
        }
        /* sel ascending by (value, index); emit value-descending, index-ascending */
        int o = 0;
        int i = M - 1;
        while (i >= 0) {
            uint32_t v = sel[i] >> 16;
            int j = i;
            while (j - 1 >= 0 && (sel[j - 1] >> 16) == v) --j;
            for (int q = j; q <= i; ++q) pred[(size_t)t * M + o++] = sel[q] & 0xffffu;
            i = j - 1;
        }
    }
    free(sel);
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* experts                                                                               */
/* ------------------------------------------------------------------------------------ */

static inline float sigmoidf_ref(float v) { return 1.0f / (1.0f + expf(-v)); }

/* SwiGLU with the per-op bf16 rounding of an MLX bf16 graph */
static inline float swiglu_bf16(float g, float u) {
    float sg = bf(sigmoidf_ref(g));
    float t = bf(g * sg);
    return bf(t * u);
}

/*
 * Routed expert block for T tokens.
 *   x      bf16 [T, H]          layer input
 *   slots  u32  [T, K]          slot (row of the slot buffers) of each routed expert
 *   scores bf16 [T, K]          routing weights (may be NULL -> only y_k / act outputs)
 *   w*     slot buffers in MLX layout: gate/up u32 [cap, I, H*bits/32] + s/b [cap, I, H/gs];
 *          down u32 [cap, H, I*bits/32] + s/b [cap, H, I/gs]
 *   addend bf16 [T, H] or NULL   (shared-expert output, added after the combine)
 *   resid  bf16 [T, H] or NULL   (residual stream, added last)
 *   y      bf16 [T, H] or NULL   combined output
 *   act    bf16 [T, K, I] or NULL  SwiGLU activations
 *   yk     bf16 [T, K, H] or NULL  per-expert down outputs (the unweighted SwitchGLU output)
 */
int orc_experts(const uint16_t *x, int T, int H, int I, int K, const uint32_t *slots,
                const uint16_t *scores,
                const uint32_t *wg, const uint16_t *sg, const uint16_t *bg,
                const uint32_t *wu, const uint16_t *su, const uint16_t *bu,
                const uint32_t *wd, const uint16_t *sd, const uint16_t *bd,
                int bits, int gs, int sb_fp16,
                const uint16_t *addend, const uint16_t *resid,
                uint16_t *y, uint16_t *act, uint16_t *yk) {
    if (bits != 2 && bits != 4 && bits != 8) return -22;
    if (gs <= 0 || H % gs || I % gs) return -22;
    const int per = 32 / bits;
    const size_t wg_row = (size_t)H / per, sg_row = (size_t)H / gs;
    const size_t wd_row = (size_t)I / per, sd_row = (size_t)I / gs;
    float *xf = (float *)malloc(sizeof(float) * (size_t)H);
    float *af = (float *)malloc(sizeof(float) * (size_t)K * I);
    float *yf = (float *)malloc(sizeof(float) * (size_t)K * H);
    if (!xf || !af || !yf) { free(xf); free(af); free(yf); return -12; }
    for (int t = 0; t < T; ++t) {
        for (int h = 0; h < H; ++h) xf[h] = bf16_to_f32(x[(size_t)t * H + h]);
#pragma omp parallel for collapse(2) schedule(static)
        for (int k = 0; k < K; ++k)
            for (int i = 0; i < I; ++i) {
                size_t sl = slots[(size_t)t * K + k];
                size_t r = sl * I + i;
                float gv = bf((float)qdot_row(wg + r * wg_row, sg + r * sg_row, bg + r * sg_row, sb_fp16, xf, H, bits, gs));
                float uv = bf((float)qdot_row(wu + r * wg_row, su + r * sg_row, bu + r * sg_row, sb_fp16, xf, H, bits, gs));
                af[(size_t)k * I + i] = swiglu_bf16(gv, uv);
            }
        if (act)
            for (size_t q = 0; q < (size_t)K * I; ++q) act[(size_t)t * K * I + q] = f32_to_bf16(af[q]);
#pragma omp parallel for collapse(2) schedule(static)
        for (int k = 0; k < K; ++k)
            for (int h = 0; h < H; ++h) {
                size_t sl = slots[(size_t)t * K + k];
                size_t r = sl * H + h;
                yf[(size_t)k * H + h] = bf((float)qdot_row(wd + r * wd_row, sd + r * sd_row, bd + r * sd_row, sb_fp16, af + (size_t)k * I, I, bits, gs));
            }
        if (yk)
            for (size_t q = 0; q < (size_t)K * H; ++q) yk[(size_t)t * K * H + q] = f32_to_bf16(yf[q]);
        if (y && scores) {
            for (int h = 0; h < H; ++h) {
                float acc = 0.f;
                for (int k = 0; k < K; ++k) {
                    float pk = bf(yf[(size_t)k * H + h] * bf16_to_f32(scores[(size_t)t * K + k]));
                    acc = (k == 0) ? pk : bf(acc + pk);
                }
                if (addend) acc = bf(acc + bf16_to_f32(addend[(size_t)t * H + h]));
                if (resid) acc = bf(bf16_to_f32(resid[(size_t)t * H + h]) + acc);
                y[(size_t)t * H + h] = f32_to_bf16(acc);
            }
        }
    }
    free(xf);
    free(af);
    free(yf);
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* shared expert (engine.cpp:394-400, loader.py:909-910) and QLinear (kernels.cpp:997-1019) */
/* ------------------------------------------------------------------------------------ */

/* y [T, N] = bf16(float(x [T, Kin] . W^T)), W affine-quantised [N, Kin*bits/32] + s/b
 * [N, Kin/gs]; qdot_row's arithmetic (float sums per group in input order, double over
 * groups in group order) */
int orc_affine_linear(const uint16_t *x, int T, int Kin, int N, const uint32_t *w, const uint16_t *s,
                      const uint16_t *b, int bits, int gs, int sb_fp16, uint16_t *y) {
    if (bits != 2 && bits != 4 && bits != 8) return -22;
    if (T <= 0 || Kin <= 0 || N <= 0 || gs <= 0 || Kin % gs || gs % (32 / bits)) return -22;
    const size_t wrow = (size_t)Kin / (32 / bits), srow = (size_t)Kin / gs;
    float *xf = (float *)malloc(sizeof(float) * (size_t)Kin);
    if (!xf) return -12;
    for (int t = 0; t < T; ++t) {
        for (int k = 0; k < Kin; ++k) xf[k] = bf16_to_f32(x[(size_t)t * Kin + k]);
#pragma omp parallel for schedule(static)
        for (int n = 0; n < N; ++n)
            y[(size_t)t * N + n] = f32_to_bf16((float)qdot_row(w + n * wrow, s + n * srow, b + n * srow, sb_fp16,
                                                               xf, Kin, bits, gs));
    }
    free(xf);
    return 0;
}

/*
 * shared_y [T, H] = bf16(bf16(sigmoid(gl)) * o), o = down(act), act = SwiGLU(gate(x), up(x)),
 * gl = expert_gate(x) [T, 1]. act [T, I] and o [T, H] are optional outputs (NULL to skip).
 */
int orc_shared_expert(const uint16_t *x, int T, int H, int I, const uint32_t *wg, const uint16_t *sg,
                      const uint16_t *bg, const uint32_t *wu, const uint16_t *su, const uint16_t *bu,
                      const uint32_t *wd, const uint16_t *sd, const uint16_t *bd, int bits, int gs,
                      const uint32_t *we, const uint16_t *se, const uint16_t *be, int gbits, int ggs,
                      int sb_fp16, uint16_t *y, uint16_t *act_out, uint16_t *o_out) {
    size_t ti = (size_t)T * I, th = (size_t)T * H;
    uint16_t *g = (uint16_t *)malloc(2 * ti), *u = (uint16_t *)malloc(2 * ti), *act = (uint16_t *)malloc(2 * ti);
    uint16_t *o = (uint16_t *)malloc(2 * th), *gl = (uint16_t *)malloc(2 * (size_t)T);
    int rc = (g && u && act && o && gl) ? 0 : -12;
    if (!rc) rc = orc_affine_linear(x, T, H, I, wg, sg, bg, bits, gs, sb_fp16, g);
    if (!rc) rc = orc_affine_linear(x, T, H, I, wu, su, bu, bits, gs, sb_fp16, u);
    if (!rc) {
        for (size_t i = 0; i < ti; ++i) act[i] = f32_to_bf16(swiglu_bf16(bf16_to_f32(g[i]), bf16_to_f32(u[i])));
        rc = orc_affine_linear(act, T, I, H, wd, sd, bd, bits, gs, sb_fp16, o);
    }
    if (!rc) rc = orc_affine_linear(x, T, H, 1, we, se, be, gbits, ggs, sb_fp16, gl);
    if (!rc) {
        for (size_t i = 0; i < th; ++i) {
            float sig = bf(sigmoidf_ref(bf16_to_f32(gl[i / H])));
            y[i] = f32_to_bf16(sig * bf16_to_f32(o[i]));
        }
        if (act_out) memcpy(act_out, act, 2 * ti);
        if (o_out) memcpy(o_out, o, 2 * th);
    }
    free(g);
    free(u);
    free(act);
    free(o);
    free(gl);
    return rc;
}

/* ------------------------------------------------------------------------------------ */
/* hyper-connection mixer before the MoE block (Qwen38Engine::run_hc, kernels.cpp:1363-1560) */
/* ------------------------------------------------------------------------------------ */

/* row totals of an affine-quantised matrix [N, Kin] times x [Kin] (floats), double results */
static void qrows(const uint32_t *w, const uint16_t *s, const uint16_t *b, int sb_fp16, int bits, int gs,
                  const float *x, int Kin, int N, double *out) {
    const size_t wrow = (size_t)Kin / (32 / bits), srow = (size_t)Kin / gs;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) out[n] = qdot_row(w + n * wrow, s + n * srow, b + n * srow, sb_fp16, x, Kin, bits, gs);
}

/*
 * One call of run_hc for T rows with hc_count HC streams of `H` values and low rank R:
 *   written = h (+ bf16(branch[t] * gate[t][c]) on stream c, rounded sums)   kernels.cpp:1380-1386
 *   normed  = per-stream RMS norm * (1 + norm_w)                              kernels.cpp:1042-1061
 *   d = down(normed) [R], v = d / HC, mix = silu(v)                           kernels.cpp:1387-1390
 *   u = up(mix) [HC*H], mixed[h] = mean_c sigmoid(u[c*H+h]) * normed[c*H+h]   kernels.cpp:1390-1393
 *   inj = 2 * sigmoid(inject(normed) / HC) [HC]                               kernels.cpp:1397-1399
 * Roundings follow the reference's two quantised paths: T <= 16 (the fused decode kernels,
 * kernels.cpp:1404-1516) keeps d, u and the inject dot products unrounded and rounds mix,
 * mixed and inj once; T > 16 (the prefill path, kernels.cpp:1518-1559 and the tail/inject
 * kernel at 788-846) rounds d and u to bf16, evaluates silu(v) and the stream sum with a bf16
 * rounding after every op, and rounds the inject value twice before its sigmoid.
 * RMS statistics: double sum of squares, rs = float(1 / sqrt(ss / H + eps)),
 * normed = bf16(float(x * rs) * (1 + w)).
 * branch/gate NULL = no write; inject NULL = the use_combine=False mixer (inj zeros).
 */
int orc_hc_mix(const uint16_t *h, int T, int HC, int H, int R, const uint16_t *branch, const uint16_t *gate,
               const uint16_t *norm_w, float eps, const uint32_t *wd, const uint16_t *sd, const uint16_t *bd,
               int dbits, int dgs, const uint32_t *wu, const uint16_t *su, const uint16_t *bu, int ubits, int ugs,
               const uint32_t *wi, const uint16_t *si, const uint16_t *bi, int ibits, int igs, int sb_fp16,
               uint16_t *written, uint16_t *normed_out, uint16_t *mixed, uint16_t *inj) {
    if (T <= 0 || HC <= 0 || H <= 0 || R <= 0) return -22;
    const int W = HC * H, prefill = T > 16;
    float *x = (float *)malloc(sizeof(float) * W), *nf = (float *)malloc(sizeof(float) * W);
    float *mf = (float *)malloc(sizeof(float) * R);
    double *dv = (double *)malloc(sizeof(double) * (W > R ? W : R)), *iv = (double *)malloc(sizeof(double) * HC);
    if (!x || !nf || !mf || !dv || !iv) { free(x); free(nf); free(mf); free(dv); free(iv); return -12; }
    for (int t = 0; t < T; ++t) {
        const uint16_t *hr = h + (size_t)t * W;
        for (int c = 0; c < HC; ++c)
            for (int i = 0; i < H; ++i) {
                const int n = c * H + i;
                float v = bf16_to_f32(hr[n]);
                if (branch && gate) {
                    float p = bf(bf16_to_f32(branch[(size_t)t * H + i]) * bf16_to_f32(gate[(size_t)t * HC + c]));
                    v = bf(v + p);
                }
                x[n] = v;
                if (written) written[(size_t)t * W + n] = f32_to_bf16(v);
            }
        for (int c = 0; c < HC; ++c) {
            double ss = 0.0;
            for (int i = 0; i < H; ++i) ss += (double)x[c * H + i] * (double)x[c * H + i];
            const float rs = (float)(1.0 / sqrt(ss / H + (double)eps));
            for (int i = 0; i < H; ++i) {
                const int n = c * H + i;
                const float y = x[n] * rs;
                nf[n] = bf(y * (1.0f + bf16_to_f32(norm_w[n])));
                if (normed_out) normed_out[(size_t)t * W + n] = f32_to_bf16(nf[n]);
            }
        }
        qrows(wd, sd, bd, sb_fp16, dbits, dgs, nf, W, R, dv);
        for (int r = 0; r < R; ++r) {
            if (prefill) {
                const float v = bf(bf((float)dv[r]) / (float)HC);
                mf[r] = bf(v * bf(sigmoidf_ref(v)));
            } else {
                const float v = (float)dv[r] / (float)HC;
                mf[r] = bf(v * sigmoidf_ref(v));
            }
        }
        qrows(wu, su, bu, sb_fp16, ubits, ugs, mf, R, W, dv);
        for (int i = 0; i < H; ++i) {
            float acc = 0.f;
            for (int c = 0; c < HC; ++c) {
                const int n = c * H + i;
                if (prefill) {
                    const float p = bf(bf(sigmoidf_ref(bf((float)dv[n]))) * nf[n]);
                    acc = c == 0 ? p : bf(acc + p);
                } else {
                    const float p = sigmoidf_ref((float)dv[n]) * nf[n];
                    acc = c == 0 ? p : acc + p;
                }
            }
            mixed[(size_t)t * H + i] = f32_to_bf16(prefill ? acc * (1.0f / (float)HC) : acc / (float)HC);
        }
        if (inj) {
            if (wi) qrows(wi, si, bi, sb_fp16, ibits, igs, nf, W, HC, iv);
            for (int c = 0; c < HC; ++c) {
                float o = 0.f;
                if (wi && prefill) {
                    const float q = bf(bf((float)iv[c]) / (float)HC);
                    o = 2.0f * bf(sigmoidf_ref(q));
                } else if (wi) {
                    o = 2.0f * sigmoidf_ref((float)iv[c] / (float)HC);
                }
                inj[(size_t)t * HC + c] = f32_to_bf16(o);
            }
        }
    }
    free(x);
    free(nf);
    free(mf);
    free(dv);
    free(iv);
    return 0;
}

/* number of OpenMP threads the oracle uses (1 when built without OpenMP) */
int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* bf16 conversion helpers exported for tests */
uint16_t orc_f64_to_bf16(double d) { return f64_to_bf16(d); }
uint16_t orc_f32_to_bf16(float f) { return f32_to_bf16(f); }
