// Building blocks of the affine-quantised linear layers (shared expert, hyper-connection mixer):
// MLX's affine format, w = scale * q + bias per group of `gs` inputs, `bits`-bit codes packed
// 32/bits per little-endian uint32, code j of a word in bits [bits*j, bits*j + bits).
//
// Arithmetic (the routed-expert GEMVs' qmv form, scale * sum(q x) + bias * sum(x) per group):
// within a group, sum(q x) and sum(x) are float sums in input order (each q x is exact in
// float); the group's value scale * sum(q x) + bias * sum(x) is formed in double (both products
// exact); the row total is the double sum of the group values in group order. The order is
// fixed, so results do not depend on the launch shape.
//
// Work split: one warp per output row (or per set of kMats rows), lane l on groups l, l + 32,
// ...; the words of the next group are loaded while the current one is used; group values go
// to shared memory and one lane per (row, token) adds them in group order. Up to kLinTok tokens
// share one pass over the weights; their x rows are staged in shared memory by the whole block
// when they fit.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace moe_qlin {

constexpr int kLinWarps = 4;                     // warps per block
constexpr int kLinThreads = kLinWarps * 32;
constexpr int kLinTok = 4;                       // tokens per pass over the weights
constexpr int kMaxGroups = 384;                  // groups per row
constexpr size_t kXStageMax = 64 * 1024;         // x rows staged in shared memory up to this size

// q (< 2^23) as float without an int -> float conversion: the float with exponent 2^23 and
// mantissa q is exactly 2^23 + q, so subtracting 2^23 leaves q exactly
MOE_D float code_f32(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }

MOE_D float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
MOE_D float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

template <int kBits, int kGs>
struct Group {
    static constexpr int kPer = 32 / kBits;      // codes per word
    static constexpr int kWords = kGs / kPer;    // words per group (2 .. 32)
    static constexpr uint32_t kMask = (1u << kBits) - 1u;

    MOE_D static void load(const uint32_t *gw, uint32_t (&wv)[kWords]) {
        if constexpr (kWords % 4 == 0) {
#pragma unroll
            for (int c = 0; c < kWords / 4; ++c) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(gw) + c);
                wv[4 * c] = v.x, wv[4 * c + 1] = v.y, wv[4 * c + 2] = v.z, wv[4 * c + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int c = 0; c < kWords / 2; ++c) {
                const uint2 v = __ldg(reinterpret_cast<const uint2 *>(gw) + c);
                wv[2 * c] = v.x, wv[2 * c + 1] = v.y;
            }
        }
    }

    // acc = sum q x, xs = sum x over the group, both in input order; xg: the group's kGs bf16
    // values (shared or global memory, 16-byte aligned)
    MOE_D static void dot(const uint32_t (&wv)[kWords], const uint16_t *xg, float &acc, float &xs) {
        acc = 0.f, xs = 0.f;
#pragma unroll
        for (int c = 0; c < kGs / 8; ++c) {
            const uint4 v = reinterpret_cast<const uint4 *>(xg)[c];
            const uint32_t pk[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int k = 8 * c + i;
                const float xv = (i & 1) ? bf16_hi(pk[i >> 1]) : bf16_lo(pk[i >> 1]);
                const float q = code_f32((wv[k / kPer] >> (kBits * (k % kPer))) & kMask);
                acc = fmaf(q, xv, acc);          // q x is exact: one rounding, as acc + q x
                xs = __fadd_rn(xs, xv);
            }
        }
    }
};

template <bool kFp16>
MOE_D double group_value(const uint16_t *s, const uint16_t *b, int g, float acc, float xs) {
    const double sc = (double)sb_to_f32<kFp16>(__ldg(s + g)), bi = (double)sb_to_f32<kFp16>(__ldg(b + g));
    return fma(sc, (double)acc, bi * (double)xs);
}

// Group values of kMats rows (row m: codes w[m], scales s[m], biases b[m]) for the nt token
// rows at xs (row stride Kin) into sv[(m * kLinTok + j) * ng + g].
template <int kBits, int kGs, bool kFp16, int kMats>
MOE_D void stage_rows(const uint16_t *xs, int Kin, int nt, const uint32_t *const (&w)[kMats],
                      const uint16_t *const (&s)[kMats], const uint16_t *const (&b)[kMats], int ng, int lane,
                      double *sv) {
    using G = Group<kBits, kGs>;
    uint32_t cur[kMats][G::kWords], nxt[kMats][G::kWords];
    if (lane < ng) {
#pragma unroll
        for (int m = 0; m < kMats; ++m) G::load(w[m] + (size_t)lane * G::kWords, cur[m]);
    }
#pragma unroll 1
    for (int g = lane; g < ng; g += 32) {
        const int gn = g + 32;
        if (gn < ng) {
#pragma unroll
            for (int m = 0; m < kMats; ++m) G::load(w[m] + (size_t)gn * G::kWords, nxt[m]);
        }
#pragma unroll 1
        for (int j = 0; j < nt; ++j) {
            const uint16_t *xg = xs + (size_t)j * Kin + (size_t)g * kGs;
#pragma unroll
            for (int m = 0; m < kMats; ++m) {
                float acc, xsum;
                G::dot(cur[m], xg, acc, xsum);
                sv[(m * kLinTok + j) * ng + g] = group_value<kFp16>(s[m], b[m], g, acc, xsum);
            }
        }
        if (gn < ng) {
#pragma unroll
            for (int m = 0; m < kMats; ++m)
#pragma unroll
                for (int q = 0; q < G::kWords; ++q) cur[m][q] = nxt[m][q];
        }
    }
}

// stage_rows for rows with few groups: the (row, group) pairs are spread over the lanes, so
// kMats * ng lanes work at once; same values in sv as stage_rows
template <int kBits, int kGs, bool kFp16, int kMats>
MOE_D void stage_rows_spread(const uint16_t *xs, int Kin, int nt, const uint32_t *const (&w)[kMats],
                             const uint16_t *const (&s)[kMats], const uint16_t *const (&b)[kMats], int ng, int lane,
                             double *sv) {
    using G = Group<kBits, kGs>;
#pragma unroll 1
    for (int it = lane; it < kMats * ng; it += 32) {
        const int m = it / ng, g = it - m * ng;
        const uint32_t *wm = w[0];
        const uint16_t *sm = s[0], *bm = b[0];
#pragma unroll
        for (int q = 1; q < kMats; ++q)
            if (m == q) wm = w[q], sm = s[q], bm = b[q];
        uint32_t wv[G::kWords];
        G::load(wm + (size_t)g * G::kWords, wv);
#pragma unroll 1
        for (int j = 0; j < nt; ++j) {
            float acc, xsum;
            G::dot(wv, xs + (size_t)j * Kin + (size_t)g * kGs, acc, xsum);
            sv[(m * kLinTok + j) * ng + g] = group_value<kFp16>(sm, bm, g, acc, xsum);
        }
    }
}

// One row of any width and group size (runtime bits / gs) for the nt token rows at xs: same
// sums in the same order as stage_rows, the (group, token) pairs spread over the lanes.
template <bool kFp16>
MOE_D void stage_row_generic(const uint16_t *xs, int Kin, int nt, const uint32_t *w, const uint16_t *s,
                             const uint16_t *b, int bits, int gs, int lane, double *sv) {
    const int lper = bits == 2 ? 4 : (bits == 4 ? 3 : 2), ng = Kin / gs;   // log2(32 / bits)
    const uint32_t mask = (1u << bits) - 1u;
#pragma unroll 1
    for (int it = lane; it < ng * nt; it += 32) {
        const int g = it % ng, j = it / ng;
        const uint16_t *xg = xs + (size_t)j * Kin + (size_t)g * gs;
        float acc = 0.f, xsum = 0.f;
#pragma unroll 1
        for (int k0 = 0; k0 < gs; k0 += 8) {
            const uint4 v = reinterpret_cast<const uint4 *>(xg + k0)[0];
            const uint32_t pk[4] = {v.x, v.y, v.z, v.w};
            uint32_t wd[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) wd[i] = __ldg(w + (((size_t)g * gs + k0 + i) >> lper));
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int k = g * gs + k0 + i;
                const float xv = (i & 1) ? bf16_hi(pk[i >> 1]) : bf16_lo(pk[i >> 1]);
                const uint32_t sh = (uint32_t)(bits * (k & ((1 << lper) - 1)));
                acc = fmaf(code_f32((wd[i] >> sh) & mask), xv, acc);
                xsum = __fadd_rn(xsum, xv);
            }
        }
        sv[j * ng + g] = group_value<kFp16>(s, b, g, acc, xsum);
    }
}

MOE_D double sum_in_order(const double *v, int n) {
    double total = 0.0;
    for (int g = 0; g < n; ++g) total += v[g];
    return total;
}

MOE_D uint16_t row_out(double total) { return f32_to_bf16_bits((float)total); }

MOE_D float sigmoidf(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); }
MOE_D float sigmoid_bf16(float v) { return bf16r(sigmoidf(v)); }

// the block copies x rows t0 .. t0+nt-1 (Kin values each, Kin a multiple of 8) to sx
MOE_D void stage_x(uint16_t *sx, const uint16_t *x, int Kin, int t0, int nt) {
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)t0 * Kin);
    uint4 *dst = reinterpret_cast<uint4 *>(sx);
    const int n16 = nt * Kin / 8;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldg(src + i);
}

// shared memory of a block: group values [kLinWarps][kMats][kLinTok][ng] doubles, then the
// staged x rows [min(T, kLinTok)][Kin] bf16 when they fit in kXStageMax
struct LinSmem {
    size_t grp, xbytes;
    MOE_HD size_t total() const { return grp + xbytes; }
};

MOE_HD LinSmem lin_smem(int mats, int ng, int T, int Kin) {
    LinSmem L;
    L.grp = (size_t)kLinWarps * mats * kLinTok * ng * sizeof(double);
    const size_t xb = (size_t)(T < kLinTok ? T : kLinTok) * Kin * 2;
    L.xbytes = xb <= kXStageMax ? xb : 0;
    return L;
}

}  // namespace moe_qlin

// host entry points defined in shared.cu for the other quantised-linear users
int moe_qlin_check(const char *who, const void *x, int T, int Kin, int N, const void *w, const void *s,
                   const void *b, int bits, int gs, const void *y);
// y (bf16, optionally scaled by bf16(sigmoid(gl[t]))) or yf (float, unrounded total) = x . W^T
int moe_qlin_linear(const void *x, int T, int Kin, int N, const void *w, const void *s, const void *b, int bits,
                    int gs, int sb_fp16, const void *gl, void *y, float *yf, cudaStream_t st);
