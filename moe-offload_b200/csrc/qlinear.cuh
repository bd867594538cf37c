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
// Work split ("one group per thread"): a block takes `rows` output rows (of up to `mats`
// matrices) and gives every (matrix, row, group) item its own thread, so the only serial chain
// is one group's gs multiply-adds. The item's words, scale and bias are loaded into registers
// before the kernel waits on its predecessor (they do not depend on it); the x rows of up to
// kLinTok tokens are staged in shared memory by the whole block; group values go to shared
// memory and one thread per (row, token) adds them in group order.
#pragma once

#include <cstdint>
#include <utility>

#include "common.cuh"

namespace moe_qlin {

constexpr int kLinTok = 4;                       // tokens per pass
constexpr int kMaxGroups = 384;                  // groups per row
constexpr int kItemThreads = 256;                // target items per block
constexpr int kMaxBlock = 512;                   // threads per block (mats * groups per row at most)
constexpr size_t kXStageMax = 64 * 1024;         // x rows staged in shared memory up to this size

// threads per block for a group size: 128-value groups hold twice the codes in registers
constexpr int max_block(int gs) { return gs >= 128 ? 256 : kMaxBlock; }

// q (< 2^23) as float without an int -> float conversion: the float with exponent 2^23 and
// mantissa q is exactly 2^23 + q, so subtracting 2^23 leaves q exactly
MOE_D float code_f32(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }

MOE_D float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
MOE_D float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

template <bool kFp16>
MOE_D double group_value(uint16_t s, uint16_t b, float acc, float xs) {
    const double sc = (double)sb_to_f32<kFp16>(s), bi = (double)sb_to_f32<kFp16>(b);
    return fma(sc, (double)acc, bi * (double)xs);
}

// one group of one row, its codes held in registers
template <int kBits, int kGs, bool kFp16>
struct GroupItem {
    static constexpr int kPer = 32 / kBits;      // codes per word
    static constexpr int kWords = kGs / kPer;    // words per group (2 .. 32)
    static constexpr uint32_t kMask = (1u << kBits) - 1u;

    uint32_t wv[kWords];
    uint16_t sc, bi;

    // wrow / srow / brow: the row's codes, scales and biases; g: the group
    MOE_D void load(const uint32_t *wrow, const uint16_t *srow, const uint16_t *brow, int g) {
        const uint32_t *gw = wrow + (size_t)g * kWords;
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
        sc = __ldg(srow + g), bi = __ldg(brow + g);
    }

    // the group value for the kGs x values at xg (shared or global memory, 16-byte aligned):
    // sum q x and sum x in input order, then scale and bias in double
    MOE_D double value(const uint16_t *xg) const {
        float acc = 0.f, xs = 0.f;
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
        return group_value<kFp16>(sc, bi, acc, xs);
    }
};

// The same group value for a row of any width and group size (runtime bits / gs); the row may
// sit in shared or global memory (plain loads).
template <bool kFp16>
MOE_D double generic_group_value(const uint16_t *xg, const uint32_t *wrow, const uint16_t *srow,
                                 const uint16_t *brow, int bits, int gs, int g) {
    const int lper = bits == 2 ? 4 : (bits == 4 ? 3 : 2);   // log2(32 / bits)
    const uint32_t mask = (1u << bits) - 1u;
    float acc = 0.f, xsum = 0.f;
#pragma unroll 1
    for (int k0 = 0; k0 < gs; k0 += 8) {
        const uint4 v = reinterpret_cast<const uint4 *>(xg + k0)[0];
        const uint32_t pk[4] = {v.x, v.y, v.z, v.w};
        uint32_t wd[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) wd[i] = wrow[((size_t)g * gs + k0 + i) >> lper];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int k = g * gs + k0 + i;
            const float xv = (i & 1) ? bf16_hi(pk[i >> 1]) : bf16_lo(pk[i >> 1]);
            const uint32_t sh = (uint32_t)(bits * (k & ((1 << lper) - 1)));
            acc = fmaf(code_f32((wd[i] >> sh) & mask), xv, acc);
            xsum = __fadd_rn(xsum, xv);
        }
    }
    return group_value<kFp16>(srow[g], brow[g], acc, xsum);
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

// Block shape of a flat launch: `rows` rows per block, items = mats * rows * ng threads (a
// multiple of 32), shared memory for the group values [rows][mats][kLinTok][ng] doubles plus the
// staged x rows [min(T, kLinTok)][Kin] bf16 when they fit (xbytes = 0: x read from global).
struct FlatShape {
    int rows, threads;
    size_t grp, xbytes;
    MOE_HD size_t smem() const { return grp + xbytes; }
};

MOE_HD FlatShape flat_shape(int mats, int ng, int T, int Kin) {
    FlatShape f;
    const int per_row = mats * ng;
    f.rows = per_row >= kItemThreads ? 1 : kItemThreads / per_row;
    f.threads = ((f.rows * per_row + 31) / 32) * 32;
    f.grp = (size_t)f.rows * mats * kLinTok * ng * sizeof(double);
    const size_t xb = (size_t)(T < kLinTok ? T : kLinTok) * Kin * 2;
    f.xbytes = xb <= kXStageMax ? xb : 0;
    return f;
}

// launch with programmatic stream serialisation: the kernel may start while its predecessor
// runs; every kernel here calls pdl_wait() before reading what an earlier kernel wrote
template <typename... P, typename... A>
cudaError_t launch_pdl_v(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A &&...args) {
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...);
}

}  // namespace moe_qlin

// host entry points defined in shared.cu for the other quantised-linear users
int moe_qlin_check(const char *who, const void *x, int T, int Kin, int N, const void *w, const void *s,
                   const void *b, int bits, int gs, const void *y);
// y (bf16, optionally scaled by bf16(sigmoid(gl[t]))) or yf (float, unrounded total) = x . W^T;
// with N2 > 0 the same launch also writes yf2 [T, N2] = float totals of a second matrix
// (w2, s2, b2) of the same width and group size
int moe_qlin_linear(const void *x, int T, int Kin, int N, const void *w, const void *s, const void *b, int bits,
                    int gs, int sb_fp16, const void *gl, void *y, float *yf, cudaStream_t st,
                    const void *w2 = nullptr, const void *s2 = nullptr, const void *b2 = nullptr, int N2 = 0,
                    float *yf2 = nullptr);
