// Shared device helpers for the sm_100a MoE kernels: status codes, bf16/fp16 bit
// conversions, streaming loads and the 2-bit -> bf16x2 "mantissa OR" expansion used by
// every decode GEMV.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/moe_b200.h"

#define MOE_HD __host__ __device__ __forceinline__
#define MOE_D __device__ __forceinline__

// ------------------------------------------------------------------ error plumbing

#define MOE_CUDA_TRY(expr)                                   \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) return moe_set_cuda_error(_e); \
    } while (0)

int moe_set_cuda_error(cudaError_t e);          // records the message; returns MOE_ECUDA
int moe_set_error(int code, const char *fmt, ...);

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

MOE_HD size_t al16(size_t v) { return (v + 15) & ~size_t(15); }
MOE_HD size_t al128(size_t v) { return (v + 127) & ~size_t(127); }
MOE_HD size_t al256(size_t v) { return (v + 255) & ~size_t(255); }
MOE_HD int pad4(int v) { return (v + 3) & ~3; }

// ------------------------------------------------------------------ scalar conversions

MOE_D float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

// round-to-nearest-even float -> bf16 bits (same rule as the CPU oracle)
MOE_D uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

MOE_D float bf16r(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

// Power-of-two RMS normalisation of a layer input: x = h * 2^-k with k = floor(e / 2) for
// sum(h^2)/n in [2^(e-1), 2^e), so RMS(x) lies in [2^-0.5, 2^0.5). A power of two keeps every
// bf16 value exact (x and h have the same mantissas), so x.W = 2^-k (h.W) exactly.
MOE_HD int pow2_rms_shift(double sumsq, int n) {
    if (!(sumsq > 0.0) || n <= 0) return 0;
    int e = 0;
    frexp(sumsq / (double)n, &e);
    return (e >= 0) ? e / 2 : -((1 - e) / 2);
}

// double -> bf16 with ONE rounding (cvt.rn.bf16.f64, sm_90+): the router's logits and
// probabilities are rounded once from an order-independent double value.
MOE_D uint16_t f64_to_bf16_bits(double d) {
    uint16_t r;
    asm("cvt.rn.bf16.f64 %0, %1;" : "=h"(r) : "d"(d));
    return r;
}

template <bool kFp16>
MOE_D float sb_to_f32(uint16_t v) {
    if constexpr (kFp16) return __half2float(__ushort_as_half(v));
    else return bf16_bits_to_f32(v);
}

// ------------------------------------------------------------------ memory access

// 16-byte streaming load of weight bytes that are read once per token: bypass L1 and ask
// L2 for a 256-byte prefetch of the surrounding sector group.
MOE_D uint4 ldg_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

MOE_D uint16_t ldg_u16(const uint16_t *p) { return __ldg(p); }

// ------------------------------------------------------------------ 2-bit expansion
//
// A 2-bit affine group is 64 codes = 16 bytes = 4 words; word m holds codes 16m..16m+15,
// code c at bits 2c. For the m16n8k16 bf16 MMA a word is expanded to 8 bf16x2 registers
// P[0..7] without per-code shifts: OR-ing a code that sits in bits [0,6) of a 16-bit half
// into 0x3F80 (bf16 1.0) gives the exact bf16 value 1 + q * 2^(pos-7).
//   P[p] holds (code p, code p+8) with position scale c[p] = 2^-7, 2^-5, 2^-3 for
//   p % 3 == 0, 1, 2 (p < 8). The B operand carries x / c[p] so that
//   sum (1 + q c) (x / c) = sum x / c + sum q x, and the kernels subtract the per-group
//   constant sum x / c ("corr") afterwards.
MOE_D void expand_word(uint32_t w, uint32_t P[8]) {
    const uint32_t one = 0x3F803F80u;
    const uint32_t w6 = w >> 6, w12 = w >> 12;
    P[0] = (w & 0x00030003u) | one;
    P[1] = (w & 0x000C000Cu) | one;
    P[2] = (w & 0x00300030u) | one;
    P[3] = (w6 & 0x00030003u) | one;
    P[4] = (w6 & 0x000C000Cu) | one;
    P[5] = (w6 & 0x00300030u) | one;
    P[6] = (w12 & 0x00030003u) | one;
    P[7] = (w12 & 0x000C000Cu) | one;
}

// inverse position scale for pair p
MOE_HD float pair_inv_scale(int p) { return (p % 3 == 0) ? 128.f : ((p % 3 == 1) ? 32.f : 8.f); }

// D(16x8 f32) += A(16x16 bf16, row) * B(16x8 bf16, col)
MOE_D void mma_bf16_16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

MOE_D uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}

// ------------------------------------------------------------------ B-operand staging
//
// For one 64-wide group of an input vector v (bf16), the MMA B operand of word m and MMA
// mi is two bf16x2 registers:
//   b01 = (v[16m+2mi] / c[2mi],   v[16m+2mi+8] / c[2mi])
//   b23 = (v[16m+2mi+1] / c[2mi+1], v[16m+2mi+9] / c[2mi+1])
// stored as uint2 entry (m*4 + mi) of the group's 16-entry (128-byte) record. The group's
// corr = sum of all 64 scaled values and xsum = sum v are stored alongside.
//
// Builds records for groups [0, ngroups) of `v` into `frag` (smem) using all threads of
// the block; groups beyond the vector length are zero-filled. Requires blockDim.x % 16 == 0.
MOE_D void stage_bfrag(const uint16_t *__restrict__ v, int n, int ngroups, uint2 *frag, float *corr,
                       float *xsum) {
    const int nent = ngroups * 16;
    for (int base = 0; base < nent; base += blockDim.x) {
        const int e = base + threadIdx.x;
        float cs = 0.f, xs = 0.f;
        if (e < nent) {
            const int G = e >> 4, m = (e >> 2) & 3, mi = e & 3;
            const int c0 = G * 64 + 16 * m + 2 * mi;
            float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
            if (G * 64 < n) {
                v0 = bf16_bits_to_f32(v[c0]);
                v1 = bf16_bits_to_f32(v[c0 + 8]);
                v2 = bf16_bits_to_f32(v[c0 + 1]);
                v3 = bf16_bits_to_f32(v[c0 + 9]);
            }
            const float i0 = pair_inv_scale(2 * mi), i1 = pair_inv_scale(2 * mi + 1);
            const float s0 = v0 * i0, s1 = v1 * i0, s2 = v2 * i1, s3 = v3 * i1;
            frag[e] = make_uint2(pack_bf16x2(s0, s1), pack_bf16x2(s2, s3));
            cs = (s0 + s1) + (s2 + s3);
            xs = (v0 + v1) + (v2 + v3);
        }
        // reduce over the 16 consecutive entries of a group (aligned 16-lane segment)
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            cs += __shfl_xor_sync(0xffffffffu, cs, off);
            xs += __shfl_xor_sync(0xffffffffu, xs, off);
        }
        if (e < nent && (e & 15) == 0) {
            corr[e >> 4] = cs;
            xsum[e >> 4] = xs;
        }
    }
}

// ------------------------------------------------------------------ TMA bulk copies + mbarrier
//
// 1-D bulk copies (cp.async.bulk, no multicast) global -> shared, completing on an mbarrier
// with a transaction byte count. Every wait is bounded: after kMbarSpinLimit polls the
// waiter records MOE_DEVERR_MBAR_TIMEOUT in the device error word and gives up, so a kernel
// never spins forever.

#define MOE_DEVERR_MBAR_TIMEOUT 1u
#define MOE_DEVERR_BAD_INPUT 2u

extern __device__ unsigned int g_moe_device_error;

constexpr uint32_t kMbarSpinLimit = 1u << 26;

MOE_D uint32_t smem_addr(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

MOE_D void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// make barrier initialisation visible to the async (TMA) proxy
MOE_D void fence_barrier_init() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

MOE_D void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

MOE_D void tma_load_1d(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

MOE_D bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// bounded wait for phase `parity`; false (and the device error word set) on timeout
MOE_D bool mbar_wait(uint64_t *bar, uint32_t parity) {
#pragma unroll 1
    for (uint32_t i = 0; i < kMbarSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr(&g_moe_device_error, MOE_DEVERR_MBAR_TIMEOUT);
    return false;
}

// ------------------------------------------------------------------ programmatic dependent launch
// The next kernel in the stream may start once every CTA of this one has called
// pdl_launch_dependents(); it must call pdl_wait() before touching this kernel's outputs.
MOE_D void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
MOE_D void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// B records of a vector already resident in shared memory (bf16, `n` values): the same
// layout as stage_bfrag, built without any global-memory round trip.
MOE_D void build_bfrag_smem(const uint16_t *v, int ngroups, uint2 *frag, float *corr, float *xsum) {
    const int nent = ngroups * 16;
    for (int base = 0; base < nent; base += blockDim.x) {
        const int e = base + threadIdx.x;
        float cs = 0.f, xs = 0.f;
        if (e < nent) {
            const int G = e >> 4, m = (e >> 2) & 3, mi = e & 3;
            const int c0 = G * 64 + 16 * m + 2 * mi;
            const uint32_t p01 = *reinterpret_cast<const uint32_t *>(v + c0);       // v[c0], v[c0+1]
            const uint32_t p89 = *reinterpret_cast<const uint32_t *>(v + c0 + 8);   // v[c0+8], v[c0+9]
            const float v0 = __uint_as_float(p01 << 16), v2 = __uint_as_float(p01 & 0xffff0000u);
            const float v1 = __uint_as_float(p89 << 16), v3 = __uint_as_float(p89 & 0xffff0000u);
            const float i0 = pair_inv_scale(2 * mi), i1 = pair_inv_scale(2 * mi + 1);
            const float s0 = v0 * i0, s1 = v1 * i0, s2 = v2 * i1, s3 = v3 * i1;
            frag[e] = make_uint2(pack_bf16x2(s0, s1), pack_bf16x2(s2, s3));
            cs = (s0 + s1) + (s2 + s3);
            xs = (v0 + v1) + (v2 + v3);
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            cs += __shfl_xor_sync(0xffffffffu, cs, off);
            xs += __shfl_xor_sync(0xffffffffu, xs, off);
        }
        if (e < nent && (e & 15) == 0) {
            corr[e >> 4] = cs;
            xsum[e >> 4] = xs;
        }
    }
}

// Launch with the programmatic-stream-serialization attribute (PDL): the kernel may begin
// while its predecessor in the stream is still running; it must pdl_wait() before reading
// anything an earlier kernel produced.
template <typename Kern, typename Args>
static cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, const Args &args) {
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
    return cudaLaunchKernelEx(&cfg, kern, args);
}
