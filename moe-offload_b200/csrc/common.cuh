// Shared device helpers for the sm_100a MoE kernels: status codes, bf16/fp16 bit
// conversions, streaming loads, 1-D TMA bulk copies with bounded mbarrier waits and
// programmatic dependent launch.
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

// ------------------------------------------------------------------ TMA bulk copies + mbarrier
//
// 1-D bulk copies (cp.async.bulk, no multicast) global -> shared, completing on an mbarrier
// with a transaction byte count. Every wait is bounded: after kMbarSpinLimit polls the
// waiter records MOE_DEVERR_MBAR_TIMEOUT in the device error word and gives up, so a kernel
// never spins forever.

#define MOE_DEVERR_MBAR_TIMEOUT 1u
#define MOE_DEVERR_BAD_INPUT 2u
#define MOE_DEVERR_PEER_TIMEOUT 4u      // an expert-parallel peer did not signal within the limit

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
