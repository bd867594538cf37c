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
// not depend on G. Grid barriers are bounded: a timeout sets the device error word. The phases
// are in f3core.cuh, shared with the kernel that fuses them with the routed block (stack.cu).
#include <cstdint>

#include <cuda_runtime.h>

#include "common.cuh"
#include "f3core.cuh"

namespace {

using namespace moe_f3;

constexpr uint32_t kF3SpinLimit = 1u << 24;

struct F3Args {
    const moe_f3_layer *layers;
    int L, H, R, I;
    float eps;
    const uint16_t *h0, *branch0, *gate0;
    uint16_t *state_out, *branch_out, *inj_out, *branch_all;
    F3Bufs bufs;
    uint16_t *state, *branch, *inj;
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
// g_f3_trace[cta][layer][slot], read back with moe_f3_trace_read. Slots: 0 layer start, 12 the
// write and norm sums done, 10 barrier 0 passed, 1 norm done, 2 mixer-down items done,
// 3 barrier 1 passed, 4 mixer up + tail done, 5 barrier 2, 6 shared gate / up done, 7 barrier
// 3, 8 shared down done, 9 barrier 4. The library build compiles them out.
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

template <bool kFp16>
__global__ void __launch_bounds__(kF3Threads, 1) f3_stack_kernel(F3Args a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int H = a.H, W = kHcStreams * H;
    const F3Smem S(H, a.R, a.I, gridDim.x);
    __shared__ float srs[kHcStreams];
    F3Phases<kFp16> f(H, a.R, a.I, a.bufs, smem + S.normed, smem + S.sx, smem + S.sv, smem + S.spart, srs);
    unsigned int nbar = 0;
    f.prefetch_mixer_down(a.layers[0]);

#pragma unroll 1
    for (int l = 0; l < a.L; ++l) {
        const moe_f3_layer &Ly = a.layers[l];
        const uint16_t *hin = l == 0 ? a.h0 : a.state + (size_t)(l & 1) * W;
        const uint16_t *br = l == 0 ? a.branch0 : a.branch + (size_t)((l - 1) & 1) * H;
        const uint16_t *gt = l == 0 ? a.gate0 : a.inj + (size_t)((l - 1) & 1) * kHcStreams;
        uint16_t *wout = a.state + (size_t)((l + 1) & 1) * W;
        F3_STAMP(l, 0);
        f.write_and_sums(hin, br, gt, wout);
        F3_STAMP(l, 12);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 10);
        f.norm(Ly, wout, a.eps);
        F3_STAMP(l, 1);
        f.mixer_down(Ly);
        F3_STAMP(l, 2);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 3);
        f.mixer_up(Ly, a.inj + (size_t)(l & 1) * kHcStreams, nullptr);
        F3_STAMP(l, 4);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 5);
        stage_l2(f.sx, a.bufs.mixed, H);
        __syncthreads();
        f.shared_gate_up(Ly, true);
        F3_STAMP(l, 6);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 7);
        {
            // P4: shared down rows this CTA owns, scaled by bf16(sigmoid(gate)): the block output
            const float gsig = f.stage_down();
            uint16_t *bro = a.branch + (size_t)(l & 1) * H;
            f.shared_down_items(Ly, f.j, f.G, f.nh, true);
            if (l + 1 < a.L) f.prefetch_mixer_down(a.layers[l + 1]);
            __syncthreads();
            for (int q = threadIdx.x; q < f.nh; q += kF3Threads) {
                const int n = f.j + q * f.G;
                const uint16_t y = f.shared_down_out(q, gsig);
                bro[n] = y;
                if (a.branch_all) a.branch_all[(size_t)l * H + n] = y;
            }
        }
        F3_STAMP(l, 8);
        f3_grid_sync(a.bar, nbar++);
        F3_STAMP(l, 9);
    }

    // the last block's write into the state, and the last block output and gate
    if (blockIdx.x == 0) {
        const int l = a.L - 1;
        const uint16_t *st = a.state + (size_t)((l + 1) & 1) * W;
        const uint16_t *br = a.branch + (size_t)(l & 1) * H;
        const uint16_t *gt = a.inj + (size_t)(l & 1) * kHcStreams;
        for (int q = threadIdx.x; q < W; q += kF3Threads) {
            const int c = q / H, i = q - c * H;
            const float gv = bf16_bits_to_f32(__ldcg(gt + c));
            const float p = bf16r(__fmul_rn(bf16_bits_to_f32(__ldcg(br + i)), gv));
            a.state_out[q] = f32_to_bf16_bits(bf16r(__fadd_rn(bf16_bits_to_f32(__ldcg(st + q)), p)));
        }
        for (int q = threadIdx.x; q < H; q += kF3Threads) a.branch_out[q] = __ldcg(br + q);
        if (threadIdx.x < kHcStreams && a.inj_out) a.inj_out[threadIdx.x] = __ldcg(gt + threadIdx.x);
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
    const F3Smem S(H, R, I, G);
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
    a.bufs.dv = reinterpret_cast<float *>(p + w.dv);
    a.bufs.iv = reinterpret_cast<float *>(p + w.iv);
    a.bufs.ssum = reinterpret_cast<double *>(p + w.ssum);
    a.bufs.gsum = reinterpret_cast<double *>(p + w.gsum);
    a.bufs.mixed = reinterpret_cast<uint16_t *>(p + w.mixed);
    a.bufs.act = reinterpret_cast<uint16_t *>(p + w.act);
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
