// Token loop around the MoE stack (the step after the routed block: the reference's greedy /
// sampled decode loop, mlx-qwen38/server.py:93-110 `_sample_next_token` and
// server.py:113-199 `_generate_stream_impl`, loader.py:1125-1244 `generate_greedy`):
//   embed_kernel      token ids -> bf16 rows of the embedding table
//   lm_head_kernel    bf16 [V, H] head x bf16 rows -> fp32 logits; every product of two bf16
//                     values is exact in fp32, the H products of a row are summed in fp64 in a
//                     fixed order (lane-strided 8-element chunks, then a butterfly over the 32
//                     lanes) and rounded once to fp32, so the logits do not depend on the launch
//   sample_kernel     temperature <= 0: argmax (first index of the maximum, as mx.argmax);
//                     temperature > 0: scaled = logits / temperature, optional top-p set (the
//                     largest probabilities whose mass reaches top_p, found by bisection on the
//                     fp32 bit pattern of exp(scaled - max)), then one categorical draw by the
//                     Gumbel-max rule with a counter-based hash of (seed, counter, row, index)
// HBM-bound: the head is the only large read (V x H x 2 bytes per step).
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"
#include "moe_b200.h"

namespace {

constexpr int kHeadThreads = 256;            // 8 warps, one row per warp at a time
// rows per warp and the chunk-loop unroll (below): 8 and 4 measured best on B200 for the
// 248,320 x 3072 head (321 us, 4.75 TB/s; unroll 2 with 4 rows 573 us at 86 registers, unroll 6
// 326 us, unroll 12 459 us)
#ifndef MOE_HEAD_ROWS_PER_WARP
#define MOE_HEAD_ROWS_PER_WARP 8
#endif
constexpr int kHeadRowsPerWarp = MOE_HEAD_ROWS_PER_WARP;
constexpr int kMaxHeadRows = 4;              // token rows per launch (x staged in shared memory)
constexpr int kSampleThreads = 1024;

__global__ void embed_kernel(const uint16_t *__restrict__ table, int V, int H, const int32_t *__restrict__ ids,
                             uint16_t *__restrict__ out) {
    const int t = blockIdx.x;
    const int id = ids[t];
    const bool ok = id >= 0 && id < V;
    if (!ok && threadIdx.x == 0) atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
    const uint4 *src = reinterpret_cast<const uint4 *>(table + (size_t)(ok ? id : 0) * H);
    uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)t * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = ok ? __ldg(src + i) : make_uint4(0u, 0u, 0u, 0u);
}

// Order-preserving 32-bit image of a float (larger float -> larger unsigned).
MOE_D uint32_t f2ord(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// argmax key: larger logit first, then the smaller index (the first index of the maximum)
MOE_D unsigned long long argmax_key(float v, int idx) {
    return ((unsigned long long)f2ord(v) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

// logits[t][v] = fp32( sum_h fp64(w[v][h] * x[t][h]) ), lane l of the row's warp summing its
// chunks h = 8 * (l + 32 i) .. +7 in order, then lanes combined by xor-butterfly 16, 8, 4, 2, 1.
// The chunk loop is unrolled kU deep so that kU loads per lane are in flight. best (optional)
// [T]: the argmax key of each token row, folded in with one 64-bit atomicMax per CTA and row
// (zero before the launch).
#ifndef MOE_HEAD_UNROLL
#define MOE_HEAD_UNROLL 4
#endif
constexpr int kHeadUnroll = MOE_HEAD_UNROLL;

__global__ void __launch_bounds__(kHeadThreads)
lm_head_kernel(const uint16_t *__restrict__ w, int V, int H, const uint16_t *__restrict__ x, int T,
               float *__restrict__ logits, unsigned long long *__restrict__ best) {
    // x staged k-major, xs[t][k][c] = x[t][8 c + k], so lane-consecutive chunks read
    // consecutive words (no bank conflicts)
    extern __shared__ float xs[];                                   // [T][8][H / 8]
    __shared__ unsigned long long sbest[kMaxHeadRows][kHeadThreads / 32];
    const int nch = H / 8;
    for (int i = threadIdx.x; i < T * H; i += blockDim.x) {
        const int t = i / H, h = i % H;
        xs[(t * 8 + (h & 7)) * nch + (h >> 3)] = bf16_bits_to_f32(x[i]);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = (blockIdx.x * (kHeadThreads / 32) + warp) * kHeadRowsPerWarp;
    unsigned long long wbest[kMaxHeadRows] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll 1
    for (int r = 0; r < kHeadRowsPerWarp; ++r) {
        const int v = row0 + r;
        if (v >= V) break;                                          // warp-uniform
        const uint4 *wr = reinterpret_cast<const uint4 *>(w + (size_t)v * H);
        double acc[kMaxHeadRows] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll kHeadUnroll
        for (int c = lane; c < nch; c += 32) {
            const uint4 q = __ldcs(wr + c);
            const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int t = 0; t < kMaxHeadRows; ++t) {
                if (t < T) {
                    const float *xr = xs + (size_t)t * 8 * nch + c;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[t] += (double)(__uint_as_float(wv[j] << 16) * xr[(2 * j) * nch]);
                        acc[t] += (double)(__uint_as_float(wv[j] & 0xffff0000u) * xr[(2 * j + 1) * nch]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kMaxHeadRows; ++t) {
            if (t < T) {
                double a = acc[t];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
                const float lv = (float)a;
                if (lane == 0 && logits) logits[(size_t)t * V + v] = lv;
                wbest[t] = max(wbest[t], argmax_key(lv, v));
            }
        }
    }
    if (best) {
        if (lane == 0) {
#pragma unroll
            for (int t = 0; t < kMaxHeadRows; ++t)
                if (t < T) sbest[t][warp] = wbest[t];
        }
        __syncthreads();
        if (threadIdx.x < T) {
            unsigned long long b = 0ull;
            for (int w8 = 0; w8 < kHeadThreads / 32; ++w8) b = max(b, sbest[threadIdx.x][w8]);
            if (b) atomicMax(best + threadIdx.x, b);
        }
    }
}

// ids[t] from the folded argmax keys; clears the keys for the next launch
__global__ void best_to_ids_kernel(unsigned long long *best, int T, int V, int32_t *ids) {
    const int t = threadIdx.x;
    if (t < T) {
        const unsigned long long b = best[t];
        const uint32_t idx = 0xffffffffu - (uint32_t)(b & 0xffffffffull);
        ids[t] = (b != 0ull && idx < (uint32_t)V) ? (int32_t)idx : 0;
        best[t] = 0ull;
    }
}

MOE_D uint64_t mix64(uint64_t z) {                                   // splitmix64 finaliser
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// uniform in (0, 1) from (seed, counter, row, index)
MOE_D double uniform01(uint64_t seed, uint64_t counter, int row, int v) {
    const uint64_t z = mix64(mix64(seed ^ (counter * 0x9e3779b97f4a7c15ull)) ^
                             (((uint64_t)(uint32_t)row << 32) | (uint32_t)v));
    return ((double)(z >> 11) + 0.5) * 0x1.0p-53;
}

// (value, index) pairs: larger value first, then the smaller index
MOE_D bool better(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

struct ArgMax {
    float v;
    int i;
};

MOE_D ArgMax block_argmax(ArgMax m, float *sv, int *si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, m.v, off);
        const int oi = __shfl_xor_sync(0xffffffffu, m.i, off);
        if (better(ov, oi, m.v, m.i)) { m.v = ov; m.i = oi; }
    }
    __syncthreads();
    if (lane == 0) { sv[warp] = m.v; si[warp] = m.i; }
    __syncthreads();
    m.v = sv[0]; m.i = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (better(sv[w], si[w], m.v, m.i)) { m.v = sv[w]; m.i = si[w]; }
    return m;
}

MOE_D double block_sum(double s, double *sd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    __syncthreads();
    if (lane == 0) sd[warp] = s;
    __syncthreads();
    s = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += sd[w];
    return s;
}

// one CTA per token row; prob [T][V] is scratch (exp(scaled - max), temperature > 0 only)
__global__ void __launch_bounds__(kSampleThreads)
sample_kernel(const float *__restrict__ logits, int V, float temperature, float top_p, uint64_t seed,
              uint64_t counter, int32_t *__restrict__ ids, float *__restrict__ prob) {
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ double sd[32];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *lg = logits + (size_t)t * V;
    if (!(temperature > 0.f)) {
        ArgMax m{-INFINITY, V};
        for (int v = tid; v < V; v += blockDim.x) {
            const float x = lg[v];
            if (better(x, v, m.v, m.i)) { m.v = x; m.i = v; }
        }
        m = block_argmax(m, sv, si);
        if (tid == 0) ids[t] = m.i < V ? m.i : 0;
        return;
    }
    float *p = prob + (size_t)t * V;
    ArgMax m{-INFINITY, V};
    for (int v = tid; v < V; v += blockDim.x) {
        const float s = lg[v] / temperature;
        if (better(s, v, m.v, m.i)) { m.v = s; m.i = v; }
    }
    m = block_argmax(m, sv, si);
    const float smax = m.v;
    double z = 0.0;
    for (int v = tid; v < V; v += blockDim.x) {
        const float e = expf(lg[v] / temperature - smax);
        p[v] = e;
        z += (double)e;
    }
    z = block_sum(z, sd);
    // top-p: the largest threshold tau (a non-negative float, searched on its bit pattern)
    // whose set {p >= tau} still holds top_p of the mass; tau = 0 keeps every token
    uint32_t tau = 0u;
    if (top_p > 0.f && top_p < 1.f) {
        const double need = (double)top_p * z;
        uint32_t lo = 0u, hi = __float_as_uint(1.0f);               // mass(p >= 1.0) > 0 always
#pragma unroll 1
        while (lo < hi) {                                            // invariant: mass(p >= lo) >= need
            const uint32_t mid = lo + (hi - lo + 1u) / 2u;
            const float fm = __uint_as_float(mid);
            double s = 0.0;
            for (int v = tid; v < V; v += blockDim.x) s += p[v] >= fm ? (double)p[v] : 0.0;
            s = block_sum(s, sd);
            if (s >= need) lo = mid; else hi = mid - 1u;
        }
        tau = lo;
    }
    const float ftau = __uint_as_float(tau);
    ArgMax g{-INFINITY, V};
    for (int v = tid; v < V; v += blockDim.x) {
        if (p[v] >= ftau && p[v] > 0.f) {
            const double u = uniform01(seed, counter, t, v);
            const float key = (float)((double)(lg[v] / temperature) - log(-log(u)));
            if (better(key, v, g.v, g.i)) { g.v = key; g.i = v; }
        }
    }
    g = block_argmax(g, sv, si);
    // no finite candidate (logits / temperature overflowed): the argmax of the scaled logits, else 0
    if (tid == 0) ids[t] = g.i < V ? g.i : (m.i < V ? m.i : 0);
}

}  // namespace

extern "C" int moe_embed_tokens(const void *table, int V, int H, const int32_t *ids, int T, void *out, void *stream) {
    if (!table || !ids || !out) return moe_set_error(MOE_EINVAL, "embed: null pointer");
    if (V <= 0 || H <= 0 || H % 8 || T <= 0) return moe_set_error(MOE_EINVAL, "embed: bad sizes V=%d H=%d T=%d", V, H, T);
    if ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15)
        return moe_set_error(MOE_EINVAL, "embed: table/out must be 16-byte aligned");
    embed_kernel<<<T, 256, 0, as_stream(stream)>>>(static_cast<const uint16_t *>(table), V, H, ids,
                                                   static_cast<uint16_t *>(out));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MOE_OK : moe_set_cuda_error(e);
}

static int launch_lm_head(const void *w, int V, int H, const void *x, int T, float *logits,
                          unsigned long long *best, void *stream) {
    if (!w || !x) return moe_set_error(MOE_EINVAL, "lm head: null pointer");
    if (V <= 0 || H <= 0 || H % 8 || T <= 0 || T > kMaxHeadRows)
        return moe_set_error(MOE_EINVAL, "lm head: bad sizes V=%d H=%d T=%d (T <= %d)", V, H, T, kMaxHeadRows);
    if (reinterpret_cast<uintptr_t>(w) & 15) return moe_set_error(MOE_EINVAL, "lm head: w must be 16-byte aligned");
    const size_t smem = (size_t)T * H * sizeof(float);
    if (smem > 160u * 1024u) return moe_set_error(MOE_EINVAL, "lm head: T*H=%d too large", T * H);
    const int rows_per_block = (kHeadThreads / 32) * kHeadRowsPerWarp;
    const int grid = (V + rows_per_block - 1) / rows_per_block;
    auto kern = lm_head_kernel;
    if (smem > 48u * 1024u)
        MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, kHeadThreads, smem, as_stream(stream)>>>(static_cast<const uint16_t *>(w), V, H,
                                                           static_cast<const uint16_t *>(x), T, logits, best);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MOE_OK : moe_set_cuda_error(e);
}

extern "C" int moe_lm_head_logits(const void *w, int V, int H, const void *x, int T, float *logits, void *stream) {
    if (!logits) return moe_set_error(MOE_EINVAL, "lm head: null logits");
    return launch_lm_head(w, V, H, x, T, logits, nullptr, stream);
}

extern "C" size_t moe_lm_head_argmax_workspace_bytes(int T) { return T > 0 ? (size_t)T * 8u : 0u; }

extern "C" int moe_lm_head_argmax(const void *w, int V, int H, const void *x, int T, float *logits, int32_t *ids,
                                  void *workspace, size_t workspace_bytes, void *stream) {
    if (!ids) return moe_set_error(MOE_EINVAL, "lm head argmax: null ids");
    if (!workspace || workspace_bytes < moe_lm_head_argmax_workspace_bytes(T) ||
        (reinterpret_cast<uintptr_t>(workspace) & 7))
        return moe_set_error(MOE_EINVAL, "lm head argmax: an 8-byte aligned workspace of %zu bytes is needed",
                             moe_lm_head_argmax_workspace_bytes(T));
    unsigned long long *best = static_cast<unsigned long long *>(workspace);
    const int rc = launch_lm_head(w, V, H, x, T, logits, best, stream);
    if (rc != MOE_OK) return rc;
    best_to_ids_kernel<<<1, 32, 0, as_stream(stream)>>>(best, T, V, ids);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MOE_OK : moe_set_cuda_error(e);
}

extern "C" size_t moe_sample_workspace_bytes(int T, int V) {
    if (T <= 0 || V <= 0) return 0;
    return (size_t)T * V * sizeof(float);
}

extern "C" int moe_sample_tokens(const float *logits, int T, int V, float temperature, float top_p, uint64_t seed,
                                 uint64_t counter, int32_t *ids, void *workspace, size_t workspace_bytes,
                                 void *stream) {
    if (!logits || !ids) return moe_set_error(MOE_EINVAL, "sample: null pointer");
    if (T <= 0 || V <= 0) return moe_set_error(MOE_EINVAL, "sample: bad sizes T=%d V=%d", T, V);
    if (temperature > 0.f && (!workspace || workspace_bytes < moe_sample_workspace_bytes(T, V)))
        return moe_set_error(MOE_EINVAL, "sample: workspace of %zu bytes needed, %zu given",
                             moe_sample_workspace_bytes(T, V), workspace_bytes);
    if (!(top_p > 0.f) || top_p > 1.f) return moe_set_error(MOE_EINVAL, "sample: top_p must be in (0, 1]");
    sample_kernel<<<T, kSampleThreads, 0, as_stream(stream)>>>(logits, V, temperature, top_p, seed, counter, ids,
                                                                static_cast<float *>(workspace));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? MOE_OK : moe_set_cuda_error(e);
}
