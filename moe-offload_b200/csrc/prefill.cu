// Prefill experts: T tokens x K routed experts as expert-grouped GEMMs on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM).
//
// Reference semantics: the prefill branch of CachedSwitchGLU (mlx-qwen38/loader.py:566-699;
// C++ run_moe_prefill, cpp/src/layers.cpp:403-600) sorts the (token, k) assignments by
// expert and runs gather_qmm per expert group (prefill_qproj.py:18-40), then unsorts and
// weights by the routing scores. Here:
//
//   bucket   assignments grouped by expert (counts, exclusive scan, scatter) and a tile list
//            (expert, 128-row block of the weight matrix, block of <= 256 of its tokens)
//   gateup   per tile D_g = Wg[rows] . X^T and D_u = Wu[rows] . X^T with M = 128 weight rows
//            and N = the expert's tokens (padded to 16): the 2-bit codes are dequantised to
//            bf16 (w = s*q + b, one rounding) straight into shared memory in the canonical
//            K-major core-matrix layout, the tokens' rows of x are gathered next to them,
//            one thread issues the MMAs (K = 16 each) into two TMEM accumulators, and the
//            epilogue (tcgen05.ld) applies SwiGLU with MLX's bf16 roundings -> act[pos][I]
//   down     the same GEMM with Wd and the act rows (contiguous per expert) -> yk[pos][H]
//   combine  y[t] = resid[t] + sum_k bf16(yk[pos(t,k)] * s[t,k]), sequential bf16 in MLX order
//
// Shared memory per K-block stage (64 columns of K): A = 128 rows x 64 bf16 per weight
// matrix (16 KB), B = up to 256 token rows x 64 bf16 (32 KB); two stages alternate so the
// dequantisation of block kb+1 overlaps the MMAs of block kb (tcgen05.commit -> mbarrier).
#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kBM = 128;          // weight rows per tile (MMA M)
constexpr int kBK = 64;           // K per stage (one 2-bit group)
constexpr int kMaxBN = 256;       // tokens per tile (MMA N)
constexpr int kATile = kBM * kBK * 2;          // 16 KB
constexpr int kBTile = kMaxBN * kBK * 2;       // 32 KB
constexpr uint32_t kTmemCols = 512;

// ------------------------------------------------------------------ tcgen05 helpers (PTX)

MOE_D uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // K-major, no swizzle: start, leading (K-chunk) and stride (8-row group) byte offsets in
    // 16-byte units, descriptor version 1 (bits 46-47), layout type 0 (bits 61-63)
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// instruction descriptor, kind::f16: D f32, A and B bf16, both K-major, N, M = 128
MOE_HD uint32_t instr_desc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

MOE_D void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

MOE_D void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

MOE_D void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

MOE_D void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MOE_D void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ------------------------------------------------------------------ bucketing

struct Tile {
    int e, row0, pos0, n;   // expert, first weight row, first assignment position, tokens
};

__global__ void count_kernel(const uint32_t *inds, int TK, int E, int *counts) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < TK; i += gridDim.x * blockDim.x) {
        const uint32_t e = inds[i];
        if (e < (uint32_t)E) atomicAdd(&counts[e], 1);
        else atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
    }
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024); returns the total.
MOE_D int block_excl_scan(int v, int *warp_sums, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    int inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += o;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, w, off);
            if (lane >= off) w += o;
        }
        if (lane < nw) warp_sums[lane] = w;        // inclusive warp prefix
    }
    __syncthreads();
    const int base = warp > 0 ? warp_sums[warp - 1] : 0;
    total = warp_sums[nw - 1];
    __syncthreads();
    return base + inc - v;
}

// One block of 1024 threads, experts in chunks of 1024: exclusive scan of the counts and
// the tile lists of both GEMMs (tiles of expert e are contiguous, in row-block order).
__global__ void __launch_bounds__(1024) scan_kernel(const int *counts, int E, int R1, int R2, int *offsets,
                                                    int *cursor, Tile *tiles1, int *ntiles1, Tile *tiles2,
                                                    int *ntiles2) {
    __shared__ int ws[32];
    int off0 = 0, t10 = 0, t20 = 0;
    const int rb1 = (R1 + kBM - 1) / kBM, rb2 = (R2 + kBM - 1) / kBM;
    for (int e0 = 0; e0 < E; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        const int c = (e < E) ? counts[e] : 0;
        const int nb = (c + kMaxBN - 1) / kMaxBN;
        int tot_c, tot_1, tot_2;
        const int o = block_excl_scan(c, ws, tot_c) + off0;
        const int s1 = block_excl_scan(nb * rb1, ws, tot_1) + t10;
        const int s2 = block_excl_scan(nb * rb2, ws, tot_2) + t20;
        if (e < E) {
            offsets[e] = o;
            cursor[e] = 0;
            int i1 = s1, i2 = s2;
            for (int p = 0; p < c; p += kMaxBN) {
                const int n = min(kMaxBN, c - p);
                for (int r = 0; r < rb1; ++r) tiles1[i1++] = Tile{e, r * kBM, o + p, n};
                for (int r = 0; r < rb2; ++r) tiles2[i2++] = Tile{e, r * kBM, o + p, n};
            }
        }
        off0 += tot_c;
        t10 += tot_1;
        t20 += tot_2;
    }
    if (threadIdx.x == 0) {
        offsets[E] = off0;
        *ntiles1 = t10;
        *ntiles2 = t20;
    }
}

// assignment i = t*K + k goes to position offsets[e] + (arrival order within e)
__global__ void scatter_kernel(const uint32_t *inds, int TK, int E, const int *offsets, int *cursor, int *pos_of,
                               int *src_of) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < TK; i += gridDim.x * blockDim.x) {
        const uint32_t e = inds[i];
        if (e >= (uint32_t)E) continue;
        const int p = offsets[e] + atomicAdd(&cursor[e], 1);
        pos_of[i] = p;
        src_of[p] = i;
    }
}

// ------------------------------------------------------------------ grouped GEMM

struct GemmArgs {
    const Tile *tiles;
    const int *ntiles;
    int Kdim, R;                      // reduction length, weight rows per expert
    const uint32_t *w0, *w1;          // codes [E][R][Kdim/16] (w1: up, gate/up GEMM only)
    const uint16_t *s0, *b0, *s1, *b1;
    const uint16_t *xrows;            // B rows: x [T][Kdim] (gather via src_of / K) or act [pos][Kdim]
    const int *src_of;                // gate/up: assignment index of each position (token = idx / K)
    int K;
    uint16_t *out;                    // gate/up: act [pos][R]; down: yk [pos][R]
};

// Dequantises chunks [c0, c0 + nc) (8 codes each) of tile row r for K-block kb (group kb of
// the row) into the canonical K-major layout: element (row, k) at chunk (k / 8) * LBO +
// (row / 8) * 128 + (row % 8) * 16 + (k % 8) * 2, LBO = 128 / 8 * 128 = 2048 bytes.
// w = bf16(s * q + b), one rounding.
template <bool kFp16>
MOE_D void dequant_row(const uint32_t *w, const uint16_t *s, const uint16_t *b, int row0, int e, int R, int Kdim,
                       int kb, unsigned char *dst, int r, int c0, int nc) {
    const int row = row0 + r;
    uint32_t words[4] = {0u, 0u, 0u, 0u};
    float sc = 0.f, bi = 0.f;
    if (row < R) {
        const uint4 q = *reinterpret_cast<const uint4 *>(w + ((size_t)e * R + row) * (Kdim / 16) + (size_t)kb * 4);
        words[0] = q.x;
        words[1] = q.y;
        words[2] = q.z;
        words[3] = q.w;
        const size_t si = ((size_t)e * R + row) * (Kdim / 64) + kb;
        sc = sb_to_f32<kFp16>(s[si]);
        bi = sb_to_f32<kFp16>(b[si]);
    }
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
        if (cc < c0 || cc >= c0 + nc) continue;
        const uint32_t bits = words[cc >> 1] >> ((cc & 1) * 16);     // codes 8cc .. 8cc+7
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float v0 = fmaf(sc, (float)((bits >> (4 * j)) & 3u), bi);
            const float v1 = fmaf(sc, (float)((bits >> (4 * j + 2)) & 3u), bi);
            o[j] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
        }
        *reinterpret_cast<uint4 *>(dst + cc * 2048 + (r >> 3) * 128 + (r & 7) * 16) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// B stage: n token rows x 64 bf16 of K-block kb, zero beyond n; layout chunk c at c * LBOB,
// LBOB = BN / 8 * 128
MOE_D void load_b_stage(const uint16_t *xrows, const int *src_of, int K, bool gather, int pos0, int n, int BN,
                        int Kdim, int kb, unsigned char *dst, int tid_in, int nthr) {
    const uint32_t lbo = (uint32_t)(BN / 8) * 128u;
    for (int it = tid_in; it < BN * 8; it += nthr) {
        const int tok = it % BN, c = it / BN;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (tok < n) {
            const int p = pos0 + tok;
            const size_t row = gather ? (size_t)(src_of[p] / K) : (size_t)p;
            v = *reinterpret_cast<const uint4 *>(xrows + row * Kdim + (size_t)kb * 64 + c * 8);
        }
        *reinterpret_cast<uint4 *>(dst + c * lbo + (tok >> 3) * 128 + (tok & 7) * 16) = v;
    }
}

template <bool kGateUp, bool kFp16>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(GemmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    constexpr int nA = kGateUp ? 2 : 1;
    unsigned char *stA[2], *stB[2];
    for (int s = 0; s < 2; ++s) {
        stA[s] = smem + s * (nA * kATile + kBTile);
        stB[s] = stA[s] + nA * kATile;
    }
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + 2 * (nA * kATile + kBTile));   // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(mbar + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tslot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    uint32_t phase[2] = {0u, 0u};
    int uses[2] = {0, 0};
    const int ntiles = *a.ntiles;
    const int nkb = a.Kdim / kBK;

    for (int ti = blockIdx.x; ti < ntiles; ti += gridDim.x) {
        const Tile tl = a.tiles[ti];
        const int BN = (tl.n + 15) & ~15;
        const uint32_t idesc = instr_desc_bf16(BN);
        const uint32_t lboB = (uint32_t)(BN / 8) * 128u;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb & 1;
            // the MMAs that read this stage two blocks ago must be done
            if (uses[s] > 0) {
                mbar_wait(&mbar[s], phase[s]);
                phase[s] ^= 1u;
                uses[s] = 0;
            }
            if (kGateUp) {           // threads 0..127: gate row tid, 128..255: up row tid - 128
                if (tid < kBM) dequant_row<kFp16>(a.w0, a.s0, a.b0, tl.row0, tl.e, a.R, a.Kdim, kb, stA[s], tid, 0, 8);
                else dequant_row<kFp16>(a.w1, a.s1, a.b1, tl.row0, tl.e, a.R, a.Kdim, kb, stA[s] + kATile, tid - kBM, 0, 8);
            } else {                 // row tid % 128, chunks 0..3 or 4..7
                dequant_row<kFp16>(a.w0, a.s0, a.b0, tl.row0, tl.e, a.R, a.Kdim, kb, stA[s], tid & (kBM - 1),
                                   (tid >> 7) * 4, 4);
            }
            load_b_stage(a.xrows, a.src_of, a.K, kGateUp, tl.pos0, tl.n, BN, a.Kdim, kb, stB[s], tid, kThreads);
            fence_barrier_init();        // generic-proxy smem writes -> visible to the tensor core (async proxy)
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t aaddr = smem_addr(stA[s]), baddr = smem_addr(stB[s]);
#pragma unroll
                for (int j = 0; j < kBK / 16; ++j) {
                    const uint64_t bd = smem_desc(baddr + 2 * j * lboB, lboB, 128);
                    const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
                    mma_bf16(tmem, smem_desc(aaddr + 2 * j * 2048, 2048, 128), bd, idesc, acc);
                    if (kGateUp)
                        mma_bf16(tmem + 256, smem_desc(aaddr + kATile + 2 * j * 2048, 2048, 128), bd, idesc, acc);
                }
                mma_commit(&mbar[s]);
            }
            uses[s] = 1;
        }
        // wait for the last block's MMAs (the commit of the final stage covers all earlier ones)
        const int sl = (nkb - 1) & 1;
        mbar_wait(&mbar[sl], phase[sl]);
        phase[sl] ^= 1u;
        uses[sl] = 0;
        if (nkb > 1 && uses[sl ^ 1]) {
            mbar_wait(&mbar[sl ^ 1], phase[sl ^ 1]);
            phase[sl ^ 1] ^= 1u;
            uses[sl ^ 1] = 0;
        }
        tc_fence_after();
        // epilogue: warps 0..3 own TMEM lanes 32w..32w+31 = weight rows of the tile
        if (warp < 4) {
            const int r = warp * 32 + lane;
            const int row = tl.row0 + r;
            const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float g[16], u[16];
                tmem_ld16(lane_addr + c0, g);
                if (kGateUp) tmem_ld16(lane_addr + 256 + c0, u);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int tok = c0 + j;
                    if (tok < tl.n && row < a.R) {
                        float v;
                        if (kGateUp) {
                            const float gv = bf16r(g[j]), uv = bf16r(u[j]);
                            const float sig = bf16r(1.0f / (1.0f + expf(-gv)));
                            v = bf16r(bf16r(gv * sig) * uv);
                        } else {
                            v = bf16r(g[j]);
                        }
                        a.out[(size_t)(tl.pos0 + tok) * a.R + row] = f32_to_bf16_bits(v);
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// y[t][h] = bf16(resid + sum_k bf16(yk * s_k)) with the k sum sequential in bf16 (MLX order)
__global__ void combine_kernel(const uint16_t *yk, const int *pos_of, const uint16_t *scores, const uint16_t *resid,
                               int T, int K, int H, uint16_t *y) {
    const size_t n = (size_t)T * H;
    const int TK = T * K;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / H), h = (int)(i % H);
        float acc = 0.f;
        for (int k = 0; k < K; ++k) {
            const int p = pos_of[t * K + k];
            if (p < 0 || p >= TK) {            // an expert id >= E was never scattered
                atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
                continue;
            }
            const float pk = bf16r(bf16_bits_to_f32(yk[(size_t)p * H + h]) * bf16_bits_to_f32(scores[t * K + k]));
            acc = (k == 0) ? pk : bf16r(acc + pk);
        }
        if (resid) acc = bf16r(bf16_bits_to_f32(resid[i]) + acc);
        y[i] = f32_to_bf16_bits(acc);
    }
}

struct PrefillWs {
    int *counts, *offsets, *cursor, *pos_of, *src_of, *ntiles;
    Tile *tiles1, *tiles2;
    uint16_t *act, *yk;
    size_t bytes;
};

PrefillWs carve(void *base, int T, int H, int I, int E, int K) {
    PrefillWs w{};
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t n) { char *q = p ? p + off : nullptr; off += al256(n); return q; };
    const size_t TK = (size_t)T * K;
    const size_t maxt = (size_t)E + TK / kMaxBN + 1;     // token blocks
    w.counts = reinterpret_cast<int *>(take((size_t)E * 4));
    w.offsets = reinterpret_cast<int *>(take((size_t)(E + 1) * 4));
    w.cursor = reinterpret_cast<int *>(take((size_t)E * 4));
    w.pos_of = reinterpret_cast<int *>(take(TK * 4));
    w.src_of = reinterpret_cast<int *>(take(TK * 4));
    w.ntiles = reinterpret_cast<int *>(take(2 * 4));
    w.tiles1 = reinterpret_cast<Tile *>(take(maxt * ((I + kBM - 1) / kBM) * sizeof(Tile)));
    w.tiles2 = reinterpret_cast<Tile *>(take(maxt * ((H + kBM - 1) / kBM) * sizeof(Tile)));
    w.act = reinterpret_cast<uint16_t *>(take(TK * I * 2));
    w.yk = reinterpret_cast<uint16_t *>(take(TK * H * 2));
    w.bytes = off;
    return w;
}

size_t gemm_smem(bool gateup) {
    return 2 * ((gateup ? 2 : 1) * kATile + kBTile) + 64;
}

}  // namespace

// x_n[t] = x[t] * 2^-k(t), the power-of-two RMS normalisation of every row (exact)
static __global__ void __launch_bounds__(256) pow2_rows_kernel(const uint16_t *x, int H, uint16_t *xn) {
    __shared__ double red[8];
    const int t = blockIdx.x;
    const uint16_t *xr = x + (size_t)t * H;
    double ss = 0.0;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const double v = (double)bf16_bits_to_f32(xr[i]);
        ss = fma(v, v, ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += red[i];
    const float mul = ldexpf(1.0f, -pow2_rms_shift(ss, H));
    for (int i = threadIdx.x; i < H; i += blockDim.x) xn[(size_t)t * H + i] = f32_to_bf16_bits(bf16_bits_to_f32(xr[i]) * mul);
}

static size_t layer_prefix_bytes(int T, int H, int E) {
    return al256((size_t)T * 4) + al256((size_t)T * E * 2) + al256((size_t)T * H * 2);
}

extern "C" size_t moe_prefill_workspace_bytes(int T, int H, int I, int E, int K) {
    if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || K <= 0) return 0;
    return carve(nullptr, T, H, I, E, K).bytes;
}

extern "C" int moe_prefill_experts(const void *x, int T, int H, int I, int E, int K, const uint32_t *inds,
                                   const void *scores, const uint32_t *wg, const void *sg, const void *bg,
                                   const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                                   const void *sd, const void *bd, int sb_fp16, const void *resid, void *y,
                                   void *act_out, void *workspace, size_t workspace_bytes, void *stream) {
    if (!x || !inds || !scores || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !y || !workspace)
        return moe_set_error(MOE_EINVAL, "prefill_experts: null pointer");
    if (T <= 0 || E <= 0 || K <= 0 || K > 64 || H % 64 || I % 64 || H < 64 || I < 64)
        return moe_set_error(MOE_EINVAL, "prefill_experts: bad sizes T=%d H=%d I=%d E=%d K=%d", T, H, I, E, K);
    if (workspace_bytes < moe_prefill_workspace_bytes(T, H, I, E, K))
        return moe_set_error(MOE_EINVAL, "prefill_experts: workspace too small");
    const void *al16p[] = {x, wg, wu, wd};
    for (const void *p : al16p)
        if (reinterpret_cast<uintptr_t>(p) % 16)
            return moe_set_error(MOE_EINVAL, "prefill_experts: x and code arrays must be 16-byte aligned");
    PrefillWs w = carve(workspace, T, H, I, E, K);
    auto st = as_stream(stream);
    const int TK = T * K;
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    MOE_CUDA_TRY(cudaMemsetAsync(w.counts, 0, (size_t)E * 4, st));
    MOE_CUDA_TRY(cudaMemsetAsync(w.pos_of, 0xff, (size_t)TK * 4, st));
    count_kernel<<<(TK + 255) / 256, 256, 0, st>>>(inds, TK, E, w.counts);
    scan_kernel<<<1, 1024, 0, st>>>(w.counts, E, I, H, w.offsets, w.cursor, w.tiles1, w.ntiles, w.tiles2, w.ntiles + 1);
    scatter_kernel<<<(TK + 255) / 256, 256, 0, st>>>(inds, TK, E, w.offsets, w.cursor, w.pos_of, w.src_of);
    MOE_CUDA_TRY(cudaGetLastError());

    uint16_t *act = act_out ? static_cast<uint16_t *>(act_out) : w.act;
    GemmArgs g1{w.tiles1, w.ntiles, H, I, wg, wu, static_cast<const uint16_t *>(sg), static_cast<const uint16_t *>(bg),
                static_cast<const uint16_t *>(su), static_cast<const uint16_t *>(bu),
                static_cast<const uint16_t *>(x), w.src_of, K, act};
    GemmArgs g2{w.tiles2, w.ntiles + 1, I, H, wd, nullptr, static_cast<const uint16_t *>(sd),
                static_cast<const uint16_t *>(bd), nullptr, nullptr, act, nullptr, K, w.yk};
    const void *k1 = sb_fp16 ? (const void *)gemm_kernel<true, true> : (const void *)gemm_kernel<true, false>;
    const void *k2 = sb_fp16 ? (const void *)gemm_kernel<false, true> : (const void *)gemm_kernel<false, false>;
    static int configured = 0;
    if (!configured) {
        MOE_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem(true)));
        MOE_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem(true)));
        MOE_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem(false)));
        MOE_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem(false)));
        configured = 1;
    }
    void *a1[] = {&g1};
    void *a2[] = {&g2};
    MOE_CUDA_TRY(cudaLaunchKernel(k1, dim3(sms), dim3(kThreads), a1, gemm_smem(true), st));
    MOE_CUDA_TRY(cudaLaunchKernel(k2, dim3(sms), dim3(kThreads), a2, gemm_smem(false), st));
    combine_kernel<<<sms * 4, 256, 0, st>>>(w.yk, w.pos_of, static_cast<const uint16_t *>(scores),
                                             static_cast<const uint16_t *>(resid), T, K, H, static_cast<uint16_t *>(y));
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" size_t moe_prefill_layer_workspace_bytes(int T, int H, int I, int E, int K) {
    const size_t p = moe_prefill_workspace_bytes(T, H, I, E, K);
    return p ? layer_prefix_bytes(T, H, E) + p : 0;
}

extern "C" int moe_prefill_layer(const void *x, int T, int H, int I, int E, int K, const void *router_w,
                                 const uint32_t *wg, const void *sg, const void *bg, const uint32_t *wu,
                                 const void *su, const void *bu, const uint32_t *wd, const void *sd, const void *bd,
                                 int sb_fp16, int norm, const void *resid, uint32_t *out_inds, void *out_scores,
                                 void *y, void *workspace, size_t workspace_bytes, void *stream) {
    if (!x || !router_w || !out_inds || !out_scores || !y || !workspace)
        return moe_set_error(MOE_EINVAL, "prefill_layer: null pointer");
    const size_t need = moe_prefill_layer_workspace_bytes(T, H, I, E, K);
    if (!need || workspace_bytes < need)
        return moe_set_error(MOE_EINVAL, "prefill_layer: workspace of %zu bytes needed, %zu given", need,
                             workspace_bytes);
    char *ws = static_cast<char *>(workspace);
    unsigned int *tickets = reinterpret_cast<unsigned int *>(ws);
    uint16_t *logits = reinterpret_cast<uint16_t *>(ws + al256((size_t)T * 4));
    uint16_t *xn = reinterpret_cast<uint16_t *>(ws + al256((size_t)T * 4) + al256((size_t)T * E * 2));
    void *pws = ws + layer_prefix_bytes(T, H, E);
    const void *xin = x;
    if (norm) {
        pow2_rows_kernel<<<T, 256, 0, as_stream(stream)>>>(static_cast<const uint16_t *>(x), H, xn);
        MOE_CUDA_TRY(cudaGetLastError());
        xin = xn;
    }
    int rc = moe_router_launch(xin, T, H, E, K, router_w, nullptr, nullptr, 16, 64, 0, nullptr, nullptr, nullptr, 0,
                               nullptr, nullptr, nullptr, out_inds, out_scores, nullptr, tickets, logits, nullptr,
                               nullptr, nullptr, nullptr, 0, stream);
    if (rc) return rc;
    return moe_prefill_experts(xin, T, H, I, E, K, out_inds, out_scores, wg, sg, bg, wu, su, bu, wd, sd, bd, sb_fp16,
                               resid, y, nullptr, pws, workspace_bytes - layer_prefix_bytes(T, H, E), stream);
}
