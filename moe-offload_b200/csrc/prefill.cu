// Prefill experts: T tokens x K routed experts as expert-grouped GEMMs on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM), fed by TMA.
//
// Reference semantics: the prefill branch of CachedSwitchGLU (mlx-qwen38/loader.py:566-699;
// C++ run_moe_prefill, cpp/src/layers.cpp:403-600) sorts the (token, k) assignments by
// expert and runs gather_qmm per expert group (prefill_qproj.py:18-40), then unsorts and
// weights by the routing scores. Here:
//
//   bucket   assignments grouped by expert (counts, exclusive scan, scatter) and a tile list
//            (expert, row block of the weight matrix, block of <= 128 of its tokens)
//   gateup   per tile D_g = Wg[rows] . X^T and D_u = Wu[rows] . X^T, M = 128 weight rows each,
//            N = the expert's tokens (padded to 16), K = H in blocks of 64 (one 2-bit group)
//   down     the same GEMM with Wd (two 128-row blocks per tile) and the act rows
//            (contiguous per expert) -> yk[pos][H]
//   combine  y[t] = resid[t] + sum_k bf16(yk[pos(t,k)] * s[t,k]), sequential bf16 in MLX order
//
// The GEMM kernel is persistent (one CTA per SM) and warp-specialised:
//   warp 0      TMA producer: raw 2-bit codes of the tile's 128 rows, 8 K-blocks (128 bytes
//               of codes per row) per 2-D box, 128-byte swizzled; the B operand per K-block in
//               16-row boxes of expert-ordered rows (gate/up: x rows gathered into position
//               order by one copy kernel; down: the act rows), 128-byte swizzled
//   warps 6-13  dequantise one K-block of codes to bf16, w = bf16(s * q + b) with one
//               rounding, into TMEM (the A operand, lane = weight row): the four values of a
//               (row, group) are built once and every pair of codes becomes a bf16x2 word with
//               one byte permute (selectors built 8 codes at a time)
//   warp 1      one thread issues the tcgen05.mma (K = 16 each) into TMEM; the accumulators
//               are double-buffered across tiles
//   warps 2-5   epilogue: tcgen05.ld of the accumulators, SwiGLU with MLX's bf16 roundings
//               (gate/up) or the bf16 rounding (down), stores to global
// Stages hand over through mbarriers (TMA transaction counts, tcgen05.commit, warp
// arrivals); every wait is bounded. A K-block stage (its dequantised weights in TMEM and its
// token rows in shared memory) is one unit: the dequant warps wait for the tokens before they
// arrive, so the MMA thread waits on one barrier per K-block and frees the stage with one
// commit (two waits and two commits cost ~9 % more).
#include <cuda.h>

#include "common.cuh"
#include "internal.h"

namespace {

constexpr int kBM = 128;          // weight rows per tile (MMA M)
constexpr int kBK = 64;           // K per block (one 2-bit group)
constexpr int kMaxBN = 128;       // tokens per tile (MMA N)

// ------------------------------------------------------------------ tcgen05 / TMA helpers (PTX)

// Shared-memory matrix descriptor for a K-major operand in the 128-byte-swizzle layout: rows
// of 128 bytes (64 bf16 of K), 8-row groups 1024 bytes apart (stride byte offset), descriptor
// version 1 (bits 46-47), layout type 2 = SWIZZLE_128B (bits 61-63). The K = 16 steps inside
// a 64-wide block advance the start address by 32 bytes.
MOE_D uint64_t desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// instruction descriptor, kind::f16: D f32, A and B bf16, both K-major, N, M = 128
MOE_HD uint32_t instr_desc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// A from tensor memory (lane = row, two bf16 of K per 32-bit column), B from shared memory
MOE_D void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
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

// this warp's 32 TMEM lanes, 32 consecutive 32-bit columns from taddr
MOE_D void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

MOE_D void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

MOE_D void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MOE_D void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

MOE_D void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait that also gives up once another warp of the CTA has aborted (the flag is
// polled every 1024 tries). On its own timeout it records the device error and raises the
// CTA's abort flag. Warp-uniform result: every lane of the calling warp must call it.
MOE_D bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort) {
    bool ok = false, gave_up = false;
#pragma unroll 1
    for (uint32_t i = 0; i < kMbarSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) {
            ok = true;
            break;
        }
        if ((i & 1023u) == 1023u && *abort) {
            gave_up = true;
            break;
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) {                                             // warp-uniform branch
        const bool timed_out = !__any_sync(0xffffffffu, gave_up);
        if ((threadIdx.x & 31) == 0) {
            if (timed_out) atomicOr(&g_moe_device_error, MOE_DEVERR_MBAR_TIMEOUT);
            *abort = 1;
        }
    }
    return ok;
}

MOE_D bool aborted(volatile int *abort) { return __any_sync(0xffffffffu, *abort != 0); }

// 2-D tiled TMA load (no multicast) completing on an mbarrier; x is the innermost coordinate
MOE_D void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

MOE_D uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// byte offset of 16-byte chunk c of row r in a 128-byte-swizzled tile of 128-byte rows
MOE_D uint32_t sw128(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

// Dequantisation tables of one (row, group): tlo / thi hold the low / high bytes of the four
// bf16 values v_q = bf16(s * q + b), q = 0..3 (byte q).
template <bool kFp16>
MOE_D void dq_tables(uint16_t sraw, uint16_t braw, uint32_t &tlo, uint32_t &thi) {
    const float s = sb_to_f32<kFp16>(sraw), b = sb_to_f32<kFp16>(braw);
    const uint32_t p01 = (uint32_t)f32_to_bf16_bits(b) | ((uint32_t)f32_to_bf16_bits(s + b) << 16);
    const uint32_t p23 = (uint32_t)f32_to_bf16_bits(fmaf(s, 2.f, b)) | ((uint32_t)f32_to_bf16_bits(fmaf(s, 3.f, b)) << 16);
    tlo = prmt(p01, p23, 0x6420u);
    thi = prmt(p01, p23, 0x7531u);
}

// K order inside every 16-element group of the GEMMs: position 2c + j of the group holds
// element t + 8h + 4j for c = 2t + h (t < 4, h, j < 2), i.e. [0,4,8,12,1,5,9,13,2,6,10,14,3,7,
// 11,15]. A and B use the same order, so the products are unchanged; it lets one byte permute
// expand a pair of codes whose selector comes from one mask and one multiply-add.
MOE_HD int kperm_pos(int e) { return 4 * (e & 3) + 2 * ((e >> 3) & 1) + ((e >> 2) & 1); }

// 16 codes (code e in bits 2e..2e+1) -> 8 bf16x2 words in the permuted K order: word 2t + h
// = (v[code t + 8h], v[code t + 8h + 4]). Selector of the pair: nibbles [q, q + 4, q', q' + 4].
MOE_D void dq_word(uint32_t w, uint32_t tlo, uint32_t thi, uint32_t *o) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t S = ((w >> (2 * t)) & 0x03030303u) * 0x11u + 0x40404040u;
        o[2 * t] = prmt(tlo, thi, S);
        o[2 * t + 1] = prmt(tlo, thi, S >> 16);
    }
}

// ------------------------------------------------------------------ bucketing

struct Tile {
    int e, row0, pos0, n;   // expert, first weight row, first assignment position, tokens
};

// Warp-aggregated increment of ctr[e] by one per active lane: the lanes holding the same e
// make one atomic (routing can send most tokens to one expert); returns this lane's value of
// the counter before its own increment (the lanes of a group in lane order).
MOE_D int warp_agg_add(int *ctr, uint32_t e, unsigned active) {
    const unsigned grp = __match_any_sync(active, e);
    const int leader = __ffs(grp) - 1, lane = threadIdx.x & 31;
    int base = 0;
    if (lane == leader) base = atomicAdd(ctr + e, __popc(grp));
    base = __shfl_sync(grp, base, leader);
    return base + __popc(grp & ((1u << lane) - 1u));
}

// expert ids are taken relative to e_begin (a rank's block of the experts); ids outside
// [e_begin, e_begin + E) are skipped when `strict` is 0 and flagged as bad input otherwise
__global__ void count_kernel(const uint32_t *inds, int TK, int E, uint32_t e_begin, int strict, int *counts) {
    for (int i0 = blockIdx.x * blockDim.x; i0 < TK; i0 += gridDim.x * blockDim.x) {
        const int i = i0 + threadIdx.x;
        const uint32_t e = i < TK ? inds[i] - e_begin : 0xffffffffu;
        const bool ok = e < (uint32_t)E;
        const unsigned active = __ballot_sync(0xffffffffu, ok);
        if (ok) warp_agg_add(counts, e, active);
        else if (i < TK && strict) atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
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
    const int rb1 = (R1 + kBM - 1) / kBM, rb2 = (R2 + 2 * kBM - 1) / (2 * kBM);
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
                for (int r = 0; r < rb2; ++r) tiles2[i2++] = Tile{e, r * 2 * kBM, o + p, n};
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
__global__ void scatter_kernel(const uint32_t *inds, int TK, int E, uint32_t e_begin, const int *offsets, int *cursor,
                               int *pos_of, int *src_of) {
    for (int i0 = blockIdx.x * blockDim.x; i0 < TK; i0 += gridDim.x * blockDim.x) {
        const int i = i0 + threadIdx.x;
        const uint32_t e = i < TK ? inds[i] - e_begin : 0xffffffffu;
        const bool ok = e < (uint32_t)E;
        const unsigned active = __ballot_sync(0xffffffffu, ok);
        if (!ok) continue;
        const int p = offsets[e] + warp_agg_add(cursor, e, active);
        pos_of[i] = p;
        src_of[p] = i;
    }
}

// xs[p] = x[src_of[p] / K] in the permuted K order: the B rows of the gate/up GEMM in expert
// order, one 16-element group (two 16-byte chunks) per work item
__global__ void gather_rows_kernel(const uint16_t *x, const int *src_of, int TK, int K, int H, uint16_t *xs) {
    const int gpr = H / 16;
    const size_t n = (size_t)TK * gpr;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t p = i / gpr;
        const int gi = (int)(i % gpr);
        const int src = src_of[p];
        if (src < 0) continue;
        const uint4 *in = reinterpret_cast<const uint4 *>(x + (size_t)(src / K) * H + (size_t)gi * 16);
        const uint4 lo = in[0], hi = in[1];
        uint4 *out = reinterpret_cast<uint4 *>(xs + p * H + (size_t)gi * 16);
        out[0] = make_uint4(prmt(lo.x, lo.z, 0x5410u), prmt(hi.x, hi.z, 0x5410u), prmt(lo.x, lo.z, 0x7632u),
                            prmt(hi.x, hi.z, 0x7632u));
        out[1] = make_uint4(prmt(lo.y, lo.w, 0x5410u), prmt(hi.y, hi.w, 0x5410u), prmt(lo.y, lo.w, 0x7632u),
                            prmt(hi.y, hi.w, 0x7632u));
    }
}

// ------------------------------------------------------------------ grouped GEMM

constexpr int kRawK = 8;                         // K-blocks per raw code stage (128 B of codes per row)
constexpr int kRS = 2;                           // raw code stages
// K-block stages: the dequantised weights of stage s in TMEM (A) and the token rows of the
// same K-block in shared memory (B, TMA) are one unit, freed by one commit
constexpr int kKS = 4;
constexpr int kGemmThreads = 448;                // 14 warps
constexpr int kDqWarp0 = 6, kDqWarps = 8;
constexpr int kEpiWarp0 = 2;
constexpr int kTile = kBM * 128;                 // one 128-row x 128-byte tile: 16 KB
constexpr uint32_t kTmemCols = 512;
// TMEM columns: accumulators [0, 128) (gate, or down rows 0..127 of the tile) and [128, 256)
// (up, or down rows 128..255); the dequantised A operand of K-block stage s at 256 + 64 s
// (matrix 0: +0, matrix 1: +32; 32 columns = 64 bf16 of K). A tile of at most 64 tokens uses
// one half of each accumulator range (columns +0 or +64, alternating), so its MMAs can run while
// the epilogue still drains the previous tile from the other half; a wider tile takes both.
constexpr uint32_t kTmemA = 256, kTmemAStage = 64;

struct GemmArgs {
    const Tile *tiles;
    const int *ntiles;
    int Kdim, R, K;                   // reduction length, weight rows per expert, top-k
    const uint16_t *s0, *b0, *s1, *b1;   // scales / biases [E][R][Kdim/64] (1: up, gate/up only)
    uint16_t *out;                    // gate/up: act [pos][R]; down: yk [pos][R]
};

template <bool kGateUp>
struct GemmSmem {
    static constexpr int kNM = 2;   // weight matrices per tile: gate + up, or two 128-row blocks of down
    static constexpr size_t raw = 0;                                       // [kRS][kNM] tiles
    static constexpr size_t b = raw + (size_t)kRS * kNM * kTile;           // [kKS] tiles
    static constexpr size_t bars = b + (size_t)kKS * kTile;
    // raw_full, raw_empty [kRS]; full, empty, b_full [kKS]; acc_full, acc_empty [2]
    // (accumulator halves); drain (MMA completion after an abort); tmem slot, abort flag
    static constexpr size_t total = bars + (2 * kRS + 3 * kKS + 5) * 8 + 16;
    static constexpr size_t alloc = total + 1024;      // + alignment slack
};

template <bool kGateUp, bool kFp16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_w0, const __grid_constant__ CUtensorMap map_w1,
                const __grid_constant__ CUtensorMap map_b, GemmArgs a) {
    using SL = GemmSmem<kGateUp>;
    constexpr int kNM = SL::kNM;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(smem + SL::bars);
    uint64_t *raw_empty = raw_full + kRS;
    uint64_t *full = raw_empty + kRS;
    uint64_t *empty = full + kKS;
    uint64_t *b_full = empty + kKS;
    uint64_t *acc_full = b_full + kKS;           // [2]
    uint64_t *acc_empty = acc_full + 2;          // [2]
    uint64_t *drain = acc_empty + 2;             // [1]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(drain + 1);
    // set by the first failed wait of any role: every role then stops, the epilogue stores
    // nothing, and the producer / MMA issuer drain what they already issued before exit
    volatile int *abort = reinterpret_cast<volatile int *>(tslot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < kRS; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kDqWarps);
        }
        for (int i = 0; i < kKS; ++i) {
            mbar_init(&full[i], kDqWarps);       // dequantised stage written and its tokens landed
            mbar_init(&empty[i], 1);             // the stage's MMAs done (one commit)
            mbar_init(&b_full[i], 1);            // the stage's token rows landed (TMA)
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&acc_full[h], 1);
            mbar_init(&acc_empty[h], 4);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tslot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const int ntiles = *a.ntiles;
    const int nkb = a.Kdim / kBK;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        uint32_t g = 0, rc = 0;
        bool stop = false;
        for (int ti = blockIdx.x; ti < ntiles && !stop; ti += gridDim.x) {
            const Tile tl = a.tiles[ti];
            const int wrow = tl.e * a.R + tl.row0;
            const int nbox = (tl.n + 15) >> 4;
            for (int kb = 0; kb < nkb; ++kb) {
                if (kb % kRawK == 0) {
                    const int rs = rc % kRS;
                    if (aborted(abort) || !wait_or_abort(&raw_empty[rs], ((rc / kRS) & 1u) ^ 1u, abort)) {
                        stop = true;
                        break;
                    }
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&raw_full[rs], kNM * kTile);
                        tma_load_2d(smem + SL::raw + (size_t)(rs * kNM) * kTile, &map_w0, kb * 4, wrow, &raw_full[rs]);
                        tma_load_2d(smem + SL::raw + (size_t)(rs * kNM + 1) * kTile, kGateUp ? &map_w1 : &map_w0,
                                    kb * 4, kGateUp ? wrow : wrow + kBM, &raw_full[rs]);
                    }
                    ++rc;
                }
                const int s = g % kKS;
                if (!wait_or_abort(&empty[s], ((g / kKS) & 1u) ^ 1u, abort)) {
                    stop = true;
                    break;
                }
                unsigned char *bst = smem + SL::b + (size_t)s * kTile;
                if (lane == 0) mbar_arrive_expect_tx(&b_full[s], (uint32_t)nbox * 2048u);
                __syncwarp();
                // the tile's B rows: 16-row boxes of the expert-ordered rows (x gathered per
                // position for gate/up, act for down)
                if (lane < nbox) tma_load_2d(bst + (size_t)lane * 2048, &map_b, kb * 64, tl.pos0 + 16 * lane, &b_full[s]);
                ++g;
            }
        }
        if (aborted(abort)) {
            // no bulk copy may still be writing shared memory when the CTA exits: wait (bounded)
            // for the last load issued into every stage; earlier ones completed before their
            // stage was reissued
            for (uint32_t i = rc > (uint32_t)kRS ? rc - kRS : 0u; i < rc; ++i) mbar_wait(&raw_full[i % kRS], (i / kRS) & 1u);
            for (uint32_t i = g > (uint32_t)kKS ? g - kKS : 0u; i < g; ++i) mbar_wait(&b_full[i % kKS], (i / kKS) & 1u);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        uint32_t g = 0, use0 = 0, use1 = 0, nxt = 0;  // acquisitions of each accumulator half
        bool stop = false, issued = false;
        for (int ti = blockIdx.x; ti < ntiles && !stop; ti += gridDim.x) {
            const Tile tl = a.tiles[ti];
            const int BN = (tl.n + 15) & ~15;
            const uint32_t idesc = instr_desc_bf16(BN);
            const bool wide = BN > 64;
            const uint32_t h = nxt;
            if (aborted(abort)) break;
            if (wide || h == 0) {
                if (!wait_or_abort(&acc_empty[0], (use0 & 1u) ^ 1u, abort)) break;
                ++use0;
            }
            if (wide || h == 1) {
                if (!wait_or_abort(&acc_empty[1], (use1 & 1u) ^ 1u, abort)) break;
                ++use1;
            }
            const uint32_t col = wide ? 0u : 64u * h;
            if (!wide) nxt ^= 1u;
            tc_fence_after();
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = g % kKS;
                // full[s]: the dequantised stage and (waited for by the dequant warps) its tokens
                if (!wait_or_abort(&full[s], (g / kKS) & 1u, abort)) {
                    stop = true;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t at = tmem + kTmemA + (uint32_t)s * kTmemAStage;
                    const uint64_t bd = desc_sw128(smem_addr(smem + SL::b + (size_t)s * kTile));
                    const uint32_t d0 = tmem + col, acc0 = kb > 0 ? 1u : 0u;
                    // one accumulator at a time: consecutive MMAs into the same TMEM columns; a
                    // K = 16 step moves the B start address 32 bytes (2 units of the descriptor)
#pragma unroll
                    for (int mm = 0; mm < 2; ++mm)
#pragma unroll
                        for (int j = 0; j < kBK / 16; ++j)
                            mma_bf16_ts(d0 + 128u * mm, at + 32u * mm + 8u * j, bd + 2u * j, idesc, j > 0 ? 1u : acc0);
                    mma_commit(&empty[s]);
                }
                issued = true;
                __syncwarp();
                ++g;
            }
            if (stop) break;
            if (lane == 0) {
                if (wide || h == 0) mma_commit(&acc_full[0]);
                if (wide || h == 1) mma_commit(&acc_full[1]);
            }
            __syncwarp();
        }
        if (aborted(abort) && issued) {
            // every MMA this thread issued must finish before the accumulators are freed
            if (lane == 0) mma_commit(drain);
            __syncwarp();
            mbar_wait(drain, 0);
        }
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;                 // TMEM lanes 32*quarter .. +31
        uint32_t f0 = 0, f1 = 0, nxt = 0;          // the MMA issuer's half assignment, replayed
        for (int ti = blockIdx.x; ti < ntiles; ti += gridDim.x) {
            const Tile tl = a.tiles[ti];
            const bool wide = ((tl.n + 15) & ~15) > 64;
            const uint32_t h = nxt;
            if (aborted(abort)) break;            // no stores of accumulators that may be incomplete
            if (wide || h == 0) {
                if (!wait_or_abort(&acc_full[0], f0 & 1u, abort)) break;
                ++f0;
            }
            if (wide || h == 1) {
                if (!wait_or_abort(&acc_full[1], f1 & 1u, abort)) break;
                ++f1;
            }
            const uint32_t col = wide ? 0u : 64u * h;
            if (!wide) nxt ^= 1u;
            tc_fence_after();
            const int row = tl.row0 + quarter * 32 + lane;
            const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
            // gate/up: act column of I-row `row` in the permuted K order of the down GEMM
            const int acol = (row & ~15) + kperm_pos(row & 15);
            for (int c0 = 0; c0 < tl.n; c0 += 16) {
                float gv[16], uv[16];
                tmem_ld16(taddr + col + c0, gv);
                tmem_ld16(taddr + 128 + col + c0, uv);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int tok = c0 + j;
                    if (tok >= tl.n) continue;
                    uint16_t *orow = a.out + (size_t)(tl.pos0 + tok) * a.R;
                    if (kGateUp) {
                        if (row < a.R) {
                            const float g1 = bf16r(gv[j]), u1 = bf16r(uv[j]);
                            const float sig = bf16r(1.0f / (1.0f + expf(-g1)));
                            orow[acol] = f32_to_bf16_bits(bf16r(bf16r(g1 * sig) * u1));
                        }
                    } else {
                        if (row < a.R) orow[row] = f32_to_bf16_bits(gv[j]);
                        if (row + kBM < a.R) orow[row + kBM] = f32_to_bf16_bits(uv[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (wide || h == 0) mbar_arrive(&acc_empty[0]);
                if (wide || h == 1) mbar_arrive(&acc_empty[1]);
            }
        }
    } else if (warp >= kDqWarp0) {
        // ------------------------------------------------------------ dequantisation
        // warp -> TMEM lane quarter (rows 32q .. 32q+31 of a matrix); the two groups of four
        // warps take the tile's two matrices (gate / up, or the two 128-row blocks of down)
        const int quarter = warp & 3;
        const int m = (warp - kDqWarp0) >> 2;
        const int r = quarter * 32 + lane;              // row within the matrix = TMEM lane
        const int roff = kGateUp ? r : r + kBM * m;     // row within the tile's weight rows
        const uint16_t *sp = (kGateUp && m) ? a.s1 : a.s0;
        const uint16_t *bp = (kGateUp && m) ? a.b1 : a.b0;
        const int ngk = a.Kdim / 64;
        const int nst = (nkb + kRawK - 1) / kRawK;
        const uint32_t tcol = tmem + ((uint32_t)(quarter * 32) << 16) + kTmemA + 32u * m;
        // scale / bias of the 8 K-blocks of a raw stage, loaded one stage ahead
        uint16_t cs[kRawK], cb[kRawK], ns[kRawK], nb[kRawK];
        auto load_sb = [&](const Tile &t, int st) {
            const bool rok = t.row0 + roff < a.R;
            const size_t base = ((size_t)t.e * a.R + (rok ? t.row0 + roff : 0)) * ngk + (size_t)st * kRawK;
#pragma unroll
            for (int i = 0; i < kRawK; ++i) {
                const bool ok = st * kRawK + i < nkb;
                ns[i] = ok ? sp[base + i] : (uint16_t)0;
                nb[i] = ok ? bp[base + i] : (uint16_t)0;
            }
        };
        uint32_t g = 0, rc = 0;
        if ((int)blockIdx.x < ntiles) load_sb(a.tiles[blockIdx.x], 0);
        bool stop = false;
        for (int ti = blockIdx.x; ti < ntiles && !stop; ti += gridDim.x) {
            const Tile tl = a.tiles[ti];
            const bool rok = tl.row0 + roff < a.R;
            for (int st = 0; st < nst && !stop; ++st) {
#pragma unroll
                for (int i = 0; i < kRawK; ++i) {
                    cs[i] = ns[i];
                    cb[i] = nb[i];
                }
                if (st + 1 < nst) load_sb(tl, st + 1);
                else if (ti + (int)gridDim.x < ntiles) load_sb(a.tiles[ti + gridDim.x], 0);
                const int rs = rc % kRS;
                if (aborted(abort) || !wait_or_abort(&raw_full[rs], (rc / kRS) & 1u, abort)) {
                    stop = true;
                    break;
                }
                const unsigned char *rbase = smem + SL::raw + (size_t)(rs * kNM + m) * kTile;
#pragma unroll
                for (int i = 0; i < kRawK; ++i) {
                    if (st * kRawK + i < nkb) {
                        const int s = g % kKS;
                        if (!wait_or_abort(&empty[s], ((g / kKS) & 1u) ^ 1u, abort)) {
                            stop = true;
                            break;
                        }
                        tc_fence_after();
                        uint4 q = *reinterpret_cast<const uint4 *>(rbase + sw128(r, i));
                        if (!rok) q = make_uint4(0u, 0u, 0u, 0u);
                        uint32_t tlo, thi;
                        dq_tables<kFp16>(cs[i], cb[i], tlo, thi);
                        uint32_t out[32];
                        dq_word(q.x, tlo, thi, out);
                        dq_word(q.y, tlo, thi, out + 8);
                        dq_word(q.z, tlo, thi, out + 16);
                        dq_word(q.w, tlo, thi, out + 24);
                        tmem_st32(tcol + (uint32_t)s * kTmemAStage, out);
                        tmem_st_wait();
                        // the MMA thread waits only for full[s]: it also stands for the stage's
                        // token rows, which every dequant warp waits for before arriving
                        if (!wait_or_abort(&b_full[s], (g / kKS) & 1u, abort)) {
                            stop = true;
                            break;
                        }
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&full[s]);
                        ++g;
                    }
                }
                __syncwarp();
                if (stop) break;
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
                ++rc;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// y[t][h] = bf16(resid + sum_k bf16(yk * s_k)) with the k sum sequential in bf16 (MLX order),
// 8 columns (16 bytes) of one token per work item
__global__ void combine_kernel(const uint16_t *yk, const int *pos_of, const uint16_t *scores, const uint16_t *resid,
                               int T, int K, int H, uint16_t *y) {
    const int cpr = H / 8;
    const size_t n = (size_t)T * cpr;
    const int TK = T * K;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / cpr), c = (int)(i % cpr);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < K; ++k) {
            const int p = pos_of ? pos_of[t * K + k] : t * K + k;   // null: rows in assignment order
            if (p < 0 || p >= TK) {            // an expert id >= E was never scattered
                atomicOr(&g_moe_device_error, MOE_DEVERR_BAD_INPUT);
                continue;
            }
            const float sc = bf16_bits_to_f32(scores[t * K + k]);
            const uint4 v = *reinterpret_cast<const uint4 *>(yk + (size_t)p * H + (size_t)c * 8);
            const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float pk = bf16r(bf16_bits_to_f32((uint16_t)(vw[j >> 1] >> (16 * (j & 1)))) * sc);
                acc[j] = (k == 0) ? pk : bf16r(acc[j] + pk);
            }
        }
        uint32_t ow[4];
        const uint4 rv = resid ? *reinterpret_cast<const uint4 *>(resid + (size_t)t * H + (size_t)c * 8)
                               : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            float a0 = acc[j], a1 = acc[j + 1];
            if (resid) {
                a0 = bf16r(bf16_bits_to_f32((uint16_t)rw[j >> 1]) + a0);
                a1 = bf16r(bf16_bits_to_f32((uint16_t)(rw[j >> 1] >> 16)) + a1);
            }
            ow[j >> 1] = (uint32_t)f32_to_bf16_bits(a0) | ((uint32_t)f32_to_bf16_bits(a1) << 16);
        }
        *reinterpret_cast<uint4 *>(y + (size_t)t * H + (size_t)c * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
}

// yk_out[i] = yk[pos_of[i]] for every assignment i = t*K + k that was bucketed (16-byte copies)
__global__ void unsort_kernel(const uint16_t *yk, const int *pos_of, int TK, int H, uint16_t *yk_out) {
    const int cpr = H / 8;
    const size_t n = (size_t)TK * cpr;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t a = i / cpr;
        const int c = (int)(i % cpr);
        const int p = pos_of[a];
        if (p < 0) continue;
        *reinterpret_cast<uint4 *>(yk_out + a * H + (size_t)c * 8) =
            *reinterpret_cast<const uint4 *>(yk + (size_t)p * H + (size_t)c * 8);
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
    w.tiles2 = reinterpret_cast<Tile *>(take(maxt * ((H + 2 * kBM - 1) / (2 * kBM)) * sizeof(Tile)));
    w.act = reinterpret_cast<uint16_t *>(take(TK * I * 2));
    w.yk = reinterpret_cast<uint16_t *>(take(TK * H * 2));
    w.bytes = off;
    return w;
}

// 2-D tensor map over a row-major [rows][cols] array with a box of box_cols x box_rows
// elements and 128-byte swizzling (box_cols * element size = 128 bytes)
int make_map(CUtensorMap *m, CUtensorMapDataType dt, size_t esize, const void *base, uint64_t cols, uint64_t rows,
             uint32_t box_cols, uint32_t box_rows) {
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * esize};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    // the driver entry point is looked up through the runtime, so the library does not link
    // libcuda directly (it loads on hosts without a driver; calls then fail with an error)
    using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        MOE_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn)
            return moe_set_error(MOE_ECUDA, "prefill: cuTensorMapEncodeTiled not available from the driver");
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    const CUresult r = encode(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return moe_set_error(MOE_ECUDA, "prefill: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return MOE_OK;
}

template <bool kGateUp, bool kFp16>
int launch_gemm(const CUtensorMap &m0, const CUtensorMap &m1, const CUtensorMap &mb, const GemmArgs &g, int grid,
                cudaStream_t st) {
    auto kern = gemm_kernel<kGateUp, kFp16>;
    const size_t smem = GemmSmem<kGateUp>::alloc;
    MOE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, kGemmThreads, smem, st>>>(m0, m1, mb, g);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
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

// The grouped expert GEMMs of T rows; experts [e_begin, e_begin + E) of the routing are
// this call's (weights indexed from e_begin); strict = 0 skips the other assignments.
// Output: y = combine (+ resid) when y is given, and/or the unweighted expert output of every
// bucketed assignment i = t*K + k in yk_out [T*K][H].
int moe_prefill_experts_ex(const void *x, int T, int H, int I, int E, int K, const uint32_t *inds, uint32_t e_begin,
                           int strict, const void *scores, const uint32_t *wg, const void *sg, const void *bg,
                           const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd, const void *sd,
                           const void *bd, int sb_fp16, const void *resid, void *y, void *yk_out, void *act_out,
                           void *workspace, size_t workspace_bytes, void *stream) {
    if (!x || !inds || !wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !workspace || (!y && !yk_out) ||
        (y && !scores))
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
    MOE_CUDA_TRY(cudaMemsetAsync(w.src_of, 0xff, (size_t)TK * 4, st));
    count_kernel<<<(TK + 255) / 256, 256, 0, st>>>(inds, TK, E, e_begin, strict, w.counts);
    scan_kernel<<<1, 1024, 0, st>>>(w.counts, E, I, H, w.offsets, w.cursor, w.tiles1, w.ntiles, w.tiles2, w.ntiles + 1);
    scatter_kernel<<<(TK + 255) / 256, 256, 0, st>>>(inds, TK, E, e_begin, w.offsets, w.cursor, w.pos_of, w.src_of);
    MOE_CUDA_TRY(cudaGetLastError());

    uint16_t *act = act_out ? static_cast<uint16_t *>(act_out) : w.act;
    // tensor maps: codes [E*R rows][Kdim/16 words] (box 32 words x 128 rows = 8 K-blocks), the
    // expert-ordered x rows [T*K][H] and act [T*K][I] (16-row boxes)
    CUtensorMap mg, mu, mx, md, ma;
    int rc = make_map(&mg, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wg, (uint64_t)H / 16, (uint64_t)E * I, 32, kBM);
    if (!rc) rc = make_map(&mu, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wu, (uint64_t)H / 16, (uint64_t)E * I, 32, kBM);
    // the gate/up B rows in expert order live in the yk buffer until the down GEMM overwrites it
    uint16_t *xs = w.yk;
    if (!rc) rc = make_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xs, (uint64_t)H, (uint64_t)TK, 64, 16);
    if (!rc) rc = make_map(&md, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wd, (uint64_t)I / 16, (uint64_t)E * H, 32, kBM);
    if (!rc) rc = make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, act, (uint64_t)I, (uint64_t)TK, 64, 16);
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(act) % 16) return moe_set_error(MOE_EINVAL, "prefill_experts: act_out not aligned");
    GemmArgs g1{w.tiles1, w.ntiles, H, I, K, static_cast<const uint16_t *>(sg), static_cast<const uint16_t *>(bg),
                static_cast<const uint16_t *>(su), static_cast<const uint16_t *>(bu), act};
    GemmArgs g2{w.tiles2, w.ntiles + 1, I, H, K, static_cast<const uint16_t *>(sd), static_cast<const uint16_t *>(bd),
                nullptr, nullptr, w.yk};
    gather_rows_kernel<<<sms * 4, 256, 0, st>>>(static_cast<const uint16_t *>(x), w.src_of, TK, K, H, xs);
    MOE_CUDA_TRY(cudaGetLastError());
    rc = sb_fp16 ? launch_gemm<true, true>(mg, mu, mx, g1, sms, st) : launch_gemm<true, false>(mg, mu, mx, g1, sms, st);
    if (!rc) rc = sb_fp16 ? launch_gemm<false, true>(md, md, ma, g2, sms, st) : launch_gemm<false, false>(md, md, ma, g2, sms, st);
    if (rc) return rc;
    if (y)
        combine_kernel<<<sms * 4, 256, 0, st>>>(w.yk, w.pos_of, static_cast<const uint16_t *>(scores),
                                                 static_cast<const uint16_t *>(resid), T, K, H, static_cast<uint16_t *>(y));
    if (yk_out)
        unsort_kernel<<<sms * 4, 256, 0, st>>>(w.yk, w.pos_of, TK, H, static_cast<uint16_t *>(yk_out));
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" int moe_prefill_experts(const void *x, int T, int H, int I, int E, int K, const uint32_t *inds,
                                   const void *scores, const uint32_t *wg, const void *sg, const void *bg,
                                   const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                                   const void *sd, const void *bd, int sb_fp16, const void *resid, void *y,
                                   void *act_out, void *workspace, size_t workspace_bytes, void *stream) {
    if (!y || !scores) return moe_set_error(MOE_EINVAL, "prefill_experts: null pointer");
    return moe_prefill_experts_ex(x, T, H, I, E, K, inds, 0u, 1, scores, wg, sg, bg, wu, su, bu, wd, sd, bd, sb_fp16,
                                  resid, y, nullptr, act_out, workspace, workspace_bytes, stream);
}

int moe_pow2_rows_launch(const void *x, int T, int H, void *xn, void *stream) {
    pow2_rows_kernel<<<T, 256, 0, as_stream(stream)>>>(static_cast<const uint16_t *>(x), H, static_cast<uint16_t *>(xn));
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

extern "C" int moe_prefill_experts_slots(const void *x, int T, int H, int I, int cap, int K, const uint32_t *slots,
                                         const uint32_t *wg, const void *sg, const void *bg, const uint32_t *wu,
                                         const void *su, const void *bu, const uint32_t *wd, const void *sd,
                                         const void *bd, int sb_fp16, void *yk_out, void *workspace,
                                         size_t workspace_bytes, void *stream) {
    if (!yk_out) return moe_set_error(MOE_EINVAL, "prefill_experts_slots: null output");
    return moe_prefill_experts_ex(x, T, H, I, cap, K, slots, 0u, 0, nullptr, wg, sg, bg, wu, su, bu, wd, sd, bd,
                                  sb_fp16, nullptr, nullptr, yk_out, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int moe_combine_rows(const void *yk, int T, int K, int H, const void *scores, const void *resid, void *y,
                                void *stream) {
    if (!yk || !scores || !y) return moe_set_error(MOE_EINVAL, "combine_rows: null pointer");
    if (T <= 0 || K <= 0 || H <= 0 || H % 8)
        return moe_set_error(MOE_EINVAL, "combine_rows: bad sizes T=%d K=%d H=%d", T, K, H);
    const void *al[] = {yk, resid, y};
    for (const void *p : al)
        if (reinterpret_cast<uintptr_t>(p) % 16) return moe_set_error(MOE_EINVAL, "combine_rows: 16-byte alignment");
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    combine_kernel<<<sms * 4, 256, 0, as_stream(stream)>>>(static_cast<const uint16_t *>(yk), nullptr,
                                                           static_cast<const uint16_t *>(scores),
                                                           static_cast<const uint16_t *>(resid), T, K, H,
                                                           static_cast<uint16_t *>(y));
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}

extern "C" int moe_pow2_rows(const void *x, int T, int H, void *xn, void *stream) {
    if (!x || !xn || T <= 0 || H <= 0) return moe_set_error(MOE_EINVAL, "pow2_rows: bad arguments");
    return moe_pow2_rows_launch(x, T, H, xn, stream);
}
