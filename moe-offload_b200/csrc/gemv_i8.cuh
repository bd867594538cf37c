// Integer tensor-core GEMV core for 2-bit affine weights (group 64).
//
// A row's dot product with an input vector v over one 64-code group G is
//     s[G] * sum_k q_k v_k + b[G] * sum_k v_k.
// The first sum runs on m16n8k32 u8 x s8 MMAs with exact int32 accumulation:
//   * A (weights): the packed codes are masked in place, no shifting to bit 0:
//       w & 0x03030303 -> codes 4j+0 (x1)   (w>>2) & 0x03030303 -> codes 4j+1 (x1)
//       w & 0x30303030 -> codes 4j+2 (x16)  (w>>2) & 0x30303030 -> codes 4j+3 (x16)
//     (byte j of a register = one code times its class multiplier); two accumulator sets
//     (x1 and x16 classes) are combined exactly as DX + (DY >> 4).
//   * B (input): v is split exactly into two int8 parts per group, v = (hi*128 + lo) * 2^E,
//     E = floor(log2 max|v_G|) - 13, hi = floor(u / 128), lo = u - 128*hi, u = rint(v/2^E),
//     which is exact for every element within 2^6 of the group maximum and off by at most
//     2^(E-1) below that (a relative error < 2^-14 of the group maximum).
//   * The N dimension carries four groups: lane quad t of every row supplies group 4j+t on
//     its k-slots, B column 2t holds that group's hi part and column 2t+1 its lo part on
//     lane t's k-slots only, so the D fragment of lane (g, t) is exactly
//     (hi, lo) of group 4j+t for rows g and g+8: dot = (D[2t]*128 + D[2t+1]) * 2^E.
//
// "Records": the B operand of one group is a 128-byte record of 16 uint2 entries,
//   entry e = (c*4 + i)*2 + h  (class c in {0: codes 4j+0/4j+1, 1: codes 4j+2/4j+3},
//   word i of the group, part h in {hi, lo}); entry.x byte j = part_h(v[16i + 4j + 2c]),
//   entry.y byte j = part_h(v[16i + 4j + 2c + 1]); plus scale = 2^E and sum = sum(v) (fp32).
#pragma once

#include "common.cuh"

MOE_D void mma_u8s8_16832(int d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Does lane L hold a non-zero B fragment (column n = L>>2 belongs to lane quad t = n>>1)?
MOE_D bool rec_lane_active(int lane) { return (lane & 3) == (lane >> 3); }
// entry part (hi = 0, lo = 1) of an active lane
MOE_D int rec_lane_part(int lane) { return (lane >> 2) & 1; }

// One MMA step over four groups for the row pair of this lane.
//   wa / wb: 16-byte group of row g / row g+8 (this lane's group 4j+t)
//   rec: the record of group 4j + (B-lane's quad) (16 uint2 entries) -- pass a zero record
//        for lanes that are not rec_lane_active or whose group is past the end
// Returns the per-row integer dots (scale 2^E not applied): dg for row g, db for row g+8.
MOE_D void mma_step_i8(const uint4 wa, const uint4 wb, const uint2 *rec, int part, int &dg, int &db) {
    int dx[4] = {0, 0, 0, 0}, dy[4] = {0, 0, 0, 0};
    const uint32_t aw[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t bw[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t a = aw[i], a2 = aw[i] >> 2, b = bw[i], b2 = bw[i] >> 2;
        const uint2 rx = rec[(0 * 4 + i) * 2 + part];
        const uint2 ry = rec[(1 * 4 + i) * 2 + part];
        mma_u8s8_16832(dx, a & 0x03030303u, b & 0x03030303u, a2 & 0x03030303u, b2 & 0x03030303u, rx.x, rx.y);
        mma_u8s8_16832(dy, a & 0x30303030u, b & 0x30303030u, a2 & 0x30303030u, b2 & 0x30303030u, ry.x, ry.y);
    }
    const int c0 = dx[0] + (dy[0] >> 4), c1 = dx[1] + (dy[1] >> 4);
    const int c2 = dx[2] + (dy[2] >> 4), c3 = dx[3] + (dy[3] >> 4);
    dg = c0 * 128 + c1;
    db = c2 * 128 + c3;
}

// Loads used by build_rec_group: kL2 reads global memory through L2 only (ld.global.cg), as
// needed for data another SM wrote earlier in the same kernel; otherwise plain loads
// (shared memory, or global data produced by an earlier kernel).
template <bool kL2>
MOE_D uint2 rec_ld2(const uint16_t *p) {
    if constexpr (kL2) return __ldcg(reinterpret_cast<const uint2 *>(p));
    else return *reinterpret_cast<const uint2 *>(p);
}
template <bool kL2>
MOE_D uint16_t rec_ld1(const uint16_t *p) {
    if constexpr (kL2) return __ldcg(p);
    else return *p;
}

// Builds the record of one 64-value group with 16 cooperating lanes (an aligned half warp,
// ent = lane & 15). `v` points at the group's 64 bf16 values (global or shared memory).
// Writes rec[ent] and, from ent 0, *scale / *sum (both times `mul`, a power of two that
// rescales the vector exactly). All 32 lanes of the warp must call it.
template <bool kL2 = false>
MOE_D void build_rec_group(const uint16_t *v, bool valid, int ent, uint2 *rec, float *scale, float *sum,
                           float mul = 1.0f) {
    // group maximum and sum: each lane reads 4 consecutive values
    float mx = 0.f, sm = 0.f;
    if (valid) {
        const uint2 q = rec_ld2<kL2>(v + 4 * ent);
        const float f0 = __uint_as_float(q.x << 16), f1 = __uint_as_float(q.x & 0xffff0000u);
        const float f2 = __uint_as_float(q.y << 16), f3 = __uint_as_float(q.y & 0xffff0000u);
        mx = fmaxf(fmaxf(fabsf(f0), fabsf(f1)), fmaxf(fabsf(f2), fabsf(f3)));
        sm = (f0 + f1) + (f2 + f3);
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        sm += __shfl_xor_sync(0xffffffffu, sm, off);
    }
    if (!valid) return;
    // E = floor(log2 mx) - 13 from the exponent bits (normal mx); u = v * 2^-E is exact
    int E = 0;
    float inv = 1.0f;
    if (mx > 0.f) {
        const int be = (int)((__float_as_uint(mx) >> 23) & 0xffu);
        if (be > 0) {
            E = be - 127 - 13;
        } else {                                      // subnormal group maximum
            int emax = 0;
            frexpf(mx, &emax);
            E = emax - 1 - 13;
        }
        const int ib = 127 - E;                       // biased exponent of 2^-E
        inv = (ib >= 1 && ib <= 254) ? __uint_as_float((uint32_t)ib << 23) : ldexpf(1.0f, -E);
    }
    const int c = ent >> 3, i = (ent >> 1) & 3, h = ent & 1;
    uint32_t bytes[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        uint32_t packed = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float f = bf16_bits_to_f32(rec_ld1<kL2>(v + 16 * i + 4 * j + 2 * c + r));
            const int u = __float2int_rn(f * inv);
            const int hi = u >> 7;                 // floor division (arithmetic shift)
            const int lo = u - hi * 128;           // 0..127
            const int part = h ? lo : hi;
            packed |= (uint32_t)(part & 0xff) << (8 * j);
        }
        bytes[r] = packed;
    }
    rec[ent] = make_uint2(bytes[0], bytes[1]);
    if (ent == 0) {
        *scale = ((E >= -126 && E <= 127) ? __uint_as_float((uint32_t)(E + 127) << 23) : ldexpf(1.0f, E)) * mul;
        *sum = sm * mul;
    }
}

// Record of one 64-value group whose values are spread over an aligned half warp: lane
// ent = lane & 15 holds values 4*ent .. 4*ent+3 as two bf16 pairs (q.x = values 0, 1;
// q.y = values 2, 3). Produces the same record, scale and sum as build_rec_group (the sum
// is taken in a different order); entry ent goes to rec[ent * stride] (stride 1: the
// record's 128 bytes back to back; larger: an entry-major table of several groups). All 32
// lanes call it, each half warp with its own group; `valid` is uniform within a half warp.
static __device__ __noinline__ void rec_from_regs(uint2 q, bool valid, uint2 *rec, float *scale, float *sum, float mul,
                                           int stride = 1) {
    const int lane = threadIdx.x & 31, ent = lane & 15, hb = lane & 16;
    const float f0 = __uint_as_float(q.x << 16), f1 = __uint_as_float(q.x & 0xffff0000u);
    const float f2 = __uint_as_float(q.y << 16), f3 = __uint_as_float(q.y & 0xffff0000u);
    float mx = fmaxf(fmaxf(fabsf(f0), fabsf(f1)), fmaxf(fabsf(f2), fabsf(f3)));
    float sm = (f0 + f1) + (f2 + f3);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        sm += __shfl_xor_sync(0xffffffffu, sm, off);
    }
    // entry (c, i, h) takes word c of lanes 4i + j (values 16i + 4j + 2c + r, r = 0, 1)
    const int c = ent >> 3, i = (ent >> 1) & 3, h = ent & 1;
    uint32_t src[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t wx = __shfl_sync(0xffffffffu, q.x, hb + 4 * i + j);
        const uint32_t wy = __shfl_sync(0xffffffffu, q.y, hb + 4 * i + j);
        src[j] = c ? wy : wx;
    }
    if (!valid) return;
    int E = 0;
    float inv = 1.0f;
    if (mx > 0.f) {
        const int be = (int)((__float_as_uint(mx) >> 23) & 0xffu);
        if (be > 0) {
            E = be - 127 - 13;
        } else {                                      // subnormal group maximum
            int emax = 0;
            frexpf(mx, &emax);
            E = emax - 1 - 13;
        }
        const int ib = 127 - E;                       // biased exponent of 2^-E
        inv = (ib >= 1 && ib <= 254) ? __uint_as_float((uint32_t)ib << 23) : ldexpf(1.0f, -E);
    }
    uint32_t bytes[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float f = __uint_as_float(r ? (src[j] & 0xffff0000u) : (src[j] << 16));
            const int u = __float2int_rn(f * inv);
            const int hi = u >> 7, lo = u - hi * 128;
            bytes[r] |= (uint32_t)((h ? lo : hi) & 0xff) << (8 * j);
        }
    }
    rec[ent * stride] = make_uint2(bytes[0], bytes[1]);
    if (ent == 0) {
        *scale = ((E >= -126 && E <= 127) ? __uint_as_float((uint32_t)(E + 127) << 23) : ldexpf(1.0f, E)) * mul;
        *sum = sm * mul;
    }
}

// mma_step_i8 with the records in an entry-major table: entry e of this lane's B group at
// rt[e * stride]. Lanes that are not rec_lane_active (act = false) load nothing.
MOE_D void mma_step_i8t(const uint4 wa, const uint4 wb, const uint2 *rt, int stride, bool act, int part, int &dg,
                        int &db) {
    int dx[4] = {0, 0, 0, 0}, dy[4] = {0, 0, 0, 0};
    const uint32_t aw[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t bw[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t a = aw[i], a2 = aw[i] >> 2, b = bw[i], b2 = bw[i] >> 2;
        const uint2 rx = act ? rt[((0 * 4 + i) * 2 + part) * stride] : make_uint2(0u, 0u);
        const uint2 ry = act ? rt[((1 * 4 + i) * 2 + part) * stride] : make_uint2(0u, 0u);
        mma_u8s8_16832(dx, a & 0x03030303u, b & 0x03030303u, a2 & 0x03030303u, b2 & 0x03030303u, rx.x, rx.y);
        mma_u8s8_16832(dy, a & 0x30303030u, b & 0x30303030u, a2 & 0x30303030u, b2 & 0x30303030u, ry.x, ry.y);
    }
    const int c0 = dx[0] + (dy[0] >> 4), c1 = dx[1] + (dy[1] >> 4);
    const int c2 = dx[2] + (dy[2] >> 4), c3 = dx[3] + (dy[3] >> 4);
    dg = c0 * 128 + c1;
    db = c2 * 128 + c3;
}
