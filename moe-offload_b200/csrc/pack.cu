// Packed expert layout for the persistent decode kernel (moe_stack_decode).
//
// The MLX layout keeps each expert's nine tensors apart (codes, scales and biases of gate,
// up and down). The decode kernel instead fetches, per CTA and layer, the slice of one
// routed expert that produces one 64-wide group G of the activation vector: the 64 gate
// rows and 64 up rows 64G..64G+63, and the down matrix's columns 64G..64G+63 for all H
// rows. The packed layout stores exactly that slice contiguously, so one expert is one
// block of bytes (one copy when it moves between host and device) and a CTA's slice is a
// handful of 1-D bulk copies. Inside the slice the order is the order in which the
// kernel's warps read it, so every shared-memory read of the MMA loop is conflict-free:
//
//   expert e          : ngI = I/64 group blocks of 60*H bytes
//   group block G     : 8 units of 5*H bytes, down codes (16*H), down scales (4*H)
//   unit u (rows 64G+8u+g, g < 8):
//       gate codes    : 16-byte chunk (g, Gj) at ((j*8 + g)*4 + t)*16, Gj = 4j + t, holding
//                       the 64 codes of row g's input group Gj (MLX words 4Gj..4Gj+3)
//       up codes      : same, at offset 2*H
//       scale records : 8 bytes (g, Gj) at 4*H + ((j*8 + g)*4 + t)*8 = {sg, bg, su, bu}
//   down codes        : row r's 64 codes of group G (MLX words 4G..4G+3) at 16*r
//   down scales       : row r's {sd, bd} of group G at 4*r
//
// The byte count equals the MLX layout's (2-bit codes and 16-bit scales, biases), so the
// roofline bytes of a token do not change.
#include "common.cuh"

namespace {

struct PackDims {
    int H, I, ngH, ngI;
    size_t ub, gbytes, ebytes;
    MOE_HD PackDims(int H_, int I_) : H(H_), I(I_), ngH(H_ / 64), ngI(I_ / 64) {
        ub = 5 * (size_t)H;
        gbytes = 60 * (size_t)H;
        ebytes = (size_t)ngI * gbytes;
    }
};

struct PackArgs {
    int E;
    PackDims d;
    const uint32_t *wg, *wu, *wd;
    const uint16_t *sg, *bg, *su, *bu, *sd, *bd;
    unsigned char *out;
};

// One thread per 16-byte gate/up code chunk, 8-byte scale record, 16-byte down code row and
// 4-byte down scale pair; grid-stride over each of the four kinds.
__global__ void pack_kernel(PackArgs a) {
    const PackDims &d = a.d;
    const size_t E = a.E, H = d.H, I = d.I, ngH = d.ngH, ngI = d.ngI;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t t0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t per_unit = 8 * ngH;   // chunks (or records) per unit and matrix
    // gate / up code chunks
    const size_t n_codes = E * ngI * 8 * 2 * per_unit;
    for (size_t x = t0; x < n_codes; x += stride) {
        size_t y = x;
        const size_t ci = y % per_unit; y /= per_unit;
        const size_t m = y % 2; y /= 2;
        const size_t u = y % 8; y /= 8;
        const size_t G = y % ngI; y /= ngI;
        const size_t e = y;
        const size_t t = ci % 4, g = (ci / 4) % 8, j = ci / 32, Gj = 4 * j + t;
        const size_t row = 64 * G + 8 * u + g;
        const uint32_t *src = (m == 0 ? a.wg : a.wu) + (e * I + row) * (H / 16) + 4 * Gj;
        unsigned char *dst = a.out + e * d.ebytes + G * d.gbytes + u * d.ub + m * 2 * H + ci * 16;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
    }
    // gate / up scale records
    const size_t n_rec = E * ngI * 8 * per_unit;
    for (size_t x = t0; x < n_rec; x += stride) {
        size_t y = x;
        const size_t ci = y % per_unit; y /= per_unit;
        const size_t u = y % 8; y /= 8;
        const size_t G = y % ngI; y /= ngI;
        const size_t e = y;
        const size_t t = ci % 4, g = (ci / 4) % 8, j = ci / 32, Gj = 4 * j + t;
        const size_t row = 64 * G + 8 * u + g, si = (e * I + row) * ngH + Gj;
        const uint2 v = make_uint2((uint32_t)a.sg[si] | ((uint32_t)a.bg[si] << 16),
                                   (uint32_t)a.su[si] | ((uint32_t)a.bu[si] << 16));
        unsigned char *dst = a.out + e * d.ebytes + G * d.gbytes + u * d.ub + 4 * H + ci * 8;
        *reinterpret_cast<uint2 *>(dst) = v;
    }
    // down code rows and scale pairs
    const size_t n_down = E * ngI * H;
    for (size_t x = t0; x < n_down; x += stride) {
        const size_t r = x % H, G = (x / H) % ngI, e = x / (H * ngI);
        const uint32_t *src = a.wd + (e * H + r) * (I / 16) + 4 * G;
        unsigned char *blk = a.out + e * d.ebytes + G * d.gbytes;
        *reinterpret_cast<uint4 *>(blk + 40 * H + r * 16) = *reinterpret_cast<const uint4 *>(src);
        const size_t si = (e * H + r) * ngI + G;
        *reinterpret_cast<uint32_t *>(blk + 56 * H + r * 4) = (uint32_t)a.sd[si] | ((uint32_t)a.bd[si] << 16);
    }
}

}  // namespace

extern "C" size_t moe_packed_expert_bytes(int H, int I) {
    if (H <= 0 || I <= 0 || H % 256 || I % 64) return 0;
    return PackDims(H, I).ebytes;
}

extern "C" int moe_pack_experts(int E, int H, int I, const uint32_t *wg, const void *sg, const void *bg,
                                const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                                const void *sd, const void *bd, void *out, void *stream) {
    if (E <= 0 || H <= 0 || I <= 0 || H % 256 || I % 64)
        return moe_set_error(MOE_EINVAL, "pack_experts: bad sizes E=%d H=%d I=%d", E, H, I);
    if (!wg || !sg || !bg || !wu || !su || !bu || !wd || !sd || !bd || !out)
        return moe_set_error(MOE_EINVAL, "pack_experts: null pointer");
    const void *ptrs16[] = {wg, wu, wd, out};
    for (const void *p : ptrs16)
        if (reinterpret_cast<uintptr_t>(p) % 16)
            return moe_set_error(MOE_EINVAL, "pack_experts: code and output pointers must be 16-byte aligned");
    PackArgs a{E, PackDims(H, I), wg, wu, wd,
               static_cast<const uint16_t *>(sg), static_cast<const uint16_t *>(bg),
               static_cast<const uint16_t *>(su), static_cast<const uint16_t *>(bu),
               static_cast<const uint16_t *>(sd), static_cast<const uint16_t *>(bd),
               static_cast<unsigned char *>(out)};
    int dev = 0, sms = 0;
    MOE_CUDA_TRY(cudaGetDevice(&dev));
    MOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    pack_kernel<<<sms * 8, 256, 0, as_stream(stream)>>>(a);
    MOE_CUDA_TRY(cudaGetLastError());
    return MOE_OK;
}
