// One decode step of one MoE layer with every expert resident in HBM: router (+ optional
// next-layer prediction) -> gate/up + SwiGLU -> down + combine, three PDL-chained kernels
// that hand each other the int8 MMA records of their input vectors (gemv_i8.cuh) through
// the workspace, so no kernel re-stages an input. This is the per-layer body of the reference's decode hook
// for a resident layer (mlx-qwen38/loader.py:903-922; cpp/src/engine.cpp:532-571).
#include "common.cuh"
#include "internal.h"

namespace {

struct DecodeWs {
    unsigned int *tickets;
    uint16_t *logits, *plogits;
    uint2 *xrec;
    float *xscale, *xsum;
    uint16_t *act;
    uint2 *arec;
    float *ascale, *asum;
    unsigned int *acnt;
    size_t bytes;
};

DecodeWs carve(void *base, int T, int H, int I, int E, int K, int M) {
    DecodeWs w{};
    const int ngH = H / 64, ngI = I / 64;
    char *p = static_cast<char *>(base);
    size_t off = 0;
    auto take = [&](size_t n) { char *q = p ? p + off : nullptr; off += al256(n); return q; };
    w.tickets = reinterpret_cast<unsigned int *>(take((size_t)T * 4));
    w.logits = reinterpret_cast<uint16_t *>(take((size_t)T * E * 2));
    w.plogits = reinterpret_cast<uint16_t *>(take(M > 0 ? (size_t)T * E * 2 : 0));
    w.xrec = reinterpret_cast<uint2 *>(take((size_t)T * ngH * 128));
    w.xscale = reinterpret_cast<float *>(take((size_t)T * pad4(ngH) * 4));
    w.xsum = reinterpret_cast<float *>(take((size_t)T * pad4(ngH) * 4));
    w.act = reinterpret_cast<uint16_t *>(take((size_t)T * K * I * 2));
    w.arec = reinterpret_cast<uint2 *>(take((size_t)T * K * ngI * 128));
    w.ascale = reinterpret_cast<float *>(take((size_t)T * pad4(K * ngI) * 4));
    w.asum = reinterpret_cast<float *>(take((size_t)T * pad4(K * ngI) * 4));
    w.acnt = reinterpret_cast<unsigned int *>(take((size_t)T * K * ngI * 4));
    w.bytes = off;
    if (M <= 0) w.plogits = nullptr;
    return w;
}

}  // namespace

extern "C" size_t moe_decode_workspace_bytes(int T, int H, int I, int E, int K, int M) {
    if (T <= 0 || H <= 0 || I <= 0 || E <= 0 || K <= 0) return 0;
    return carve(nullptr, T, H, I, E, K, M).bytes;
}

extern "C" int moe_decode_layer(const void *x, int T, int H, int I, int E, int K, const void *router_w,
                                const void *router_next_w, int M, const float *pred_bias,
                                const uint32_t *wg, const void *sg, const void *bg, const uint32_t *wu,
                                const void *su, const void *bu, const uint32_t *wd, const void *sd,
                                const void *bd, int sb_fp16, int norm, const void *addend, const void *resid,
                                uint32_t *out_inds, void *out_scores, uint32_t *out_pred, void *y,
                                void *workspace, size_t workspace_bytes, void *stream) {
    if (!y || !out_inds || !out_scores) return moe_set_error(MOE_EINVAL, "decode_layer: null output");
    if (H % 64 || I % 64) return moe_set_error(MOE_EINVAL, "decode_layer: H and I must be multiples of 64");
    const size_t need = moe_decode_workspace_bytes(T, H, I, E, K, M);
    if (!workspace || workspace_bytes < need)
        return moe_set_error(MOE_EINVAL, "decode_layer: workspace of %zu bytes needed, %zu given", need,
                             workspace_bytes);
    DecodeWs w = carve(workspace, T, H, I, E, K, M);
    int rc = moe_router_launch(x, T, H, E, K, router_w, nullptr, nullptr, 16, 64, 0, router_next_w, nullptr,
                               nullptr, M, pred_bias, nullptr, nullptr, out_inds, out_scores, out_pred,
                               w.tickets, w.logits, w.plogits, w.xrec, w.xscale, w.xsum, norm, stream);
    if (rc) return rc;
    rc = moe_experts_gateup_ex(x, w.xrec, w.xscale, w.xsum, T, H, I, K, E, out_inds, wg, sg, bg, wu, su, bu, 2, 64,
                               sb_fp16, w.act, w.arec, w.ascale, w.asum, w.acnt, stream);
    if (rc) return rc;
    return moe_experts_down_ex(w.act, w.arec, w.ascale, w.asum, T, H, I, K, E, out_inds, out_scores, wd, sd, bd, 2, 64,
                               sb_fp16, addend, resid, y, nullptr, stream);
}
