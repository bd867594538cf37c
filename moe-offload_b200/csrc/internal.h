// Internal (non-exported) entry points shared between translation units of libmoe_b200.
#pragma once

#include <stddef.h>
#include <stdint.h>

int moe_router_launch(const void *x, int T, int H, int E, int K, const void *w,
                      const void *w_scales, const void *w_biases, int rbits, int group_size,
                      int sb_fp16, const void *wn, const void *wn_scales, const void *wn_biases,
                      int M, const float *pred_bias, void *out_logits, void *out_probs,
                      uint32_t *out_inds, void *out_scores, uint32_t *out_pred,
                      unsigned int *tickets, uint16_t *logits_buf, uint16_t *plogits_buf,
                      void *xrec, float *xscale, float *xsum, int norm, void *stream);

// slot_base: the kernels use slots[] - slot_base as the slot id (a rank holding experts
// [slot_base, slot_base + cap) of an expert-parallel shard); ids outside the shard are skipped
// (their outputs are zero).
int moe_experts_gateup_ex(const void *x, const void *xrec, const float *xscale, const float *xsum, int T,
                          int H, int I, int K, int cap, const uint32_t *slots, const uint32_t *wg,
                          const void *sg, const void *bg, const uint32_t *wu, const void *su, const void *bu,
                          int bits, int group_size, int sb_fp16, void *act, void *arec, float *ascale,
                          float *asum, unsigned int *acnt, void *stream, uint32_t slot_base = 0);

int moe_experts_down_ex(const void *act, const void *arec, const float *ascale, const float *asum, int T, int H,
                        int I, int K, int cap, const uint32_t *slots, const void *scores, const uint32_t *wd,
                        const void *sd, const void *bd, int bits, int group_size, int sb_fp16,
                        const void *addend, const void *resid, void *y, void *yk, void *stream,
                        uint32_t slot_base = 0);

// Grouped expert GEMMs (prefill.cu): experts [e_begin, e_begin + E) of the routing, weights
// indexed from e_begin; strict = 0 skips other assignments; y (combine + resid) and / or
// yk_out [T*K][H] (unweighted expert outputs in assignment order).
int moe_prefill_experts_ex(const void *x, int T, int H, int I, int E, int K, const uint32_t *inds, uint32_t e_begin,
                           int strict, const void *scores, const uint32_t *wg, const void *sg, const void *bg,
                           const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd, const void *sd,
                           const void *bd, int sb_fp16, const void *resid, void *y, void *yk_out, void *act_out,
                           void *workspace, size_t workspace_bytes, void *stream);

// xn[t] = x[t] * 2^-k(t), the per-row power-of-two RMS normalisation (prefill.cu)
int moe_pow2_rows_launch(const void *x, int T, int H, void *xn, void *stream);
