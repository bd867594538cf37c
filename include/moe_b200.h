/*
 * moe_b200.h -- C ABI of libmoe_b200.so, the B200 (sm_100a) implementation of the
 * routed-expert MoE block of Jakevin/moe-offload.
 *
 * Conventions
 *   - Every device buffer is a raw device pointer owned by the caller (PyTorch tensors on
 *     the Python side); the library never frees caller memory.
 *   - bf16 / fp16 tensors are passed as `void *` and are 16-bit IEEE bit patterns;
 *     `sb_fp16` selects fp16 (1) or bf16 (0) for affine scales and biases.
 *   - `stream` is a cudaStream_t passed as `void *` (NULL = legacy default stream).
 *   - Functions returning int return MOE_OK (0) or a negative status; moe_last_error()
 *     gives a message for the calling thread's last failure.
 *   - Expert weights use MLX's affine layout with transpose=True, exactly as the reference
 *     keeps them in its slot buffers (mlx-qwen38/loader.py:332-368):
 *       gate/up  codes u32 [cap, I, H*bits/32], scales/biases [cap, I, H/group_size]
 *       down     codes u32 [cap, H, I*bits/32], scales/biases [cap, H, I/group_size]
 *     `slots` index the leading `cap` axis (expert ids when all experts are resident).
 *
 * Citations name files of the reference project (paths inside Jakevin/moe-offload).
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_OK 0
#define MOE_EIO (-5)
#define MOE_ENOMEM (-12)
#define MOE_ENODEV (-19)
#define MOE_EINVAL (-22)
#define MOE_ETIMEDOUT (-110)
#define MOE_ECUDA (-1000)

/* Library version (major*10000 + minor*100 + patch) and the calling thread's last error. */
int moe_version(void);
const char *moe_last_error(void);

/* ------------------------------------------------------------------------------------ */
/* Router: gate matmul + precise softmax + top-k + renormalisation, optionally fused with   */
/* the next layer's top-M prediction.                                                     */
/* ------------------------------------------------------------------------------------ */

/*
 * Bytes of workspace moe_router_topk needs for T tokens, E experts and an optional
 * prediction of M experts (M = 0: none). The workspace must be zero-filled once before its
 * first use; every call leaves it zero-filled again.
 */
size_t moe_router_workspace_bytes(int T, int E, int M);

/*
 * Replaces, per token row of x:
 *   gates = gate(x); gates = softmax(gates, precise=True); inds = argpartition(gates, -K)[-K:];
 *   scores = take(gates, inds); scores /= scores.sum()          -- mlx-qwen38/loader.py:903-908,
 *                                                                  cpp/src/layers.cpp:311-325
 * and, when wn != NULL, topk_sorted_indices(gate_next(x) + pred_bias, M)
 *                                                               -- loader.py:237-242,950-956,
 *                                                                  cpp/src/layers.cpp:327-341
 *   x        bf16 [T, H]
 *   w        router weight: bf16 [E, H] when rbits == 16, else affine u32 [E, H*rbits/32]
 *            with w_scales/w_biases [E, H/group_size]
 *   wn       next layer's router (same format) or NULL; pred_bias fp32 [E] or NULL
 *   out_logits bf16 [T, E] or NULL; out_probs bf16 [T, E] or NULL
 *   out_inds  u32 [T, K] (MLX argpartition order), out_scores bf16 [T, K]
 *   out_pred  u32 [T, M] sorted by value descending, or NULL
 * Arithmetic: dot products in double, rounded once to bf16; softmax in double, rounded
 * once to bf16; ties in the top-k resolved toward the higher expert index.
 */
int moe_router_topk(const void *x, int T, int H, int E, int K,
                    const void *w, const void *w_scales, const void *w_biases,
                    int rbits, int group_size, int sb_fp16,
                    const void *wn, const void *wn_scales, const void *wn_biases,
                    int M, const float *pred_bias,
                    void *out_logits, void *out_probs, uint32_t *out_inds, void *out_scores,
                    uint32_t *out_pred, void *workspace, size_t workspace_bytes, void *stream);

/*
 * moe_router_topk without a workspace, for callers that cannot allocate device memory: a C
 * or FFI host that only receives device pointers from elsewhere and has no allocator of
 * its own, or a process whose device memory is fully reserved by another allocator.
 * This entry point has no counterpart in the reference (its C library never touches the
 * GPU). Same arguments, arithmetic and results as moe_router_topk, minus the workspace.
 * Scratch lives in a fixed array of 257 KiB that every device which loads the library holds
 * until the process exits; limits: T <= 256 and T * E <= 65536, larger sizes return
 * MOE_EINVAL. The first call on a device looks up that device's copy of the array (make it
 * with the device current, before any stream capture). Every call shares the array and it
 * keeps the last call's contents (the per-token tickets are cleared at the start of each
 * call); calls that overlap on the GPU race. Allocates nothing (no cudaMalloc/cudaFree).
 */
int moe_router_topk_noalloc(const void *x, int T, int H, int E, int K,
                            const void *w, const void *w_scales, const void *w_biases,
                            int rbits, int group_size, int sb_fp16,
                            const void *wn, const void *wn_scales, const void *wn_biases,
                            int M, const float *pred_bias,
                            void *out_logits, void *out_probs, uint32_t *out_inds,
                            void *out_scores, uint32_t *out_pred, void *stream);

/* ------------------------------------------------------------------------------------ */
/* Routed experts, decode (one row of x per token).                                       */
/* ------------------------------------------------------------------------------------ */

/*
 * act[t,k,:] = SwiGLU(gate_qmm(x[t], W_gate[slots[t,k]]), up_qmm(x[t], W_up[slots[t,k]]))
 * Replaces the up/gate gather_qmm + swiglu of mlx_vlm SwitchGLU
 * (cpp/src/layers.cpp:343-358, cpp/src/kernels.cpp:1027-1040,1090-1094).
 *   x bf16 [T, H], slots u32 [T, K] (each < cap, the slot-buffer depth), act bf16 [T, K, I].
 *   bits == 2, group_size == 64. A slot >= cap is not read; its activations are zero.
 */
int moe_experts_gateup(const void *x, int T, int H, int I, int K, int cap, const uint32_t *slots,
                       const uint32_t *wg, const void *sg, const void *bg,
                       const uint32_t *wu, const void *su, const void *bu,
                       int bits, int group_size, int sb_fp16, void *act, void *stream);

/*
 * yk[t,k,:] = down_qmm(act[t,k], W_down[slots[t,k]])               (layers.cpp:359-361)
 * y[t,:]    = sum_k yk[t,k,:] * scores[t,k] (+ addend[t]) (+ resid[t])
 *                                          (loader.py:914,965; cpp/src/layers.cpp:400,599)
 *   act bf16 [T, K, I]; scores bf16 [T, K] or NULL (then y is not written);
 *   addend / resid bf16 [T, H] or NULL; y bf16 [T, H] or NULL; yk bf16 [T, K, H] or NULL.
 */
int moe_experts_down(const void *act, int T, int H, int I, int K, int cap, const uint32_t *slots,
                     const void *scores, const uint32_t *wd, const void *sd, const void *bd,
                     int bits, int group_size, int sb_fp16, const void *addend, const void *resid,
                     void *y, void *yk, void *stream);

/* ------------------------------------------------------------------------------------ */
/* Fused decode step of one all-resident layer.                                           */
/* ------------------------------------------------------------------------------------ */

/* Workspace bytes for moe_decode_layer; zero-fill it once before first use. */
size_t moe_decode_workspace_bytes(int T, int H, int I, int E, int K, int M);

/*
 * y = combine(experts(x, router(x))) for a layer whose E experts are all resident (slot id ==
 * expert id): the decode body of the reference's hook for a resident layer
 * (mlx-qwen38/loader.py:903-922 router + switch_mlp + combine; cpp/src/engine.cpp:532-571).
 * Three kernels chained with programmatic dependent launch; the router is bf16 [E, H];
 * router_next_w / M / pred_bias as in moe_router_topk. Expert weights as in
 * moe_experts_gateup / moe_experts_down with cap = E. resid/addend optional (bf16 [T, H]).
 * norm = 1: the MoE input is x * 2^-k, the power of two nearest x's RMS (k = floor(e/2) for
 * mean(x^2) in [2^(e-1), 2^e)), standing in for the model's pre-MoE RMSNorm while keeping the
 * rescale exact; the residual stays x. norm = 0: the input is x as given.
 */
int moe_decode_layer(const void *x, int T, int H, int I, int E, int K, const void *router_w,
                     const void *router_next_w, int M, const float *pred_bias,
                     const uint32_t *wg, const void *sg, const void *bg,
                     const uint32_t *wu, const void *su, const void *bu,
                     const uint32_t *wd, const void *sd, const void *bd, int sb_fp16, int norm,
                     const void *addend, const void *resid, uint32_t *out_inds, void *out_scores,
                     uint32_t *out_pred, void *y, void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------------ */
/* Persistent decode of a whole resident stack (one token through L layers, one launch).  */
/* ------------------------------------------------------------------------------------ */

/* Packed expert layout used by moe_stack_decode: one contiguous block per expert holding,
 * for each 64-wide group G of the expert's intermediate dimension, the 64 gate and 64 up
 * rows of G and the down matrix's 64 columns of G for all H rows, ordered as the decode
 * kernel reads them (codes and 16-bit scales / biases, same byte count as the MLX layout).
 * No reference counterpart: the reference reads each expert's nine MLX tensors
 * (mlx-qwen38/expert_io.c:34-71 pread per tensor). Bytes per expert (H % 256 == 0 and
 * I % 64 == 0, else 0). */
size_t moe_packed_expert_bytes(int H, int I);

/* Packs E experts from the MLX layout of moe_experts_gateup / moe_experts_down (cap = E)
 * into out[E][moe_packed_expert_bytes(H, I)] on the stream. Code arrays and out 16-byte
 * aligned. */
int moe_pack_experts(int E, int H, int I, const uint32_t *wg, const void *sg, const void *bg,
                     const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                     const void *sd, const void *bd, void *out, void *stream);

/* Per-layer weights of moe_stack_decode, passed as a DEVICE array of L descriptors: the
 * transposed router ([H][E] bf16, row h = the E router weights of input h) and the layer's
 * E packed experts. Both 16-byte aligned. */
typedef struct {
    const void *router_t;
    const void *experts;
} moe_stack_layer;

/* Workspace bytes for moe_stack_decode (no zero-filling needed: each call clears it). */
size_t moe_stack_workspace_bytes(int H, int I, int E, int K);

/*
 * h_{l+1} = h_l + MoE_l(h_l) for l = 0..L-1 on one token (batch 1), all experts resident:
 * the reference's decode loop over resident layers (mlx-qwen38/loader.py:1176-1195 around
 * the per-layer block of loader.py:903-922), as ONE cooperative kernel with one CTA per SM
 * (num_ctas = 0: all SMs) and two grid barriers per layer. x, y bf16 [H]; inds_out u32
 * [L][K] and scores_out bf16 [L][K] (MLX order, as moe_router_topk); hs_out bf16 [L+1][H]
 * (every layer's input and the final output) or NULL. Requires H % 256 == 0, H <= 4096,
 * I % 64 == 0, K <= 32, E <= 2048 and at least H/32 CTAs. Router logits are sums of per-CTA exact partial dot products in double
 * (order of the partial sums varies between runs at the 2^-52 level). norm as in
 * moe_decode_layer (applied to every layer's input).
 */
int moe_stack_decode(const void *layers, int L, int H, int I, int E, int K, int sb_fp16, int norm,
                     const void *x, void *y, uint32_t *inds_out, void *scores_out, void *hs_out,
                     void *workspace, size_t workspace_bytes, int num_ctas, void *stream);

/*
 * Device-side error word (bit 1: a bounded mbarrier/flag wait gave up, bit 2: invalid
 * input seen by a kernel). Returns the current value (>= 0) and clears it when `clear`.
 * Kernels never trap: they record the condition here and skip the affected work.
 */
int moe_device_error(int clear);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
