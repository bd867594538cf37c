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
 *   wn       next layer's router in this router's format (an affine one behind a bf16 router
 *            is refused: MOE_EINVAL) or NULL; pred_bias fp32 [E] or NULL
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
 * with the device current, before any stream capture); the lookup is repeated when the
 * device's context has changed since (after a cudaDeviceReset, which reloads the module at
 * a new address), so that first call after a reset must come before any stream capture
 * too. Every call shares the array and it
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


/* ------------------------------------------------------------------------------------ */
/* Prefill: T tokens through one layer's routed experts as expert-grouped tcgen05 GEMMs.  */
/* ------------------------------------------------------------------------------------ */

/* Workspace bytes for moe_prefill_experts (bucketing, tile lists, act [T*K][I], yk [T*K][H]). */
size_t moe_prefill_workspace_bytes(int T, int H, int I, int E, int K);

/*
 * The prefill branch of the MoE block (mlx-qwen38/loader.py:566-699, cpp/src/layers.cpp:403-600;
 * gather_qmm per expert group as prefill_qproj.py:18-40): x bf16 [T][H], inds u32 [T][K] and
 * scores bf16 [T][K] from the router (moe_router_topk), experts in the MLX layout with
 * cap = E. Assignments are grouped by expert on the device; gate/up and down run as GEMMs
 * with M = 128 weight rows and N = the expert's tokens on the tensor cores (weight codes
 * and activations staged by TMA, weights dequantised to bf16 into tensor memory, fp32
 * accumulation in TMEM); y bf16 [T][H] = resid + sum_k bf16(expert_k(x) * score_k)
 * (sequential bf16 in MLX order). resid may be NULL. act_out (bf16 [T*K][I], positions in
 * expert order) may be NULL; its columns are in the GEMMs' K order: inside every 16-column
 * group, column c holds activation [0,4,8,12,1,5,9,13,2,6,10,14,3,7,11,15][c]. H, I
 * multiples of 64; x and code arrays 16-byte aligned.
 */
int moe_prefill_experts(const void *x, int T, int H, int I, int E, int K, const uint32_t *inds,
                        const void *scores, const uint32_t *wg, const void *sg, const void *bg,
                        const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                        const void *sd, const void *bd, int sb_fp16, const void *resid, void *y,
                        void *act_out, void *workspace, size_t workspace_bytes, void *stream);

/* Workspace bytes for moe_prefill_layer; zero-fill it once before first use (the router's
 * tickets inside it are left at zero by every call). */
size_t moe_prefill_layer_workspace_bytes(int T, int H, int I, int E, int K);

/*
 * One resident layer's prefill: router over the T rows (bf16 [E, H] router, exact softmax /
 * MLX-order top-k as moe_router_topk) then moe_prefill_experts, i.e. the prefill branch of
 * the reference's hook for a layer whose experts are all resident (mlx-qwen38/loader.py:
 * 903-908 router + 566-699 experts; cpp/src/layers.cpp:403-600). norm = 1 feeds router and
 * experts x[t] * 2^-k(t) (the per-row power-of-two RMS rule of moe_decode_layer); resid may
 * be NULL or x. Outputs: inds u32 [T][K], scores bf16 [T][K], y bf16 [T][H].
 */
int moe_prefill_layer(const void *x, int T, int H, int I, int E, int K, const void *router_w,
                      const uint32_t *wg, const void *sg, const void *bg, const uint32_t *wu,
                      const void *su, const void *bu, const uint32_t *wd, const void *sd, const void *bd,
                      int sb_fp16, int norm, const void *resid, uint32_t *out_inds, void *out_scores,
                      void *y, void *workspace, size_t workspace_bytes, void *stream);

/*
 * The cached-layer form of the prefill GEMMs (CachedSwitchGLU.__call__ with L > 1,
 * mlx-qwen38/loader.py:566-699): experts in slot buffers [cap][...] (MLX layout), slots u32
 * [T][K] = the slot of each (token, k) assignment, or any value >= cap to skip it. Writes the
 * unweighted expert outputs of the assignments it runs to yk_out bf16 [T*K][H] (assignment
 * order t*K + k) and leaves the other rows untouched, so chunks of a prompt's experts can be
 * run one after another into the same buffer. Workspace: moe_prefill_workspace_bytes(T, H, I,
 * cap, K).
 */
int moe_prefill_experts_slots(const void *x, int T, int H, int I, int cap, int K, const uint32_t *slots,
                              const uint32_t *wg, const void *sg, const void *bg, const uint32_t *wu,
                              const void *su, const void *bu, const uint32_t *wd, const void *sd,
                              const void *bd, int sb_fp16, void *yk_out, void *workspace,
                              size_t workspace_bytes, void *stream);

/* y[t] = bf16(resid[t] + sum_k bf16(yk[t*K + k] * scores[t][k])), the sum sequential in bf16
 * over k in MLX order (loader.py:914,965); resid may be NULL. */
int moe_combine_rows(const void *yk, int T, int K, int H, const void *scores, const void *resid, void *y,
                     void *stream);

/* xn[t] = x[t] * 2^-k(t): the per-row power-of-two RMS normalisation of moe_decode_layer. */
int moe_pow2_rows(const void *x, int T, int H, void *xn, void *stream);

/* ------------------------------------------------------------------------------------ */
/* Shared expert and affine-quantised linear layers (csrc/shared.cu).                      */
/* ------------------------------------------------------------------------------------ */

/*
 * y [T, N] bf16 = x [T, Kin] bf16 . W^T with W an affine-quantised matrix in MLX layout:
 * codes u32 [N, Kin*bits/32], scales/biases [N, Kin/group_size] (bf16, or fp16 with
 * sb_fp16 = 1). Replaces QLinear::forward (mlx-qwen38/cpp/src/kernels.cpp:997-1019, a
 * quantized_matmul with transpose=True). bits 2, 4 or 8; group_size a multiple of 32/bits
 * that divides Kin; at most 384 groups per row. Arithmetic: per group, float sums of q*x and
 * of x in input order; scale*sum(qx) + bias*sum(x) in double; the double sum over groups in
 * group order, rounded to float then bf16.
 */
int moe_affine_linear(const void *x, int T, int Kin, int N, const void *w, const void *scales, const void *biases,
                      int bits, int group_size, int sb_fp16, void *y, void *stream);

/* bytes of device workspace moe_shared_expert needs for T tokens (0 for bad sizes) */
size_t moe_shared_expert_workspace_bytes(int T, int H, int I);

/*
 * The layer's shared expert (mlx-qwen38/cpp/src/engine.cpp:394-400, loader.py:909-910):
 *   g = x.Wg^T, u = x.Wu^T ([T, I]), act = bf16(bf16(g*bf16(sigmoid(g)))*u),
 *   o = act.Wd^T ([T, H]), gl = x.We^T ([T, 1]), y = bf16(bf16(sigmoid(gl)) * o).
 * Wg/Wu/Wd share `bits`/`group_size` (4-bit g64 in the reference's models); the scalar gate
 * We has its own (8-bit g64). y [T, H] bf16 is the `shared_y` addend of moe_experts_down /
 * moe_decode_layer. workspace >= moe_shared_expert_workspace_bytes(T, H, I).
 */
int moe_shared_expert(const void *x, int T, int H, int I, const void *wg, const void *sg, const void *bg,
                      const void *wu, const void *su, const void *bu, const void *wd, const void *sd, const void *bd,
                      int bits, int group_size, const void *weg, const void *seg, const void *beg, int gate_bits,
                      int gate_group_size, int sb_fp16, void *y, void *workspace, size_t workspace_bytes,
                      void *stream);

/* ------------------------------------------------------------------------------------ */
/* Hyper-connection mixer before the MoE block (csrc/hc.cu).                              */
/* ------------------------------------------------------------------------------------ */

/* bytes of device workspace moe_hc_mix needs (0 for bad sizes) */
size_t moe_hc_workspace_bytes(int T, int HC, int H, int R);

/*
 * One call of Qwen38Engine::run_hc (mlx-qwen38/cpp/src/kernels.cpp:1363-1560) with
 * affine-quantised mixer matrices, for T rows of HC streams of H values:
 *   h [T, HC*H] bf16; branch [T, H] and gate [T, HC] bf16 (both NULL = no write);
 *   norm_w [HC*H] bf16 (the norm scales 1 + norm_w); eps the RMS epsilon;
 *   down [R, HC*H], up [HC*H, R], inject [HC, HC*H] (codes u32 + scales/biases, NULL inject =
 *   the use_combine=False mixer, inj then zeros).
 * Outputs: written [T, HC*H] (h plus the write; required with a write, untouched without),
 * mixed [T, H] (the block input), inj [T, HC] (the next write's gate; may be NULL).
 * T <= 16 uses the reference's decode rounding (unrounded dot products), T > 16 its prefill
 * rounding. HC must be 4. workspace >= moe_hc_workspace_bytes(T, HC, H, R).
 */
int moe_hc_mix(const void *h, int T, int HC, int H, int R, const void *branch, const void *gate, const void *norm_w,
               float eps, const void *wd, const void *sd, const void *bd, int dbits, int dgs, const void *wu,
               const void *su, const void *bu, int ubits, int ugs, const void *wi, const void *si, const void *bi,
               int ibits, int igs, int sb_fp16, void *written, void *mixed, void *inj, void *workspace,
               size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------------ */
/* Expert parallelism: one process per GPU, experts split in contiguous blocks.           */
/* ------------------------------------------------------------------------------------ */

/* Bytes of a CUDA IPC handle as moe_ep_buffer_alloc writes it. */
#define MOE_EP_HANDLE_BYTES 64

/* Bytes of one rank's exchange buffer for batches of up to T tokens (flags + two receive
 * buffers [T][K][H] bf16). */
size_t moe_ep_buffer_bytes(int T, int K, int H);

/* Allocates (cudaMalloc) and zero-fills an exchange buffer on the current device and writes
 * its CUDA IPC handle (MOE_EP_HANDLE_BYTES) to out_handle for the other ranks. */
int moe_ep_buffer_alloc(size_t bytes, void **out_ptr, void *out_handle);

/* Maps another rank's exchange buffer from its handle (cudaIpcOpenMemHandle, peer access
 * enabled); moe_ep_buffer_close unmaps it, moe_ep_buffer_free frees this rank's own. */
int moe_ep_buffer_open(const void *handle, void **out_ptr);
int moe_ep_buffer_close(void *ptr);
int moe_ep_buffer_free(void *ptr);

/* Workspace bytes for moe_ep_decode_layer; zero-fill it once before first use. */
size_t moe_ep_workspace_bytes(int T, int H, int I, int E, int K);

/*
 * One decode step of a layer whose E experts are split across nranks GPUs: this rank holds
 * experts [e_begin, e_begin + e_count) (weights in the MLX layout, indexed from e_begin) and
 * the whole bf16 router [E, H]. Router (+ norm as in moe_decode_layer) and top-k run on every
 * rank (identical results), the local experts run on their (token, k) slots, and one kernel
 * exchanges the unweighted expert outputs over NVLink (peer stores into every rank's exchange
 * buffer, bounded waits on per-rank epoch flags) and combines them in MLX order:
 * y = bf16(resid + sum_k bf16(yk * score_k)), the same bits on every rank and, for T < 32,
 * as moe_decode_layer; from T = 32 up the local experts run as the grouped tensor-core GEMMs
 * of the prefill path and the result equals moe_prefill_layer's. peers: device array [nranks] of exchange-buffer pointers (this rank's own
 * at [rank], the others from moe_ep_buffer_open), all sized for at least T tokens. Every rank
 * must call this the same number of times, in the same order, with the same T. Replaces the
 * per-layer decode body of mlx-qwen38/loader.py:903-922 (single device in the reference).
 */
int moe_ep_decode_layer(const void *x, int T, int H, int I, int E, int K, int e_begin, int e_count,
                        const void *router_w, const uint32_t *wg, const void *sg, const void *bg,
                        const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                        const void *sd, const void *bd, int sb_fp16, int norm, const void *resid,
                        void *const *peers, int rank, int nranks, uint32_t *out_inds, void *out_scores,
                        void *y, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Token-sharded expert parallelism (routed all-to-all) for batches with several tokens per
 * GPU. Rank r of nranks owns tokens [first, first + n) of the batch (moe_ep_a2a_local_tokens:
 * contiguous blocks of ceil(T / nranks)) and experts [e_first[r], e_first[r + 1]) (e_first:
 * host array of nranks + 1 boundaries, e_first[0] = 0, e_first[nranks] = E). Per call, on
 * every rank: power-of-two normalisation and router / top-k of its own tokens; ONE kernel
 * stores each own token's normalised row into the exchange buffer of every rank owning one
 * of its routed experts (once per token and rank) and its routing row into every rank's
 * table, then waits (bounded, epoch flags) for every rank; the local experts over all tokens
 * routed to them (grouped tcgen05 GEMMs for T >= 32, int8 GEMVs below); ONE kernel stores each
 * computed (token, k) output row into its token owner's exchange buffer, waits, and the owner
 * combines y = bf16(resid + sum_k bf16(yk * score_k)) in MLX order. Results equal the same call
 * with nranks = 1 bit for bit. x, resid, y: [n][H] of this rank's tokens; out_inds u32 /
 * out_scores bf16 [n][K]. peers: device array of every rank's exchange buffer (this rank's
 * own at [rank]); own_buffer: this rank's buffer (host-known device address). Exchange
 * buffers of moe_ep_a2a_buffer_bytes(T, K, H, nranks) from moe_ep_buffer_alloc; every rank
 * makes the same calls in the same order with the same T. No reference counterpart (the
 * reference runs on one device); replaces the per-layer block of mlx-qwen38/loader.py:903-922.
 */
size_t moe_ep_a2a_buffer_bytes(int T, int K, int H, int nranks);
size_t moe_ep_a2a_workspace_bytes(int T, int H, int I, int E, int K, int nranks);
/* number of tokens rank owns, *first = its first token */
int moe_ep_a2a_local_tokens(int T, int nranks, int rank, int *first);
int moe_ep_a2a_layer(const void *x, int T, int H, int I, int E, int K, const int *e_first,
                     const void *router_w, const uint32_t *wg, const void *sg, const void *bg,
                     const uint32_t *wu, const void *su, const void *bu, const uint32_t *wd,
                     const void *sd, const void *bd, int sb_fp16, int norm, const void *resid,
                     void *const *peers, const void *own_buffer, int rank, int nranks,
                     uint32_t *out_inds, void *out_scores, void *y, void *workspace,
                     size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------------ */
/* Mixer + shared expert for all layers in one launch per token (decode).                */
/* ------------------------------------------------------------------------------------ */

/* One layer's weights (device pointers, MLX affine layout, bf16 or fp16 scales/biases as
 * sb_fp16 says): the mixer's norm weight (bf16 [4H]), down [R][4H], up [4H][R] and inject
 * [4][4H] (8-bit, group 64; inject may be NULL), the shared expert's gate / up [I][H] and
 * down [H][I] (4-bit, group 64) and its scalar gate [1][H] (8-bit, group 64). */
typedef struct {
    const void *norm_w;
    const void *wd, *sd, *bd, *wu, *su, *bu, *wi, *si, *bi;
    const void *wsg, *ssg, *bsg, *wsu, *ssu, *bsu, *wsd, *ssd, *bsd, *wse, *sse, *bse;
} moe_f3_layer;

/* Workspace bytes for moe_f3_stack_decode. */
size_t moe_f3_stack_workspace_bytes(int H, int R, int I);

/*
 * One token through L layers of the step in front of each MoE block, the block's output being
 * the shared expert: per layer (mixed, state, inj) = moe_hc_mix(state, write = (branch, inj of
 * the layer before)), branch = moe_shared_expert(mixed), with the same bits as those two calls
 * (decode regime), in ONE cooperative launch (one CTA per SM, or num_ctas >= 128; five grid
 * barriers per layer). layers: device array [L] of moe_f3_layer. h: the first layer's streams bf16
 * [4H]; branch0 / gate0: a pending write (bf16 [H] / [4]) or both NULL. Outputs: state_out
 * [4H] (the last block's output written into the streams), branch_out [H] and inj_out [4] (the
 * last block output and its stream gate; inj_out may be NULL), branch_all [L][H] (every
 * layer's block output) or NULL. H, R, I multiples of 64; buffers 16-byte aligned. Replaces
 * the per-layer run_hc + shared-expert launches of Qwen38Engine (mlx-qwen38/cpp/src/
 * engine.cpp:390-400, kernels.cpp:1363-1560) for a decode step.
 */
int moe_f3_stack_decode(const void *layers, int L, int H, int R, int I, int sb_fp16, float eps, const void *h,
                        const void *branch0, const void *gate0, void *state_out, void *branch_out, void *inj_out,
                        void *branch_all, void *workspace, size_t workspace_bytes, int num_ctas, void *stream);

/* One layer of moe_f3moe_stack_decode: its mixer + shared expert (as moe_f3_layer) and its
 * routed block (as moe_stack_layer: the transposed router [H][E] bf16 and the E packed experts). */
typedef struct {
    moe_f3_layer mix;
    const void *router_t;
    const void *experts;
} moe_f3moe_layer;

/* Workspace bytes for moe_f3moe_stack_decode (Is: the shared expert's intermediate size,
 * I: the routed experts'). */
size_t moe_f3moe_stack_workspace_bytes(int H, int R, int Is, int I, int E, int K);

/*
 * The MoE half of L decoder layers on one token in ONE cooperative launch: per layer
 *   (mixed, state, inj) = moe_hc_mix(state, write = (branch, inj of the layer before))
 *   routing of mixed (router logits, precise softmax, MLX-order top-k, renorm: moe_router_topk)
 *   shared = moe_shared_expert(mixed)
 *   branch = sum_k bf16(expert_k(mixed) * s_k) + shared   (moe_experts_gateup / moe_experts_down
 *            with the shared output as the addend: the reference's routed + shared combine,
 *            loader.py:909-914, engine.cpp:390-400)
 * with the same bits as those calls (decode regime; router logits as in moe_stack_decode:
 * exact partial dot products summed in double). layers: device array [L] of moe_f3moe_layer;
 * sb_fp16_mix / sb_fp16_experts: fp16 (1) or bf16 (0) scales of the mixer + shared weights /
 * of the packed experts. h, branch0, gate0, state_out, branch_out, inj_out, branch_all as in
 * moe_f3_stack_decode; inds_out u32 [L][K] and scores_out bf16 [L][K] as in moe_stack_decode;
 * mixed_all bf16 [L][H] (every layer's mixer output, the block input) or NULL.
 * One CTA per SM (num_ctas = 0) or num_ctas >= 128, five grid barriers per layer. Requires
 * H % 256 == 0, H <= 4096, R, Is, I multiples of 64, E <= 512 and a multiple of 8, K <= 32; buffers
 * 16-byte aligned.
 */
int moe_f3moe_stack_decode(const void *layers, int L, int H, int R, int Is, int I, int E, int K, int sb_fp16_mix,
                           int sb_fp16_experts, float eps, const void *h, const void *branch0, const void *gate0,
                           void *state_out, void *branch_out, void *inj_out, uint32_t *inds_out, void *scores_out,
                           void *branch_all, void *mixed_all, void *workspace, size_t workspace_bytes, int num_ctas,
                           void *stream);

/* ------------------------------------------------------------------------------------ */
/* K50 expert pack (one directory per layer: codes.bin, scales.bf16, bias.bf16,          */
/* index.json; replaces ExpertPackCpp, mlx-qwen38/cpp/src/loader.cpp:1187-1470).          */
/* ------------------------------------------------------------------------------------ */

/* Opens a layer directory and parses its index; NULL on error (moe_last_error()). */
void *moe_k50_open(const char *layer_dir);
void moe_k50_close(void *pack);
/* Number of expert records of a projection ("gate_proj", ...), or of dense records ("dense"). */
int moe_k50_count(void *pack, const char *proj);
/* Name of dense record i, NUL-terminated into out. */
int moe_k50_dense_name(void *pack, int i, char *out, size_t out_bytes);
/* Record of (proj, expert) -- expert < 0: the dense record named proj -- as out8 = {bits,
 * group_size, rows, cols, uint32 code words per row, groups per row, kind (0 tern, 1 2t,
 * 2 "2", 3 "3", 4 "4", 5 "6", 6 "8"), unit (0 hot, 1 warm, 2 mid, 3 cold, 4 dense, -1 other)}
 * of its materialised form (ExpertPackCpp::materialize_as_affine2, loader.cpp:1379-1470). */
int moe_k50_record(void *pack, const char *proj, int expert, int64_t *out8);
/* Materialises the record into host buffers: codes uint32 [rows][words], scales / biases bf16
 * bits [rows][groups]. "tern": base-3 digits unpacked into 2-bit codes, biases = -scales;
 * other kinds: codes as stored, biases from bias.bf16 (or -scales when it has none). */
int moe_k50_materialize(void *pack, const char *proj, int expert, uint32_t *codes, uint16_t *scales,
                        uint16_t *biases);

/* ------------------------------------------------------------------------------------ */
/* Per-layer LRU expert-slot cache with its state on the GPU.                             */
/* ------------------------------------------------------------------------------------ */

/* Device bytes of one layer's cache state (E experts, cap slots; E <= 2048, cap <= E), 0 if
 * invalid. Allocate 16-byte aligned device memory of this size per layer. */
size_t moe_lru_state_bytes(int E, int cap);

/* Initialises a layer's state: empty cache (free stack pops slots 0, 1, 2, ...), zero counters;
 * expert_bytes is the unit of the byte counters. Replaces c_layer_init's cache part
 * (mlx-qwen38/expert_io.c:497-520, reset 450-468). */
int moe_lru_init(void *state, int E, int cap, uint64_t expert_bytes, void *stream);

/* what = 0: empty the cache (expert_io.c:450-468); 1: zero the counters (470-495). */
int moe_lru_reset(void *state, int E, int cap, int what, void *stream);

/* One decode step (expert_io.c:583-676, c_layer_step_decode_ex): eids = device u32 [k]
 * (the router's output, read in place), k <= 32 and k <= cap. Writes out_slots (device u32
 * [k]) and out_miss = device i32 [1 + 2k] {n_miss, missing eids (request order) .., their
 * slots ..}. Hit/prefetch-hit/miss counting against the last prefetch's snapshot, eviction
 * from the LRU end skipping this step's experts, all as the reference. An eid >= E sets the
 * device error word and writes n_miss = -1 without touching the cache. */
int moe_lru_step(void *state, int E, int cap, const uint32_t *eids, int k, uint32_t *out_slots,
                 int32_t *out_miss, void *stream);

/* Router-driven prefetch (expert_io.c:527-581, c_layer_start_prefetch): pred = device i32 [n]
 * (ranked predictions, n <= 64), 1 <= max_fetch <= 32. Writes out_fetch = device i32
 * [1 + 2*max_fetch] {count, eids .., slots ..} of the experts to fill (inserted in reverse
 * rank order). */
int moe_lru_prefetch(void *state, int E, int cap, const int32_t *pred, int n, int max_fetch,
                     int32_t *out_fetch, void *stream);

/* Device bytes of the per-token I/O accounting record shared by every layer
 * (cpp/third_party/expert_io.c:97-111): {int32 enabled, int32 current token (-1: none),
 * 8 pad bytes, u64 counters[9] in c_end_decode_token order}. Allocate 16-byte aligned device
 * memory of this size, zero it and set the token to -1. */
size_t moe_lru_acct_bytes(void);

/* moe_lru_step with per-token accounting and the scheduled-step variant. acct: null or the
 * record above; with enabled != 0 the step adds its LRU hits, prefetch hits, wasted
 * prefetches and demand misses, and (token >= 0) its demand re-reads of experts evicted at
 * most 16 / 64 tokens earlier, and stamps evicted experts with the token
 * (cpp/third_party/expert_io.c:745-806). sched != 0 (cpp/third_party/expert_io.c:1129-1270):
 * eviction also skips the experts the layer's last prefetch fetched, and out_miss must hold
 * 1 + 3k entries: after the lists, hit flags [k] (1: the expert was resident) in request
 * order. */
int moe_lru_step_ex(void *state, int E, int cap, const uint32_t *eids, int k, uint32_t *out_slots,
                    int32_t *out_miss, void *acct, int sched, void *stream);

/* moe_lru_prefetch with accounting (prefetch loads; prefetch re-reads, token >= 0) and, with
 * sched != 0, a prediction listed twice fetched once (cpp/third_party/expert_io.c:1290-1340). */
int moe_lru_prefetch_ex(void *state, int E, int cap, const int32_t *pred, int n, int max_fetch,
                        int32_t *out_fetch, void *acct, int sched, void *stream);

/* out = device i32 [1 + 2*cap] {count, eids (LRU -> MRU) .., slots ..}
 * (expert_io.c:726-747, c_layer_get_lru_state). */
int moe_lru_get_state(void *state, int E, int cap, int32_t *out, void *stream);

/* Rebuilds the cache from device arrays eids/slots [n] in LRU -> MRU order and adds to the
 * prefill counters (expert_io.c:749-789, c_layer_set_lru_state). */
int moe_lru_set_state(void *state, int E, int cap, const int32_t *eids, const int32_t *slots, int n,
                      uint64_t add_req, uint64_t add_hits, uint64_t add_misses, void *stream);

/* out18 = device u64 [18], the counters in c_layer_get_stats order (expert_io.c:791-812). */
int moe_lru_get_stats(void *state, int E, int cap, uint64_t *out18, void *stream);

/* counters[index] += value (the prefill byte accounting of c_layer_load_sync). */
int moe_lru_add_stat(void *state, int E, int cap, int index, uint64_t value, void *stream);

/* Fills the experts of a list {n, eids[stride], slots[stride]} (device memory, as written
 * by moe_lru_step / moe_lru_prefetch) from a pinned host pool into device slot buffers, for
 * ntensors (<= 9) per-expert row arrays: row e of tensor t at host_src[t] + e * row_bytes[t]
 * goes to dev_dst[t] + slot * row_bytes[t]. A kernel reads the list and the mapped pinned
 * pool (no host round trip). Replaces the pread pool (expert_io.c:113-356). host_src, dev_dst
 * and row_bytes are host arrays; bases and row bytes 16-byte aligned. num_ctas 0 = all SMs. */
int moe_fill_slots(const int32_t *list, int stride, int E, int cap, int ntensors,
                   const void *const *host_src, void *const *dev_dst, const uint64_t *row_bytes,
                   int num_ctas, void *stream);

/* Same fill for a list in host memory: one cudaMemcpyAsync per (expert, tensor) on stream. */
int moe_fill_slots_host(const int32_t *list_host, int stride, int E, int cap, int ntensors,
                        const void *const *host_src, void *const *dev_dst, const uint64_t *row_bytes,
                        void *stream);

/* ------------------------------------------------------------------------------------ */
/* The reference's expert cache C ABI, drop-in (mlx-qwen38/expert_io.c:428-852; the       */
/* waits of cpp/third_party/expert_io.c:1048). Same names, signatures and conventions     */
/* (one calling thread, layers 0..63, bad layer ids ignored); the cache state is on the   */
/* GPU and expert bytes come from a pinned host pool by cudaMemcpyAsync.                  */
/* ------------------------------------------------------------------------------------ */

void c_io_init(int num_threads);
/* fd and base_offsets are accepted and unused (no SSD shard): register the pinned host pool
 * with c_layer_set_host_pool. E = 512 and a 1,536,000-byte counter unit, as the reference. */
void c_layer_init(int layer_idx, int fd, int capacity, const uint64_t *base_offsets,
                  const uint64_t *row_bytes, const uint64_t *base_ptrs, uint64_t slot_inds_ptr);
/* Extension: any E, counter unit, tensor count, and the host pool at once. */
int c_layer_init_ex(int layer_idx, int num_experts, int capacity, uint64_t expert_bytes, int ntensors,
                    const uint64_t *row_bytes, const uint64_t *base_ptrs, const uint64_t *host_ptrs,
                    uint64_t slot_inds_ptr);
/* Extension: pinned host pool bases per tensor (row e of tensor t at host_ptrs[t] + e*row_bytes[t]). */
void c_layer_set_host_pool(int layer_idx, const uint64_t *host_ptrs);
void c_layer_reset_cache(int layer_idx);
void c_layer_reset_stats(int layer_idx);
void c_layer_wait_prefetch(int layer_idx);
void c_layer_wait_demand(int layer_idx);
void c_layer_start_prefetch(int layer_idx, const int32_t *pred_eids, int pred_count, int max_fetch);
void c_layer_start_prefetch10(int layer_idx, int max_fetch, int32_t e0, int32_t e1, int32_t e2, int32_t e3,
                              int32_t e4, int32_t e5, int32_t e6, int32_t e7, int32_t e8, int32_t e9);
void c_layer_start_prefetch12(int layer_idx, int max_fetch, int32_t e0, int32_t e1, int32_t e2, int32_t e3,
                              int32_t e4, int32_t e5, int32_t e6, int32_t e7, int32_t e8, int32_t e9,
                              int32_t e10, int32_t e11);
int c_layer_step_decode_ex(int layer_idx, const uint32_t *eids, int k, int async_io);
int c_layer_step_decode(int layer_idx, const uint32_t *eids, int k);
int c_layer_step_decode10(int layer_idx, uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3, uint32_t e4,
                          uint32_t e5, uint32_t e6, uint32_t e7, uint32_t e8, uint32_t e9);
int c_layer_step_decode10_async(int layer_idx, uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3,
                                uint32_t e4, uint32_t e5, uint32_t e6, uint32_t e7, uint32_t e8, uint32_t e9);
void c_layer_load_sync(int layer_idx, const int32_t *eids, const int32_t *slots, int count, int is_prefill);
void c_layer_get_lru_state(int layer_idx, int32_t *out_eids, int32_t *out_slots, int *out_count);
void c_layer_set_lru_state(int layer_idx, const int32_t *ordered_eids, const int32_t *ordered_slots, int count,
                           uint64_t add_prefill_requests, uint64_t add_prefill_hits, uint64_t add_prefill_misses);
void c_layer_get_stats(int layer_idx, uint64_t *out_stats);
void c_get_decode_totals(int num_layers, uint64_t *out6);

/* The newer reference's additions (cpp/src/expert_io.h:8-12, 87-106; behaviour of
 * cpp/third_party/expert_io.c:1002-1396). Accounting is off by default; when on, every step
 * and prefetch counts into one record shared by all layers, read per token: */
void c_set_io_accounting(int enabled);           /* off also ends the token in progress */
void c_begin_decode_token(int token_idx);        /* token_idx unused: tokens are counted */
/* out10 = {LRU hits, demand misses, prefetch loads, prefetch hits, wasted prefetches,
 * demand re-reads within 16 / 64 tokens, prefetch re-reads within 16 / 64 tokens, bytes
 * filled into slots} since c_begin_decode_token */
void c_end_decode_token(uint64_t *out10);
/* bytes of this module's own buffers: device LRU states and staging buffers */
uint64_t c_get_native_buffer_bytes(void);
/* the last recorded hit/miss split of layer_idx (a scheduled step with flag 4 whose demand
 * missed some but not all experts): hit slots, miss slots, and for each request its index
 * in hits ++ misses */
void c_layer_get_split_inds(int layer_idx, uint32_t *out_hit_slots, uint32_t *out_miss_slots,
                            int32_t *out_inv_order);
/* One call per layer (cpp/third_party/expert_io.c:1094-1396): demand step of layer_idx
 * (> 0; k capped at 16; its last prefetch's experts stay protected) and, unless flags & 2,
 * the deduplicated prefetch of pred [n_pred <= 64] into next_layer (> 0, at most
 * prefetch_cap, 32 when out of 1..31). Demand fills are queued before prefetch fills;
 * flags & 1, or no demand miss, waits for all fills; flags & 4 records the split above.
 * Returns the demand misses; c_layer_wait_demand waits for the fills. */
int c_layer_decode_step_sched(int layer_idx, const int32_t *eids, int k, const int32_t *pred, int n_pred,
                              int next_layer, int prefetch_cap, int flags);

/*
 * P1 I/O scheduler (replaces qwen38::P1IoScheduler, mlx-qwen38/cpp/src/io_sched.h:46-245, with
 * the observable behaviour of mlx-qwen38/cpp/src/io_sched.cpp, tested by
 * mlx-qwen38/cpp/tests/test_io_sched.cpp): URGENT / PREFETCH read queues, prefetch cancel /
 * promote, per-slot pins with a reader-wait callback, an LRU slot cache per layer (layers
 * 0..63, experts 0..511, up to 9 tensors per expert). The scheduler's whole state lives in
 * device memory (the device that is current at moe_p1_create); every method is one control
 * kernel on that state, and the rows it takes from the queues are copied by a copy kernel
 * (pool sources, device slots) or by the calling host thread (file sources or host slots).
 * Each method of the reference class is one function taking the handle; void methods return
 * 0 (or a negative status). Rows come from a file (fd, byte offsets: moe_p1_layer_init, the
 * reference's form) or from a pool of num_experts experts (addresses of expert 0 of every
 * tensor, pinned host or device memory: moe_p1_layer_init_pool) into host or device slot
 * buffers. Workers: without moe_p1_init nothing is taken until a caller waits (the
 * reference's behaviour without workers, deterministic); after moe_p1_init(n) every queued
 * row is taken at the end of each call. The wait-reader callback may only wait for readers
 * and unpin; a call that finds only pinned slots evictable resumes after it returns.
 */
#define MOE_P1_STATS 16
/* stats order: decode_requests, lru_hits, urgent_reads, prefetch_issued, prefetch_cancelled,
 * prefetch_promoted, prefetch_used, prefetch_wasted, pin_waits, bytes, io_wait_ns,
 * forced_invalidations, prefill_requests, prefill_lru_hits, prefill_demand_misses,
 * prefill_demand_bytes (the fields of qwen38::P1LayerStats) */
void *moe_p1_create(void);
void moe_p1_destroy(void *h);
int moe_p1_init(void *h, int num_threads);                     /* P1IoScheduler::init */
int moe_p1_shutdown(void *h);                                  /* ::shutdown */
int moe_p1_num_threads(void *h);
/* ::set_wait_reader_callback: fn(user, layer) is called, without the scheduler lock, when a
 * slot allocation finds only slots pinned by a GPU reader; it should wait for that reader and
 * unpin (moe_p1_unpin_layer_slots) */
int moe_p1_set_wait_reader_callback(void *h, void (*fn)(void *user, int layer), void *user);
int moe_p1_layer_init(void *h, int layer, int fd, int capacity, int num_tensors, const uint64_t *base_offsets,
                      const uint64_t *row_bytes, const uint64_t *base_ptrs, uint64_t slot_inds_ptr);
int moe_p1_layer_init_pool(void *h, int layer, int capacity, int num_tensors, int num_experts,
                           const uint64_t *src_ptrs, const uint64_t *row_bytes, const uint64_t *slot_ptrs,
                           uint64_t slot_inds_ptr, int slots_on_device, int device);
int moe_p1_resize_layer(void *h, int layer, int new_capacity, const uint64_t *new_base_ptrs, uint64_t slot_inds_ptr,
                        const int32_t *ordered_eids, const int32_t *ordered_slots, int count);
int moe_p1_reset_cache(void *h, int layer);
int moe_p1_reset_stats(void *h, int layer);
int moe_p1_start_prefetch(void *h, int layer, const int32_t *pred_eids, int pred_count, int max_fetch);
/* returns the number of the k slots still loading (wait with moe_p1_wait_layer_urgent) */
int moe_p1_step_decode(void *h, int layer, const uint32_t *eids, int k, uint32_t *out_slots);
int moe_p1_wait_layer_urgent(void *h, int layer);
int moe_p1_wait_layer_all(void *h, int layer);
int moe_p1_wait_all(void *h);
int moe_p1_unpin_layer_slots(void *h, int layer);
int moe_p1_pin_slots(void *h, int layer, const uint32_t *slots, int count);
int moe_p1_unpin_slots(void *h, int layer, const uint32_t *slots, int count);
int moe_p1_get_slot_pin_count(void *h, int layer, int slot);
/* ::force_invalidate with the handle's std::mt19937_64 (seeded by moe_p1_seed); returns the count */
int moe_p1_seed(void *h, uint64_t seed);
int moe_p1_force_invalidate(void *h, int layer, double rate);
int moe_p1_load_sync(void *h, int layer, const int32_t *eids, const int32_t *slots, int count, int is_prefill);
int moe_p1_get_lru_state(void *h, int layer, int32_t *out_eids, int32_t *out_slots, int *out_count);
int moe_p1_set_lru_state(void *h, int layer, const int32_t *ordered_eids, const int32_t *ordered_slots, int count,
                         uint64_t add_prefill_requests, uint64_t add_prefill_hits, uint64_t add_prefill_misses);
int moe_p1_get_layer_stats(void *h, int layer, uint64_t *out_stats);
int moe_p1_get_total_stats(void *h, int num_layers, uint64_t *out_stats);
uint64_t moe_p1_copy_errors(void *h);          /* rows that could not be copied (short reads, bad ids) */
uint64_t moe_p1_launches(void *h);             /* control and copy kernels launched so far */

/* ------------------------------------------------------------------------------------ */
/* Token loop around the stack: embedding rows, LM-head logits, next-token choice.          */
/* ------------------------------------------------------------------------------------ */

/*
 * out[t] = table[ids[t]] (bf16 rows of H). The prompt/next-token embedding lookup of the
 * reference's decode loop (mlx-qwen38/server.py:148-151,184-185, loader.py:1150-1180: the
 * model call on token ids). ids int32 on the device; an id outside [0, V) gives a zero row and
 * sets bit 2 of the device error word. H % 8 == 0, table/out 16-byte aligned.
 */
int moe_embed_tokens(const void *table, int V, int H, const int32_t *ids, int T, void *out, void *stream);

/*
 * logits [T, V] fp32 = head [V, H] bf16 x rows [T, H] bf16 (T <= 4): the LM head that yields
 * `out.logits` in the reference's loop (server.py:150-151,185). Every bf16 x bf16 product is
 * exact in fp32; each row's products are summed in double in a fixed order and rounded once to
 * fp32 (results do not depend on the launch configuration).
 */
int moe_lm_head_logits(const void *head, int V, int H, const void *x, int T, float *logits, void *stream);

/* Bytes of workspace moe_lm_head_argmax needs (8 per token row). */
size_t moe_lm_head_argmax_workspace_bytes(int T);

/*
 * The LM head and the greedy choice in one pass (loader.py:1171-1176: lm(cur_tok) then
 * mx.argmax(out.logits[:, -1:, :])): ids[t] = the first index of the maximum of the logits
 * moe_lm_head_logits computes (same values; logits may be NULL when only the ids are wanted).
 * The workspace (8-byte aligned) must be zero-filled before its first use; every call leaves it
 * zero-filled again, so calls that share one must not overlap on the GPU.
 */
int moe_lm_head_argmax(const void *head, int V, int H, const void *x, int T, float *logits, int32_t *ids,
                       void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of workspace moe_sample_tokens needs (temperature > 0 only). */
size_t moe_sample_workspace_bytes(int T, int V);

/*
 * Next token per row of logits [T, V] fp32, replacing server.py:93-110 `_sample_next_token`:
 * temperature <= 0: argmax (the first index of the maximum, as mx.argmax);
 * temperature > 0: scaled = logits / temperature; with 0 < top_p < 1 the candidates are the
 * largest probabilities of softmax(scaled) whose mass reaches top_p (every token tied at the
 * boundary probability is kept; the reference keeps the boundary tokens in its sort order);
 * one categorical draw from softmax(scaled) over the candidates by the Gumbel-max rule, the
 * uniform variate of (seed, counter, row, index) from a splitmix64 hash (a different random
 * stream from MLX's; the same (seed, counter) gives the same tokens). top_p in (0, 1].
 * ids int32 [T] on the device.
 */
int moe_sample_tokens(const float *logits, int T, int V, float temperature, float top_p, uint64_t seed,
                      uint64_t counter, int32_t *ids, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Device-side error word (bit 1: a bounded mbarrier/flag wait gave up, bit 2: invalid
 * input seen by a kernel, bit 4: an expert-parallel peer did not signal within 2 s). Returns the current value (>= 0) and clears it when `clear`.
 * Kernels never trap: they record the condition here and skip the affected work.
 */
int moe_device_error(int clear);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
