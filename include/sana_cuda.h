/*
 * sana_cuda.h — C ABI of the B200 (sm_100a) implementation of the Sana-0.6B denoiser path
 * of cconthekeyboard/sana.cpp: the linear-attention DiT blocks, their step and the
 * DPM-Solver++ classifier-free-guidance loop; and the steps on either side of it: the text
 * encoder's output contract (the conditioning the loop reads) and the DC-AE VAE decoder.
 *
 * Plain C: opaque handle, raw pointers and sizes, int status codes. Every call that takes
 * host buffers copies them to the device, runs, copies results back and synchronises; the
 * *_device variants take device pointers and run asynchronously on the handle's stream
 * (sana_cuda_stream) until sana_cuda_synchronize.
 *
 * Layouts are the reference's unless stated otherwise: fp32, row-major; activations
 * [batch, tokens, hidden]; images / latents NCHW; linear weights [in, out]
 * (SanaDenoiserWeights as load_linear_weight_tensor leaves them, weights_io.cpp:367-377)
 * or [out, in] with SANA_LAYOUT_TORCH; conv weights [out, in, kh, kw].
 *
 * Errors: every function returns SANA_OK or an error code; the message of the last
 * failure on a handle is sana_cuda_last_error(handle). SANA_ERR_INVALID corresponds to the
 * reference's std::invalid_argument, SANA_ERR_CUDA / SANA_ERR_TIMEOUT / SANA_ERR_STATE to
 * std::runtime_error. A handle is not thread-safe (the reference is single-threaded).
 */
#ifndef SANA_CUDA_H
#define SANA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sana_cuda_ctx sana_cuda_ctx;

enum {
    SANA_OK = 0,
    SANA_ERR_INVALID = 1, /* argument / shape error */
    SANA_ERR_CUDA = 2,    /* CUDA runtime error */
    SANA_ERR_TIMEOUT = 3, /* a bounded device-side wait gave up; the kernel returned early */
    SANA_ERR_STATE = 4,   /* call order (e.g. no weights uploaded) */
    SANA_ERR_NOMEM = 5
};

enum { SANA_MODE_BF16 = 0, SANA_MODE_F32 = 1 };
enum { SANA_LAYOUT_REFERENCE = 0, SANA_LAYOUT_TORCH = 1 };

/* Model dimensions (SanaDenoiserWeights / SanaBlockWeights shapes, transformer.h:26-79). */
typedef struct {
    int n_blocks;        /* 28 for Sana-0.6B */
    int hidden;          /* 1152 */
    int latent_channels; /* 32 */
    int caption_dim;     /* 2304 */
    int ff_expanded;     /* 5760 (GLUMBConv inverted width; the point conv reads half) */
    int self_heads;      /* 36 in the reference's callers (infer_main.cpp:366) */
    int cross_heads;     /* 16 */
} sana_dims;

/* --- lifetime ------------------------------------------------------------------------ */

/* Creates a handle on CUDA device `device`. mode: SANA_MODE_BF16 (bf16 operands, fp32
 * accumulation and residual stream, tcgen05 tensor cores) or SANA_MODE_F32 (fp32
 * everywhere, CUDA-core GEMMs; the parity check mode). No reference counterpart: the
 * reference has no device state. */
int sana_cuda_create(int device, int mode, sana_cuda_ctx **out);
void sana_cuda_destroy(sana_cuda_ctx *ctx);
const char *sana_cuda_last_error(const sana_cuda_ctx *ctx);
/* The cudaStream_t all work of the handle runs on (as void*). */
void *sana_cuda_stream(sana_cuda_ctx *ctx);
/* Runs later work on `stream` (a cudaStream_t; NULL restores the handle's own stream). */
int sana_cuda_set_stream(sana_cuda_ctx *ctx, void *stream);
/* Waits for the handle's stream and reports device-side timeouts. */
int sana_cuda_synchronize(sana_cuda_ctx *ctx);
/* Failure detection (no reference counterpart; the reference has no device waits). Every
 * spin in this library's kernels (mbarrier waits of the TMA / tensor-core pipelines, flag
 * waits) gives up after the handle's wait limit, records the
 * timeout in the handle's device error word and unwinds; the call then returns
 * SANA_ERR_TIMEOUT and the handle stays usable. sana_cuda_set_wait_limit sets that limit in
 * nanoseconds (>= 1000; default 2 s), sana_cuda_wait_limit reads it. */
int sana_cuda_set_wait_limit(sana_cuda_ctx *ctx, unsigned long long ns);
unsigned long long sana_cuda_wait_limit(const sana_cuda_ctx *ctx);
/* Self-test of that path: one device thread waits, with the handle's limit, for the int at
 * device address `flag` to equal `expect`. SANA_OK once it does, SANA_ERR_TIMEOUT when the
 * limit runs out first. */
int sana_cuda_selftest_wait(sana_cuda_ctx *ctx, const int *flag, int expect);
/* --- classifier-free guidance across two GPUs (latency mode) ----------------------------------
 * One process and handle per GPU. The two noise predictions of a step meet once, inside the
 * guidance + scheduler kernel, over NVLink peer memory (apply_classifier_free_guidance,
 * transformer.cpp:570-602; step_sana_scheduler, scheduler.cpp:272-318): each GPU pushes its
 * prediction into the other's receive buffer and waits (bounded by the wait limit) for the
 * other's. Setup: both export, swap the 64-byte handles (any host channel), both connect; GPU 0
 * takes branch 0 (unconditional), GPU 1 branch 1 (conditional). Both then call
 * sana_cuda_denoise_loop_pair_device with the same latents, shapes and schedule, each with its
 * own branch's B encoder sequences [B, L, enc_dim] and bias [B, 1, L], and both receive the
 * same guided latents. A timeout (SANA_ERR_TIMEOUT) leaves the exchange out of step: export and
 * connect again. */
#define SANA_PAIR_HANDLE_BYTES 64
int sana_cuda_cfg_pair_export(sana_cuda_ctx *ctx, size_t max_latent_elems, void *handle);
int sana_cuda_cfg_pair_connect(sana_cuda_ctx *ctx, int branch, const void *peer_handle);
int sana_cuda_cfg_pair_close(sana_cuda_ctx *ctx);
int sana_cuda_denoise_loop_pair_device(sana_cuda_ctx *ctx, const float *latents, int B, int H, int W,
                                       const float *enc, int L, int enc_dim, const float *bias, float guidance,
                                       int num_steps, float flow_shift, float *out);

/* Kernel launches in the last captured denoising loop replay (0 before the first replay). */
int sana_cuda_last_launch_count(const sana_cuda_ctx *ctx);
/* Process-wide number of dense projections dispatched to the tcgen05 tensor-core kernel
 * and to the CUDA-core kernel (fp32 check mode, tiny or unaligned shapes). */
void sana_cuda_gemm_counts(long long *tensor_core, long long *cuda_core);

/* Profiling: runs the denoising loop of sana_cuda_denoise_loop_device once without graph
 * capture, with CUDA events around every kernel launch on the handle's stream, and writes a
 * JSON object {"kernel class": [launches, total milliseconds], ...} to `report`. */
int sana_cuda_profile_loop(sana_cuda_ctx *ctx, const float *latents, int B, int H, int W, const float *enc, int L,
                           int enc_dim, const float *bias, float guidance, int num_steps, float flow_shift, float *out,
                           char *report, size_t report_len);

/* Diagnostics: copies `bytes` at `offset` of a named workspace buffer of the last call
 * (a, qkv, ao, cq, xb, ffh, glu, x, x1, x2, x3, mods, tmod, emb, ckv1, ctx, kvlen, noise,
 * lat, part) to `host`; *size_out receives the buffer's size. No reference counterpart. */
int sana_cuda_debug_read(sana_cuda_ctx *ctx, const char *name, size_t offset, size_t bytes, void *host,
                         size_t *size_out);

/* --- weights --------------------------------------------------------------------------- */

/* Uploads the denoiser weights into the handle's device cache (bf16 or fp32 by mode).
 * Replaces holding SanaDenoiserWeights (transformer.h:64-79) as built by
 * load_denoiser_weights (transformer.cpp:453-488).
 *   model[16]: caption.linear_1_weight, caption.linear_1_bias, caption.linear_2_weight,
 *     caption.linear_2_bias, patch_embed_weight, patch_embed_bias,
 *     time_embed_linear_1_weight, _bias, time_embed_linear_2_weight, _bias,
 *     time_projection_weight, _bias, caption_norm_weight, final_scale_shift_table,
 *     proj_out_weight, proj_out_bias                (the struct's field order)
 *   blocks[26 * n_blocks]: per block the SanaBlockWeights fields in order
 *     (scale_shift_table, attn_norm_gamma, attn_norm_beta, q_weight, q_bias, k_weight,
 *      k_bias, v_weight, v_bias, out_weight, out_bias, cross_q_weight, cross_q_bias,
 *      cross_k_weight, cross_k_bias, cross_v_weight, cross_v_bias, cross_out_weight,
 *      cross_out_bias, mlp_norm_gamma, mlp_norm_beta, ff_inverted_weight,
 *      ff_inverted_bias, ff_depth_weight, ff_depth_bias, ff_point_weight).
 * Bias pointers may be NULL (zero), norm gamma/beta NULL (identity), as the loader's
 * defaults (transformer.cpp:361-398). Weight pointers must not be NULL. */
int sana_cuda_upload_weights(sana_cuda_ctx *ctx, const sana_dims *dims, const float *const *model,
                             const float *const *blocks, int layout);

/* GGUF weight files, read without ggml: the reference's model_weights.gguf,
 * caption_weights.gguf and denoiser_weights.gguf (infer_main.cpp:347-365), whose tensors
 * load_weight_index / load_weight_tensor (weights_io.cpp:134-164, 325-377) read as fp32 and
 * load_denoiser_weights (transformer.cpp:166-488) assembles by name. sana_gguf_* index one
 * file (no device needed); sana_cuda_upload_gguf maps the three files, resolves the
 * reference's names and block prefixes ("<prefix>.scale_shift_table", ordered by trailing
 * index), checks the shapes as the loaders do and uploads straight from the mapping into the
 * device cache (linear weights stay in the files' [out, in] layout), filling *dims_out if
 * not NULL. Errors follow the loaders: a missing tensor is SANA_ERR_INVALID ("weight name not
 * found in weight index"), an unreadable or malformed file, a non-fp32 tensor or a shape
 * mismatch SANA_ERR_STATE (std::runtime_error). */
typedef struct sana_gguf sana_gguf;
int sana_gguf_open(const char *path, sana_gguf **out, char *err, size_t err_len);
void sana_gguf_close(sana_gguf *file);
int sana_gguf_tensor_count(const sana_gguf *file);
/* index of the named tensor, or -1 */
int sana_gguf_find(const sana_gguf *file, const char *name);
/* tensor i: name, element type (0 fp32, 1 fp16, 30 bf16, others as the file says), rank,
 * the first max_rank extents slowest-first (numpy / PyTorch order), its bytes in the
 * mapping (valid until sana_gguf_close) and their count (0 for types other than those three). */
int sana_gguf_tensor_info(const sana_gguf *file, int i, const char **name, int *type, int *rank, int64_t *shape,
                          int max_rank, const void **data, uint64_t *nbytes);
/* byte offset of tensor i's data from the start of the file (SavedWeightInfo::offset of
 * weights_io.h:19-25, gguf_get_data_offset + gguf_get_tensor_offset in weights_io.cpp:156) */
int sana_gguf_tensor_offset(const sana_gguf *file, int i, uint64_t *offset);
int sana_cuda_upload_gguf(sana_cuda_ctx *ctx, const char *model_path, const char *caption_path,
                          const char *denoiser_path, int self_heads, int cross_heads, sana_dims *dims_out);

/* Optional RMSNorm of the cross-attention query and key projections over each token's
 * hidden channels (q = RMSNorm(x Wq + bq) * q_weight, k = RMSNorm(ctx Wk + bk) * k_weight, eps
 * inside the root), as later Sana checkpoints normalise q / k. No counterpart in the reference:
 * its block (transformer_ops.cpp:572-608) has no such norm, and the option is off by default
 * and after every weight upload. q_weights / k_weights: n_blocks pointers to [hidden] fp32
 * (a NULL array or entry = ones); enable = 0 switches it off. Applies to every later call. */
int sana_cuda_set_cross_qk_norm(sana_cuda_ctx *ctx, int enable, const float *const *q_weights,
                                const float *const *k_weights, float eps);

/* --- the denoiser path (host buffers) --------------------------------------------------- */

/* run_full_denoising_loop_with_cfg (transformer.h:140-148, transformer.cpp:692-724) with a
 * fresh scheduler state of `num_steps` steps (init_sana_scheduler_state, scheduler.h:40):
 * caption projection, then the 20-step (or num_steps) DPM-Solver++ loop.
 *   latents [B, Cl, H, W]; enc [2B, L, caption_dim] (uncond block first); bias [2B, 1, L]
 *   additive mask or NULL; out [B, Cl, H, W]. The whole loop runs as one CUDA graph from
 *   the second call with the same shapes on. */
int sana_cuda_denoise_loop(sana_cuda_ctx *ctx, const float *latents, int B, int H, int W, const float *enc, int L,
                           int enc_dim, const float *bias, float guidance, int num_steps, float flow_shift,
                           float *out);

/* The same with device pointers (fp32), asynchronous on the handle's stream. */
int sana_cuda_denoise_loop_device(sana_cuda_ctx *ctx, const float *latents, int B, int H, int W, const float *enc,
                                  int L, int enc_dim, const float *bias, float guidance, int num_steps,
                                  float flow_shift, float *out);

/* run_full_denoising_step_with_cfg (transformer.h:131-139, transformer.cpp:604-690): one
 * step on latents [B, Cl, H, W] (updated in place) with the projected context
 * [2B, L, hidden], at timestep value `timestep`, with an explicit scheduler state
 * (SanaSchedulerState, scheduler.h:27-32): sigmas[n_sigmas], *step_index,
 * *lower_order_count, history[*n_history x numel] (converted outputs, oldest first,
 * capacity 2 x numel), all updated as step_sana_scheduler does (scheduler.cpp:272-318). */
int sana_cuda_denoise_step(sana_cuda_ctx *ctx, float *latents, int B, int H, int W, const float *context, int L,
                           const float *bias, float guidance, float timestep, const float *sigmas, int n_sigmas,
                           int *step_index, int *lower_order_count, float *history, int *n_history);

/* The timestep embedding (sinusoidal features, timestep_embedder MLP with SiLU; emb, which the
 * final layer's modulation reads) and t_block (SiLU then the 6C projection) for S sequences at
 * timesteps t[S] (transformer.cpp:77-122, 638-656): emb [S, hidden] and tmod [S, 6 * hidden] to
 * host buffers (either may be NULL). In bf16 mode the three projections run on the tensor cores
 * as inside the loop. */
int sana_cuda_time_embed(sana_cuda_ctx *ctx, const float *timesteps, int S, float *emb, float *tmod);

/* One denoiser forward without CFG or scheduler for S independent sequences at timestep t:
 * patch embed, time embedding, all blocks, final layer (transformer.cpp:631-681).
 *   latents [S, Cl, H, W]; context [S, L, hidden] (projected); bias [S, 1, L] or NULL;
 *   noise_pred out [S, Cl, H, W]. */
int sana_cuda_forward(sana_cuda_ctx *ctx, const float *latents, int S, int H, int W, float t, const float *context,
                      int L, const float *bias, float *noise_pred);

/* block_forward (transformer.h:149-155, transformer.cpp:726-778) of block `block`.
 *   x [S, T, hidden] (T a square), context [S, L, hidden], timestep modulation
 *   tmod [S, 6 * hidden], bias [S, 1, L] or NULL; any stage output may be NULL
 *   (SanaBlockStageOutputs, transformer.h:20-24). */
int sana_cuda_block_forward(sana_cuda_ctx *ctx, int block, const float *x, int S, int T, const float *context, int L,
                            const float *tmod, const float *bias, float *after_self, float *after_cross,
                            float *after_ff);

/* run_model_blocks (transformer.h:118-126, transformer.cpp:544-568): blocks [begin, end). */
int sana_cuda_run_model_blocks(sana_cuda_ctx *ctx, const float *x, int S, int T, const float *context, int L,
                               const float *tmod, const float *bias, int begin, int end, float *out);

/* project_caption_context with the uploaded caption weights (transformer.cpp:701-708;
 * transformer_ops.cpp:64-76): enc [S, L, caption_dim] -> out [S, L, hidden]. */
int sana_cuda_project_caption(sana_cuda_ctx *ctx, const float *enc, int S, int L, int enc_dim, float *out);

/* --- single operations (host buffers, reference semantics and layouts) ------------------ */

/* linear_3d_lastdim / linear_2d (common_ops.cpp:114-209): x [rows, K], w [K, N], bias [N]. */
int sana_op_linear(sana_cuda_ctx *ctx, const float *x, int rows, int K, const float *w, const float *bias, int N,
                   float *out);
/* Tensor::layer_norm_3d_lastdim (tensor.cpp:188-271): x [rows, C]. */
int sana_op_layer_norm(sana_cuda_ctx *ctx, const float *x, int rows, int C, float eps, const float *gamma,
                       const float *beta, float *out);
/* Tensor::rms_norm_3d_lastdim (tensor.cpp:276-316). */
int sana_op_rms_norm(sana_cuda_ctx *ctx, const float *x, int rows, int C, float eps, const float *weight, float *out);
/* Tensor::modulate_3d_lastdim (tensor.cpp:323-376): x [B, T, C], shift/scale [B, 1, C]. */
int sana_op_modulate(sana_cuda_ctx *ctx, const float *x, int B, int T, int C, const float *shift, const float *scale,
                     float *out);
/* linear_attention_4d (transformer_ops.cpp:402-543): q [B, H, Tq, D], k/v [B, H, Tk, D]. */
int sana_op_linear_attention(sana_cuda_ctx *ctx, const float *q, const float *k, const float *v, int B, int H, int Tq,
                             int Tk, int D, float *out);
/* attention_4d (transformer_ops.cpp:348-392): softmax(q k^T / sqrt(D) + bias) v, bias [B, 1, Tk]. */
int sana_op_attention(sana_cuda_ctx *ctx, const float *q, const float *k, const float *v, int B, int H, int Tq,
                      int Tk, int D, const float *bias, float *out);
/* conv2d_1x1 (common_ops.cpp:322-405): x [B, Cin, H, W], w [Cout, Cin, 1, 1]. */
int sana_op_conv1x1(sana_cuda_ctx *ctx, const float *x, int B, int Cin, int H, int W, const float *w,
                    const float *bias, int Cout, float *out);
/* depthwise_conv2d_3x3 (common_ops.cpp:510-572): x [B, C, H, W], w [C, 1, 3, 3]. */
int sana_op_depthwise3x3(sana_cuda_ctx *ctx, const float *x, int B, int C, int H, int W, const float *w,
                         const float *bias, float *out);
/* glumb_conv (common_ops.cpp:733-761): x [B, Cin, H, W] -> [B, Cout, H, W]. */
int sana_op_glumb_conv(sana_cuda_ctx *ctx, const float *x, int B, int Cin, int H, int W, const float *w_inv,
                       const float *b_inv, int E, const float *w_dw, const float *b_dw, const float *w_pt, int Cout,
                       float *out);
/* project_caption_context (transformer_ops.cpp:64-76) with explicit weights ([in, out]). */
int sana_op_project_caption(sana_cuda_ctx *ctx, const float *enc, int B, int L, int Din, const float *w1,
                            const float *b1, int C, const float *w2, const float *b2, const float *norm_w, float *out);
/* attention_block_3d (transformer_ops.cpp:545-570): weights [C, C] ([in, out]), biases may be NULL. */
int sana_op_attention_block(sana_cuda_ctx *ctx, const float *x, int B, int T, int C, const float *wq, const float *bq,
                            const float *wk, const float *bk, const float *wv, const float *bv, const float *wo,
                            const float *bo, int heads, float *out);
/* cross_attention_block_3d (transformer_ops.cpp:572-608): context [B, L, C], bias [B, 1, L] or NULL. */
int sana_op_cross_attention_block(sana_cuda_ctx *ctx, const float *x, int B, int T, int C, const float *context,
                                  int L, const float *bias, const float *wq, const float *bq, const float *wk,
                                  const float *bk, const float *wv, const float *bv, const float *wo, const float *bo,
                                  int heads, float *out);
/* apply_classifier_free_guidance (transformer.cpp:570-602): noise [2B, Cl, H, W] -> [B, Cl, H, W]. */
int sana_op_cfg(sana_cuda_ctx *ctx, const float *noise, int B, int Cl, int H, int W, float guidance, float *out);

/* split_heads_3d (transformer_ops.cpp:83-122): [B, T, hidden] -> [B, heads, T, hidden/heads]. */
int sana_op_split_heads(sana_cuda_ctx *ctx, const float *in, int B, int T, int hidden, int heads, float *out);
/* merge_heads_4d (transformer_ops.cpp:128-171): [B, H, T, D] -> [B, T, H*D]. */
int sana_op_merge_heads(sana_cuda_ctx *ctx, const float *in, int B, int H, int T, int D, float *out);
/* attention_scores_4d (transformer_ops.cpp:178-225): unscaled q k^T per (batch, head);
 * q [B, H, Tq, D], k [B, H, Tk, D] -> [B, H, Tq, Tk]. */
int sana_op_attention_scores(sana_cuda_ctx *ctx, const float *q, const float *k, int B, int H, int Tq, int Tk, int D,
                             float *out);
/* softmax_lastdim_4d (transformer_ops.cpp:278-339) over `rows` rows of n values. */
int sana_op_softmax_lastdim(sana_cuda_ctx *ctx, const float *in, long long rows, int n, float *out);
/* attention_values_4d (transformer_ops.cpp:232-273): probs [B, H, Tq, Tk] . v [B, H, Tk, D]. */
int sana_op_attention_values(sana_cuda_ctx *ctx, const float *probs, const float *v, int B, int H, int Tq, int Tk,
                             int D, float *out);
/* compute_sana_block_modulation (transformer.cpp:496-542): t_mod [B, 6C] + table [6, C]
 * -> [B, 6C]; its six C-wide column blocks are shift_msa, scale_msa, gate_msa, shift_mlp,
 * scale_mlp, gate_mlp. */
int sana_op_block_modulation(sana_cuda_ctx *ctx, const float *tmod, const float *table, int B, int C, float *out);

/* --- device-pointer kernels (microbenchmarks; bf16 activations, token-major, asynchronous
 *     on the handle's stream) ------------------------------------------------------------ */

/* out[M, N] (bf16) = act(A[M, K] . B[N, K]^T + bias): the dense projections of
 * linear_3d_lastdim / conv2d_1x1 (common_ops.cpp:177, :322). act: 0 none, 1 SiLU, 2 GELU-tanh. */
int sana_op_gemm_device(sana_cuda_ctx *ctx, const void *A, const void *B, int M, int N, int K, const float *bias,
                        int act, void *out);
/* The same product with an fp32 output out[M, N] (the projections that write the fp32
 * residual stream and the noise prediction do), e.g. to read the epilogue's activations at
 * full precision. */
int sana_op_gemm_f32out_device(sana_cuda_ctx *ctx, const void *A, const void *B, int M, int N, int K,
                               const float *bias, int act, float *out);
/* The residual projection of a block stage (the attention / cross-attention output and the
 * Mix-FFN point projection, transformer.cpp:740-777): out[M, N] (fp32) =
 * resid + gate[row / rows_per_gate] * (A . B^T + bias), gate NULL = 1, bias NULL = 0; out
 * may alias resid; out_bf16 (may be NULL) receives a bf16 copy of out. */
int sana_op_gemm_residual_device(sana_cuda_ctx *ctx, const void *A, const void *B, int M, int N, int K,
                                 const float *bias, const float *resid, const float *gate, int rows_per_gate,
                                 float *out, void *out_bf16);
/* linear_attention_4d on the fused QKV rows [S*T, 3*heads*D] -> [S*T, heads*D]; partial is
 * fp32 scratch of sana_op_linear_attention_workspace() bytes. */
int sana_op_linear_attention_device(sana_cuda_ctx *ctx, const void *qkv, int S, int T, int heads, int D,
                                    float *partial, void *out);
size_t sana_op_linear_attention_workspace(int S, int T, int heads, int D);

/* Size of the fixed scratch behind sana_op_linear_attention_noalloc (8 MiB). */
#define SANA_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)

/* sana_op_linear_attention_device without the workspace argument, and without any device
 * allocation: the fp32 scratch comes from one fixed array of SANA_NOALLOC_SCRATCH_BYTES
 * built into this library's device image. There is no counterpart in the reference (its
 * linear_attention_4d allocates its intermediates on the host); it is an addition for
 * callers that cannot allocate device memory at the point of the call and have no
 * workspace of their own to lend: a host that has already handed its device memory to its
 * own pool allocator, or a tight loop where cudaMalloc/cudaFree would stall it (cudaFree
 * synchronises the whole device). Inputs, output and results are those of
 * sana_op_linear_attention_device; the work is queued on the handle's stream.
 *  - Limit: sana_op_linear_attention_workspace(S, T, heads, D) must not exceed
 *    SANA_NOALLOC_SCRATCH_BYTES (two 1024-token sequences fit, at 36 x 32 or 16 x 72 heads).
 *    Larger shapes return SANA_ERR_INVALID, with the sizes in sana_cuda_last_error(), and
 *    launch nothing.
 *  - First call on each device: it looks up the scratch's device address, with the handle's
 *    device made current for the call, and the CUDA runtime may load this library's device
 *    code there at that moment. Make that first call before any stream capture begins. The
 *    address is remembered per device together with the id of the CUDA context it belongs
 *    to; if that context has been replaced (cudaDeviceReset re-creates the primary context),
 *    the next call looks the address up again, so the first call after a reset is another
 *    set-up call with the same rule.
 *  - Nothing in the scratch has to start at zero: every call writes each scratch word
 *    before reading it.
 *  - All handles, streams and host threads on one device share the one scratch. Two calls
 *    whose GPU work can overlap (different streams or handles with no ordering between
 *    them) race on it and give wrong results: keep such calls on one stream, or order them
 *    with events. */
int sana_op_linear_attention_noalloc(sana_cuda_ctx *ctx, const void *qkv, int S, int T, int heads, int D, void *out);
/* depthwise_conv2d_3x3 + GLU gate on NHWC rows [S*H*W, E] -> [S*H*W, E/2]; w [E, 9], b [E] fp32,
 * both 16-byte aligned (the kernel bulk-copies them into shared memory). */
int sana_op_depthwise_glu_device(sana_cuda_ctx *ctx, const void *in, int S, int H, int W, int E, const float *w,
                                 const float *b, void *out);
/* layer_norm (no affine) followed by modulate_3d_lastdim (tensor.cpp:243-265, 323-376) on
 * device rows: x [rows, C] fp32, sequence s = row / rows_per_seq takes shift = mod + s*mod_ld
 * + shift_idx*C and scale = mod + s*mod_ld + scale_idx*C; out [rows, C] bf16. */
int sana_op_ln_modulate_device(sana_cuda_ctx *ctx, const float *x, long long rows, int C, int rows_per_seq,
                               const float *mod, long long mod_ld, int shift_idx, int scale_idx, float eps,
                               void *out);
/* attention_4d for cross-attention: q [S*T, heads*D], kv [S*L, 2*heads*D] (k | v), bias
 * [S, L] fp32 or NULL, kv_len int[S] scratch (filled from bias), out [S*T, heads*D]. */
int sana_op_cross_attention_device(sana_cuda_ctx *ctx, const void *q, const void *kv, const float *bias,
                                   int *kv_len, int S, int T, int L, int heads, int D, void *out);

/* --- scheduler (scheduler.h:34-65) ----------------------------------------------------- */

/* SanaSchedulerConfig (scheduler.h:9-20) as plain fields. The string-valued fields map to
 * flags: use_flow_sigmas, final_sigmas_zero (final_sigmas_type == "zero"), solver_heun
 * (solver_type "heun" rather than "midpoint"); timestep_spacing "linspace",
 * prediction_type "flow_prediction" and algorithm_type "dpmsolver++" are the only values
 * the reference accepts and are not carried. sana_scheduler_config_default fills the
 * reference's defaults (make_sana_scheduler_config, scheduler.cpp:85-87). Every entry
 * point below that takes a config checks it as validate_scheduler_config does
 * (scheduler.cpp:8-24): solver_order 1 or 2, else SANA_ERR_INVALID. */
typedef struct sana_scheduler_config {
    int num_train_timesteps;
    float flow_shift;
    int use_flow_sigmas;
    int solver_order;
    int lower_order_final;
    int final_sigmas_zero;
    int solver_heun;
} sana_scheduler_config;
void sana_scheduler_config_default(sana_scheduler_config *config);

/* build_sana_scheduler_timesteps (scheduler.cpp:89-141) for any config: timesteps[n],
 * sigmas[n + 1]; SANA_ERR_INVALID where the reference throws (flow sigmas, zero final
 * sigma and num_train_timesteps > 0 required). Host only. */
int sana_scheduler_schedule_config(const sana_scheduler_config *config, int n, float *timesteps, float *sigmas);
/* sana_scheduler_update with a config: flow or variance-preserving sigmas
 * (sigma_to_alpha_sigma_t, scheduler.cpp:71-77), midpoint or heun second order
 * (scheduler.cpp:250-269). */
int sana_scheduler_update_config(sana_cuda_ctx *ctx, const sana_scheduler_config *config, int order,
                                 const float *sigmas, int n_sigmas, int step_index, const float *m0, const float *m1,
                                 const float *sample, int numel, float *out);
/* sana_scheduler_step with a config: the order chosen as step_sana_scheduler chooses it
 * (solver_order, lower_order_final, final_sigmas_type; scheduler.cpp:291-311), the history
 * kept to solver_order outputs. */
int sana_scheduler_step_config(sana_cuda_ctx *ctx, const sana_scheduler_config *config, const float *sigmas,
                               int n_sigmas, int *step_index, int *lower_order_count, float *history, int *n_history,
                               const float *model_output, const float *sample, int numel, float *out);
/* sana_cuda_denoise_step with a config (run_full_denoising_step_with_cfg passes its
 * SanaSchedulerConfig to step_sana_scheduler, transformer.cpp:683-689). */
int sana_cuda_denoise_step_config(sana_cuda_ctx *ctx, const sana_scheduler_config *config, float *latents, int B,
                                  int H, int W, const float *context, int L, const float *bias, float guidance,
                                  float timestep, const float *sigmas, int n_sigmas, int *step_index,
                                  int *lower_order_count, float *history, int *n_history);
/* sana_cuda_denoise_loop with a config: a fresh state built from `config`
 * (init_sana_scheduler_state) run to its last step, as one CUDA graph from the second call. */
int sana_cuda_denoise_loop_config(sana_cuda_ctx *ctx, const sana_scheduler_config *config, const float *latents,
                                  int B, int H, int W, const float *enc, int L, int enc_dim, const float *bias,
                                  float guidance, int num_steps, float *out);

/* build_sana_scheduler_timesteps (scheduler.cpp:89-141), default config with flow_shift;
 * host only: timesteps[n], sigmas[n + 1]. */
int sana_scheduler_schedule(int n, float flow_shift, float *timesteps, float *sigmas);
/* convert_sana_scheduler_model_output (scheduler.cpp:155-173) on the device. */
int sana_scheduler_convert(sana_cuda_ctx *ctx, const float *sigmas, int n_sigmas, int step_index,
                           const float *model_output, const float *sample, int numel, float *out);
/* sana_scheduler_first_order_update (order 1, m0 = converted output) or
 * sana_scheduler_second_order_update (order 2, history [m1, m0]) (scheduler.cpp:175-270). */
int sana_scheduler_update(sana_cuda_ctx *ctx, int order, const float *sigmas, int n_sigmas, int step_index,
                          const float *m0, const float *m1, const float *sample, int numel, float *out);
/* step_sana_scheduler (scheduler.cpp:272-318) with an explicit state: history
 * [n_history x numel] oldest first (n_history <= 2, capacity 2 x numel), updated in place
 * together with *step_index, *lower_order_count and *n_history. */
int sana_scheduler_step(sana_cuda_ctx *ctx, const float *sigmas, int n_sigmas, int *step_index,
                        int *lower_order_count, float *history, int *n_history, const float *model_output,
                        const float *sample, int numel, float *out);

/* --- synthetic inputs -------------------------------------------------------------------- */

/* randn_torch_cpu (torch_rng.cpp:35-68): torch.randn of n >= 16 float32 values on a CPU
 * generator seeded with `seed`, bit-identical to the reference's restatement. Host only. */
int sana_randn_torch_cpu(float *out, size_t n, uint64_t seed);

/* --- the text-encoder output contract ----------------------------------------------------- */

/* select_rows_first_and_last (gemma_encoder.h:45-48, gemma_encoder.cpp:51-77): row 0 of
 * in [rows, cols], then its last keep-1 rows, into out [keep, cols]. Host only;
 * SANA_ERR_INVALID with the reference's message in err when keep is not in (0, rows]. */
int sana_select_rows_first_and_last(const float *in, size_t rows, size_t cols, size_t keep, float *out, char *err,
                                    size_t err_len);

/* The host tail of encode_prompt_pair (gemma_encoder.h:50-55, gemma_encoder.cpp:188-244),
 * after the encoder produced its hidden states: negative [max_seq, hidden] (the negative
 * prompt padded straight to max_seq, negative_real real tokens) and positive
 * [positive_rows, hidden] (instruction prefix + prompt padded to positive_rows,
 * positive_real real tokens) -> embeddings [2, max_seq, hidden] negative first, the positive
 * branch sliced to row 0 plus its last max_seq-1 rows, and bias [2, 1, max_seq] =
 * (1 - mask) * -10000 over the real tokens kept. Host only; the reference's
 * std::invalid_argument cases return SANA_ERR_INVALID with its message in err. */
int sana_prompt_pair_assemble(const float *negative, size_t negative_rows, size_t negative_real,
                              const float *positive, size_t positive_rows, size_t positive_real, size_t hidden,
                              size_t max_sequence_length, float *embeddings, float *bias, char *err,
                              size_t err_len);

/* The same for `pairs` (1..64) prompt pairs on the device, one launch on the handle's stream:
 * negative [pairs, L, hidden] and positive [pairs, positive_rows, hidden] fp32 device
 * buffers, real-token counts in host arrays negative_real[pairs] / positive_real[pairs] ->
 * enc [2 * pairs, L, hidden] (all negative branches first, the denoiser's batch order) and
 * bias [2 * pairs, 1, L], ready for sana_cuda_denoise_loop_device. */
int sana_cuda_prompt_pairs_device(sana_cuda_ctx *ctx, int pairs, const float *negative, const int *negative_real,
                                  const float *positive, int positive_rows, const int *positive_real, int hidden,
                                  int L, float *enc, float *bias);

/* --- the VAE decoder (vae.h:11-92, vae.cpp:243-325, vae_ops.cpp) ---------------------------- */

/* The decoder's structure, mirroring SanaVaeWeights (vae.h:43-73): up block i has `channels`
 * outputs, an optional nearest-2x upsample conv from block i+1's channels (every block but
 * the innermost), then `layers` ResBlocks (is_res_block) or attention + GLUMBConv layers.
 * head_dim is the attention head size (32, run_vae_decode's value, vae.cpp:292); ms_kernel
 * the multiscale depthwise size (proj_in's 3 or 5); scaling_factor divides the latents first
 * (0.41407 for Sana, infer_main.cpp:369-374). */
typedef struct sana_vae_block {
    int channels, has_upsample, is_res_block, layers;
} sana_vae_block;
typedef struct sana_vae_dims {
    int latent_channels, out_channels, n_blocks, head_dim, ms_kernel;
    float scaling_factor;
    sana_vae_block blocks[8];
} sana_vae_dims;

/* load_vae_weights (vae.cpp:147-170) from host fp32 tensors in PyTorch layouts, in order:
 *   conv_in.w [C_{n-1}, latent, 3, 3], conv_in.b, norm_out.w [C_0], norm_out.b,
 *   conv_out.w [out, C_0, 3, 3], conv_out.b; then per up block i = 0..n-1:
 *   [upsample conv.w [C_i, C_{i+1}, 3, 3], conv.b] when it has one;
 *   per ResBlock: conv1.w [C, C, 3, 3], conv1.b, conv2.w, norm.w, norm.b;
 *   per attention layer: to_q.w [C, C], to_k.w, to_v.w, proj_in.w [3C, 1, k, k],
 *   proj_out.w [3C, head_dim, 1, 1], to_out.w [C, 2C], norm_out.w, norm_out.b,
 *   conv_inverted.w [8C, C, 1, 1], conv_inverted.b, conv_depth.w [8C, 1, 3, 3],
 *   conv_depth.b, conv_point.w [C, 4C, 1, 1], norm.w, norm.b.
 * Shape errors of validate_vae_weights (vae.cpp:172-208) are SANA_ERR_INVALID. */
int sana_cuda_vae_upload(sana_cuda_ctx *ctx, const sana_vae_dims *dims, const float *const *tensors);

/* load_vae_weights (vae.cpp:147-170) from the reference's vae_decoder_weights.gguf: up blocks
 * found by their "decoder.up_blocks.<n>" prefixes in numeric order, an upsample conv at
 * layer 0 when "<prefix>.0.conv.weight" exists, ResBlocks when the first layer after it has
 * conv1, else attention + GLUMBConv layers; three layers per block; fp32 tensors under their
 * diffusers names uploaded straight from the mapping. Fills *dims_out if not NULL. A missing
 * tensor is SANA_ERR_INVALID ("weight name not found in weight index"); an unreadable file, a
 * non-fp32 tensor or a shape mismatch SANA_ERR_STATE. */
int sana_cuda_vae_upload_gguf(sana_cuda_ctx *ctx, const char *path, float scaling_factor, sana_vae_dims *dims_out);

/* run_vae_decode (vae.cpp:243-325): latents [B, latent, h, w] fp32 NCHW (host) -> image
 * [B, out, h * 2^u, w * 2^u] fp32 NCHW (host), u = the number of upsampling blocks (5 for
 * DC-AE f32c32: 32x32 latents give a 1024x1024 image). */
int sana_cuda_vae_decode(sana_cuda_ctx *ctx, const float *latents, int B, int h, int w, float *out);
/* The same with device pointers, asynchronous on the handle's stream. */
int sana_cuda_vae_decode_device(sana_cuda_ctx *ctx, const float *latents, int B, int h, int w, float *out);
/* Kernel and GEMM launches of the last decode on this handle. */
int sana_cuda_vae_last_launch_count(const sana_cuda_ctx *ctx);

#ifdef __cplusplus
}
#endif
#endif /* SANA_CUDA_H */
