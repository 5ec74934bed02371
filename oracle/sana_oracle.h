/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the Sana denoiser hot path.
 *
 * A plain-C restatement of the reference's fp32 CPU algorithm (cconthekeyboard/sana.cpp,
 * src/tensor.cpp, src/common_ops.cpp, src/transformer_ops.cpp, src/transformer.cpp,
 * src/scheduler.cpp, src/torch_rng.cpp). Each function names the reference lines it
 * follows. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it, and only as the checker; the product never calls it.
 *
 * Parity pin: tests/test_oracle_pin.py checks every function here against the
 * reference's own known-answer tests (values transcribed in tests/golden/reference_kats.json)
 * and against the compiled reference (oracle/_ref/libsana_ref.so, fixtures in tests/golden/).
 *
 * Layout conventions are the reference's: activations [batch, tokens, hidden] fp32
 * row-major; linear weights [in, out]; conv weights [out, in, kh, kw]; images NCHW.
 * Status: 0 ok, 1 invalid argument, 2 other error (message in orc_last_error()).
 */
#ifndef SANA_ORACLE_H
#define SANA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char *orc_last_error(void);

int orc_randn(float *out, size_t n, uint64_t seed);

int orc_linear_3d(const float *x, size_t B, size_t T, size_t K, const float *w, const float *bias,
                  size_t N, float *out);
int orc_layer_norm(const float *x, size_t B, size_t T, size_t C, float eps, const float *gamma,
                   const float *beta, float *out);
int orc_rms_norm(const float *x, size_t B, size_t T, size_t C, float eps, const float *weight,
                 float *out);
int orc_modulate(const float *x, size_t B, size_t T, size_t C, const float *shift,
                 const float *scale, float *out);
int orc_linear_attention(const float *q, const float *k, const float *v, size_t B, size_t H,
                         size_t Tq, size_t Tk, size_t D, float *out);
int orc_attention(const float *q, const float *k, const float *v, size_t B, size_t H, size_t Tq,
                  size_t Tk, size_t D, const float *bias, float *out);
int orc_conv1x1(const float *x, size_t B, size_t Cin, size_t H, size_t W, const float *w,
                const float *bias, size_t Cout, float *out);
int orc_depthwise3x3(const float *x, size_t B, size_t C, size_t H, size_t W, const float *w,
                     const float *bias, float *out);
int orc_glumb_conv(const float *x, size_t B, size_t Cin, size_t H, size_t W, const float *w_inv,
                   const float *b_inv, size_t E, const float *w_dw, const float *b_dw,
                   const float *w_pt, size_t Cout, float *out);
int orc_project_caption(const float *enc, size_t B, size_t L, size_t Din, const float *w1,
                        const float *b1, size_t C, const float *w2, const float *b2,
                        const float *norm_w, float *out);
int orc_cfg(const float *noise, size_t B, size_t Cl, size_t H, size_t W, float g, float *out);

int orc_scheduler_schedule(size_t n, float flow_shift, float *timesteps, float *sigmas);
int orc_scheduler_run(size_t n_steps, float flow_shift, const float *model_outputs,
                      const float *sample, size_t numel, float *samples_out);

/* SanaSchedulerConfig (scheduler.h:9-20) as plain fields (the C ABI's sana_scheduler_config). */
typedef struct orc_sched_config {
    int num_train_timesteps;
    float flow_shift;
    int use_flow_sigmas;
    int solver_order;
    int lower_order_final;
    int final_sigmas_zero;
    int solver_heun;
} orc_sched_config;
/* init_sana_scheduler_state + n_steps x step_sana_scheduler (scheduler.cpp:89-153,272-318) for
 * any config. sigmas_in [n_steps + 1] replaces the built schedule when not NULL (the step
 * functions accept schedules the builder refuses, e.g. without flow sigmas); timesteps_out
 * [n_steps] and sigmas_out [n_steps + 1] receive the schedule used, samples_out
 * [n_steps, numel] the sample after every step. */
int orc_scheduler_run_config(const orc_sched_config *c, size_t n_steps, const float *sigmas_in,
                             const float *model_outputs, const float *sample, size_t numel,
                             float *timesteps_out, float *sigmas_out, float *samples_out);

int orc_attention_block(const float *x, size_t B, size_t T, size_t C, const float *wq,
                        const float *bq, const float *wk, const float *bk, const float *wv,
                        const float *bv, const float *wo, const float *bo, size_t heads,
                        float *out);
int orc_cross_attention_block(const float *x, size_t B, size_t T, size_t C, const float *ctx,
                              size_t L, const float *bias, const float *wq, const float *bq,
                              const float *wk, const float *bk, const float *wv, const float *bv,
                              const float *wo, const float *bo, size_t heads, float *out);
/* Scheduler pieces with an explicit state: sigmas[n_sigmas] (n_sigmas - 1 steps). */
int orc_scheduler_convert(const float *sigmas, size_t n_sigmas, size_t step_index,
                          const float *model_output, const float *sample, size_t numel,
                          float *out);
int orc_scheduler_update(int order, const float *sigmas, size_t n_sigmas, size_t step_index,
                         const float *m0, const float *m1, const float *sample, size_t numel,
                         float *out);
int orc_scheduler_step(const float *sigmas, size_t n_sigmas, size_t step_index, size_t lower,
                       const float *hist, size_t n_hist, const float *model_output,
                       const float *sample, size_t numel, float *out, float *hist_out,
                       size_t *n_hist_out, size_t *lower_out);

/* Model: tensors in the synthetic checkpoint order and PyTorch layout (see
 * oracle/ref_build/ref_capi.cpp ref_model_create for the list). */
void *orc_model_create(const float *const *tensors, size_t n_blocks, size_t C, size_t Cl,
                       size_t Din, size_t E, size_t self_heads, size_t cross_heads);
void orc_model_destroy(void *m);
/* Overrides the loader defaults of one block (zero q/k/v bias, identity norms); any
 * pointer may be NULL to keep the default. Vectors of length C. */
int orc_model_set_cross_qk_norm(void *m, size_t block, int enable, const float *q_weight,
                                const float *k_weight, float eps);
int orc_model_set_block_extras(void *m, size_t block, const float *q_bias, const float *k_bias,
                               const float *v_bias, const float *attn_gamma,
                               const float *attn_beta, const float *mlp_gamma,
                               const float *mlp_beta);
int orc_block_forward(void *m, size_t block, const float *x, size_t S, size_t T, const float *ctx,
                      size_t L, const float *tmod, const float *bias, float *after_self,
                      float *after_cross, float *after_ff);
int orc_run_model_blocks(void *m, const float *x, size_t S, size_t T, const float *ctx, size_t L,
                         const float *tmod, const float *bias, size_t begin, size_t end,
                         float *out);
int orc_model_project_caption(void *m, const float *enc, size_t S, size_t L, size_t Din,
                              float *out);
int orc_time_embed(void *m, const float *tvals, size_t S, float *emb_out, float *tmod_out);
int orc_forward_nocfg(void *m, const float *latents, size_t S, size_t H, size_t W, float t,
                      const float *ctx, size_t L, const float *bias, float *noise_pred);
int orc_denoise(void *m, const float *latents, size_t B, size_t H, size_t W, const float *enc,
                size_t L, size_t Din, const float *bias, float guidance, size_t num_steps,
                size_t run_steps, float *out, size_t *step_index_out);

/* Text-encoder output contract (gemma_encoder.cpp). */
int orc_select_rows_first_and_last(const float *in, size_t rows, size_t cols, size_t keep, float *out);
int orc_prompt_pair_assemble(const float *negative, size_t negative_rows, size_t negative_real,
                             const float *positive, size_t positive_rows, size_t positive_real,
                             size_t hidden, size_t max_sequence_length, float *embeddings, float *bias);

/* VAE decoder (vae.h, vae.cpp, vae_ops.cpp): the DC-AE decoder the reference runs after the
 * denoiser. Up block i has `channels` output channels, an optional nearest-2x upsample conv
 * (from the channels of block i+1; the innermost block has none), then `layers` ResBlocks
 * or attention + GLUMBConv layers. Tensor table order (PyTorch layouts):
 *   conv_in.w [C_{n-1}, latent, 3, 3], conv_in.b, norm_out.w [C_0], norm_out.b,
 *   conv_out.w [out, C_0, 3, 3], conv_out.b; then per block i = 0..n-1:
 *   [upsample conv.w [C_i, C_{i+1}, 3, 3], conv.b] if has_upsample;
 *   per ResBlock: conv1.w, conv1.b, conv2.w, norm.w, norm.b;
 *   per attention layer: to_q [C, C], to_k, to_v, proj_in [3C, 1, k, k], proj_out
 *   [3C, head_dim, 1, 1], to_out [C, 2C], norm_out.w, norm_out.b, conv_inverted.w [8C, C, 1, 1],
 *   conv_inverted.b, conv_depth.w [8C, 1, 3, 3], conv_depth.b, conv_point.w [C, 4C, 1, 1],
 *   norm.w, norm.b. */
typedef struct orc_vae_block {
    int channels, has_upsample, is_res_block, layers;
} orc_vae_block;
typedef struct orc_vae_dims {
    int latent_channels, out_channels, n_blocks, head_dim, ms_kernel;
    float scaling_factor;
    orc_vae_block blocks[8];
} orc_vae_dims;
size_t orc_vae_tensor_count(const orc_vae_dims *d);
/* run_vae_decode (vae.cpp:243-325): latents [B, latent, h, w] -> out [B, out, h*2^u, w*2^u]
 * with u the number of upsampling blocks. */
int orc_vae_decode(const orc_vae_dims *d, const float *const *tensors, const float *latents, size_t B,
                   size_t h, size_t w, float *out);

#ifdef __cplusplus
}
#endif
#endif
