// Test infrastructure only (oracle side): a C wrapper over the reference's own,
// unmodified CPU implementation so that Python tests, the golden-fixture generator and
// bench.py's CPU arm can call it through ctypes. Compiled together with the reference
// sources where they lie (oracle/Makefile); nothing here is part of the product.
//
// Every function copies raw fp32 arrays into the reference's `Tensor`, calls the
// reference function named in its comment, and copies the result out. Exceptions are
// caught and turned into a status (1 = std::invalid_argument, 2 = other) with the
// message kept for ref_last_error().
#include "common_ops.h"
#include "scheduler.h"
#include "tensor.h"
#include "torch_rng.h"
#include "transformer.h"
#include "transformer_ops.h"
#include "vae.h"
#include "vae_ops.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

thread_local std::string g_last_error;

Tensor from_ptr(const float * p, std::vector<size_t> shape) {
    Tensor t(std::move(shape));
    std::memcpy(t.data().data(), p, t.numel() * sizeof(float));
    return t;
}

void to_ptr(const Tensor & t, float * p) {
    std::memcpy(p, t.data().data(), t.numel() * sizeof(float));
}

template <class F>
int guarded(F && f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument & e) {
        g_last_error = e.what();
        return 1;
    } catch (const std::exception & e) {
        g_last_error = e.what();
        return 2;
    }
}

// PyTorch [out, in] -> reference [in, out], as load_linear_weight_tensor does
// (weights_io.cpp:367-377).
Tensor linear_from_torch(const float * p, size_t out_f, size_t in_f) {
    return from_ptr(p, {out_f, in_f}).transpose_2d();
}

struct RefModel {
    SanaDenoiserWeights w;
};

}  // namespace

extern "C" {

const char * ref_last_error() { return g_last_error.c_str(); }

// torch_rng.cpp:35 randn_torch_cpu
int ref_randn(float * out, size_t n, uint64_t seed) {
    return guarded([&] { to_ptr(randn_torch_cpu({n}, seed), out); });
}

// common_ops.cpp:177 linear_3d_lastdim (weight in the reference's [in, out] layout)
int ref_linear_3d(const float * x, size_t B, size_t T, size_t K, const float * w, const float * bias,
                  size_t N, float * out) {
    return guarded([&] {
        Tensor xt = from_ptr(x, {B, T, K});
        Tensor wt = from_ptr(w, {K, N});
        Tensor bt = bias ? from_ptr(bias, {N}) : Tensor({N});
        to_ptr(linear_3d_lastdim(xt, wt, bias ? &bt : nullptr), out);
    });
}

// tensor.cpp:188 layer_norm_3d_lastdim
int ref_layer_norm(const float * x, size_t B, size_t T, size_t C, float eps, const float * gamma,
                   const float * beta, float * out) {
    return guarded([&] {
        Tensor xt = from_ptr(x, {B, T, C});
        Tensor g = gamma ? from_ptr(gamma, {C}) : Tensor({C});
        Tensor b = beta ? from_ptr(beta, {C}) : Tensor({C});
        to_ptr(xt.layer_norm_3d_lastdim(eps, gamma ? &g : nullptr, beta ? &b : nullptr), out);
    });
}

// tensor.cpp:276 rms_norm_3d_lastdim
int ref_rms_norm(const float * x, size_t B, size_t T, size_t C, float eps, const float * weight,
                 float * out) {
    return guarded([&] {
        Tensor xt = from_ptr(x, {B, T, C});
        Tensor g = weight ? from_ptr(weight, {C}) : Tensor({C});
        to_ptr(xt.rms_norm_3d_lastdim(eps, weight ? &g : nullptr), out);
    });
}

// tensor.cpp:323 modulate_3d_lastdim; shift/scale are [B, 1, C]
int ref_modulate(const float * x, size_t B, size_t T, size_t C, const float * shift,
                 const float * scale, float * out) {
    return guarded([&] {
        Tensor xt = from_ptr(x, {B, T, C});
        to_ptr(xt.modulate_3d_lastdim(from_ptr(shift, {B, 1, C}), from_ptr(scale, {B, 1, C})), out);
    });
}

// transformer_ops.cpp:402 linear_attention_4d; q [B,H,Tq,D], k/v [B,H,Tk,D]
int ref_linear_attention(const float * q, const float * k, const float * v, size_t B, size_t H,
                         size_t Tq, size_t Tk, size_t D, float * out) {
    return guarded([&] {
        to_ptr(linear_attention_4d(from_ptr(q, {B, H, Tq, D}), from_ptr(k, {B, H, Tk, D}),
                                   from_ptr(v, {B, H, Tk, D})), out);
    });
}

// transformer_ops.cpp:348 attention_4d; bias [B, 1, Tk] or null
int ref_attention(const float * q, const float * k, const float * v, size_t B, size_t H, size_t Tq,
                  size_t Tk, size_t D, const float * bias, float * out) {
    return guarded([&] {
        Tensor bt = bias ? from_ptr(bias, {B, 1, Tk}) : Tensor({1});
        to_ptr(attention_4d(from_ptr(q, {B, H, Tq, D}), from_ptr(k, {B, H, Tk, D}),
                            from_ptr(v, {B, H, Tk, D}), bias ? &bt : nullptr), out);
    });
}

// common_ops.cpp:322 conv2d_1x1; x NCHW, w [Cout, Cin, 1, 1]
int ref_conv1x1(const float * x, size_t B, size_t Cin, size_t Hh, size_t Ww, const float * w,
                const float * bias, size_t Cout, float * out) {
    return guarded([&] {
        Tensor bt = bias ? from_ptr(bias, {Cout}) : Tensor({Cout});
        to_ptr(conv2d_1x1(from_ptr(x, {B, Cin, Hh, Ww}), from_ptr(w, {Cout, Cin, 1, 1}),
                          bias ? &bt : nullptr), out);
    });
}

// common_ops.cpp:510 depthwise_conv2d_3x3; w [C, 1, 3, 3]
int ref_depthwise3x3(const float * x, size_t B, size_t C, size_t Hh, size_t Ww, const float * w,
                     const float * bias, float * out) {
    return guarded([&] {
        Tensor bt = bias ? from_ptr(bias, {C}) : Tensor({C});
        to_ptr(depthwise_conv2d_3x3(from_ptr(x, {B, C, Hh, Ww}), from_ptr(w, {C, 1, 3, 3}),
                                    bias ? &bt : nullptr), out);
    });
}

// common_ops.cpp:733 glumb_conv; x NCHW [B, Cin, H, W]
int ref_glumb_conv(const float * x, size_t B, size_t Cin, size_t Hh, size_t Ww, const float * w_inv,
                   const float * b_inv, size_t E, const float * w_dw, const float * b_dw,
                   const float * w_pt, size_t Cout, float * out) {
    return guarded([&] {
        Tensor bi = from_ptr(b_inv, {E});
        Tensor bd = from_ptr(b_dw, {E});
        to_ptr(glumb_conv(from_ptr(x, {B, Cin, Hh, Ww}), from_ptr(w_inv, {E, Cin, 1, 1}), &bi,
                          from_ptr(w_dw, {E, 1, 3, 3}), &bd, from_ptr(w_pt, {Cout, E / 2, 1, 1})),
               out);
    });
}

// transformer_ops.cpp:64 project_caption_context (weights in the reference's [in, out] layout)
int ref_project_caption(const float * enc, size_t B, size_t L, size_t Din, const float * w1,
                        const float * b1, size_t C, const float * w2, const float * b2,
                        const float * norm_w, float * out) {
    return guarded([&] {
        Tensor b1t = from_ptr(b1, {C});
        Tensor b2t = from_ptr(b2, {C});
        to_ptr(project_caption_context(from_ptr(enc, {B, L, Din}), from_ptr(w1, {Din, C}), &b1t,
                                       from_ptr(w2, {C, C}), &b2t, from_ptr(norm_w, {C})),
               out);
    });
}

// Builds the reference's weight struct from the synthetic tensor list, in PyTorch
// checkpoint layout, the way load_block_weights / load_denoiser_weights do
// (transformer.cpp:200-399, 453-488): linear weights transposed to [in, out], q/k/v
// biases zero, attention/MLP norms identity.
//   model tensors (16): caption l1 w [C,Din], b; l2 w [C,C], b; patch w [C,Cl,1,1], b;
//     t_emb l1 w [C,256], b; l2 w [C,C], b; t_proj w [6C,C], b; caption_norm [C];
//     final table [2,C]; proj_out w [Cl,C], b [Cl]
//   per block (19): table [6,C]; q,k,v,out w [C,C]; out b; cross q w,b; k w,b; v w,b;
//     out w,b; ff inverted w [E,C,1,1], b [E]; depth w [E,1,3,3], b [E]; point w [C,E/2,1,1]
void * ref_model_create(const float * const * t, size_t n_blocks, size_t C, size_t Cl, size_t Din,
                        size_t E, size_t self_heads, size_t cross_heads) {
    RefModel * m = nullptr;
    int rc = guarded([&] {
        Tensor zero({C});
        zero.fill(0.0f);
        Tensor ones({C});
        ones.fill(1.0f);
        std::vector<SanaBlockWeights> blocks;
        for (size_t i = 0; i < n_blocks; ++i) {
            const float * const * b = t + 16 + 19 * i;
            blocks.push_back(SanaBlockWeights{
                from_ptr(b[0], {6, C}),
                ones, zero,
                linear_from_torch(b[1], C, C), zero,
                linear_from_torch(b[2], C, C), zero,
                linear_from_torch(b[3], C, C), zero,
                linear_from_torch(b[4], C, C), from_ptr(b[5], {C}),
                linear_from_torch(b[6], C, C), from_ptr(b[7], {C}),
                linear_from_torch(b[8], C, C), from_ptr(b[9], {C}),
                linear_from_torch(b[10], C, C), from_ptr(b[11], {C}),
                linear_from_torch(b[12], C, C), from_ptr(b[13], {C}),
                ones, zero,
                from_ptr(b[14], {E, C, 1, 1}), from_ptr(b[15], {E}),
                from_ptr(b[16], {E, 1, 3, 3}), from_ptr(b[17], {E}),
                from_ptr(b[18], {C, E / 2, 1, 1}),
                self_heads, cross_heads,
            });
        }
        SanaDenoiserWeights w{
            SanaCaptionWeights{linear_from_torch(t[0], C, Din), from_ptr(t[1], {C}),
                               linear_from_torch(t[2], C, C), from_ptr(t[3], {C})},
            blocks,
            from_ptr(t[4], {C, Cl, 1, 1}), from_ptr(t[5], {C}),
            linear_from_torch(t[6], C, 256), from_ptr(t[7], {C}),
            linear_from_torch(t[8], C, C), from_ptr(t[9], {C}),
            linear_from_torch(t[10], 6 * C, C), from_ptr(t[11], {6 * C}),
            from_ptr(t[12], {C}),
            from_ptr(t[13], {2, C}),
            linear_from_torch(t[14], Cl, C), from_ptr(t[15], {Cl}),
        };
        validate_denoiser_weights(w);
        m = new RefModel{std::move(w)};
    });
    return rc == 0 ? m : nullptr;
}

void ref_model_destroy(void * m) { delete static_cast<RefModel *>(m); }

// transformer.cpp:726 block_forward; x [S,T,C], ctx [S,L,C], tmod [S,6C], bias [S,1,L] or null
int ref_block_forward(void * mp, size_t block, const float * x, size_t S, size_t T,
                      const float * ctx, size_t L, const float * tmod, const float * bias,
                      float * after_self, float * after_cross, float * after_ff) {
    return guarded([&] {
        const auto & w = static_cast<RefModel *>(mp)->w;
        const size_t C = w.blocks.at(block).scale_shift_table.dim_size(1);
        Tensor bt = bias ? from_ptr(bias, {S, 1, L}) : Tensor({1});
        SanaBlockStageOutputs o = block_forward(from_ptr(x, {S, T, C}), from_ptr(ctx, {S, L, C}),
                                                from_ptr(tmod, {S, 6 * C}), w.blocks.at(block),
                                                bias ? &bt : nullptr);
        if (after_self) to_ptr(o.after_self, after_self);
        if (after_cross) to_ptr(o.after_cross, after_cross);
        if (after_ff) to_ptr(o.after_ff, after_ff);
    });
}

// transformer.cpp:544 run_model_blocks
int ref_run_model_blocks(void * mp, const float * x, size_t S, size_t T, const float * ctx, size_t L,
                         const float * tmod, const float * bias, size_t begin, size_t end,
                         float * out) {
    return guarded([&] {
        const auto & w = static_cast<RefModel *>(mp)->w;
        const size_t C = w.blocks.at(0).scale_shift_table.dim_size(1);
        Tensor bt = bias ? from_ptr(bias, {S, 1, L}) : Tensor({1});
        to_ptr(run_model_blocks(from_ptr(x, {S, T, C}), from_ptr(ctx, {S, L, C}),
                                from_ptr(tmod, {S, 6 * C}), w, begin, end, bias ? &bt : nullptr),
               out);
    });
}

// Caption projection with the model's weights (transformer.cpp:701-708)
int ref_model_project_caption(void * mp, const float * enc, size_t S, size_t L, size_t Din,
                              float * out) {
    return guarded([&] {
        const auto & w = static_cast<RefModel *>(mp)->w;
        to_ptr(project_caption_context(from_ptr(enc, {S, L, Din}), w.caption.linear_1_weight,
                                       &w.caption.linear_1_bias, w.caption.linear_2_weight,
                                       &w.caption.linear_2_bias, w.caption_norm_weight),
               out);
    });
}

// The timestep path of run_full_denoising_step_with_cfg (transformer.cpp:638-656), whose
// sinusoid helper timestep_embedding_2d (transformer.cpp:77-122) sits in an anonymous
// namespace and is restated here in the same arithmetic order.
int ref_time_embed(void * mp, const float * tvals, size_t S, float * emb_out, float * tmod_out) {
    return guarded([&] {
        const auto & w = static_cast<RefModel *>(mp)->w;
        const size_t dim = 256, half = 128;
        Tensor proj({S, dim});
        std::vector<float> freq(half);
        const float log_scale = -std::log(10000.0f) / static_cast<float>(half);
        for (size_t i = 0; i < half; ++i) freq[i] = std::exp(static_cast<float>(i) * log_scale);
        for (size_t b = 0; b < S; ++b) {
            for (size_t i = 0; i < half; ++i) {
                const float v = tvals[b] * freq[i];
                proj.data()[b * dim + i] = std::cos(v);
                proj.data()[b * dim + half + i] = std::sin(v);
            }
        }
        Tensor emb = linear_2d(proj, w.time_embed_linear_1_weight, &w.time_embed_linear_1_bias);
        emb.silu_inplace();
        emb = linear_2d(emb, w.time_embed_linear_2_weight, &w.time_embed_linear_2_bias);
        Tensor hid = emb;
        hid.silu_inplace();
        Tensor tmod = linear_2d(hid, w.time_projection_weight, &w.time_projection_bias);
        if (emb_out) to_ptr(emb, emb_out);
        if (tmod_out) to_ptr(tmod, tmod_out);
    });
}

// One denoiser forward without CFG or scheduler (the config-0 case): the body of
// run_full_denoising_step_with_cfg between the batch repeat and the guidance
// (transformer.cpp:631-681) at timestep t for S independent sequences.
//   latents [S, Cl, H, W], ctx [S, L, C] (already projected), bias [S, 1, L] or null
//   noise_pred out [S, Cl, H, W]
int ref_forward_nocfg(void * mp, const float * latents, size_t S, size_t Hh, size_t Ww, float t,
                      const float * ctx, size_t L, const float * bias, float * noise_pred) {
    return guarded([&] {
        const auto & w = static_cast<RefModel *>(mp)->w;
        const size_t C = w.blocks.at(0).scale_shift_table.dim_size(1);
        const size_t Cl = w.patch_embed_weight.dim_size(1);
        Tensor lat = from_ptr(latents, {S, Cl, Hh, Ww});
        Tensor tokens = conv2d_1x1(lat, w.patch_embed_weight, &w.patch_embed_bias).grid_to_tokens_3d();
        std::vector<float> tv(S, t);
        std::vector<float> emb(S * C), tmod(S * 6 * C);
        if (ref_time_embed(mp, tv.data(), S, emb.data(), tmod.data()) != 0) {
            throw std::runtime_error(g_last_error);
        }
        Tensor bt = bias ? from_ptr(bias, {S, 1, L}) : Tensor({1});
        Tensor hidden = run_model_blocks(tokens, from_ptr(ctx, {S, L, C}),
                                         from_ptr(tmod.data(), {S, 6 * C}), w, 0, w.blocks.size(),
                                         bias ? &bt : nullptr);
        Tensor normalized = hidden.layer_norm_3d_lastdim(1e-6f);
        // compute_final_modulation (transformer.cpp:126-163): shift = emb + table[0],
        // scale = emb + table[1]
        Tensor shift({S, 1, C}), scale({S, 1, C});
        const float * table = w.final_scale_shift_table.data().data();
        for (size_t b = 0; b < S; ++b) {
            for (size_t h = 0; h < C; ++h) {
                shift.data()[b * C + h] = emb[b * C + h] + table[h];
                scale.data()[b * C + h] = emb[b * C + h] + table[C + h];
            }
        }
        Tensor projected = linear_3d_lastdim(normalized.modulate_3d_lastdim(shift, scale),
                                             w.proj_out_weight, &w.proj_out_bias);
        to_ptr(projected.tokens_to_grid_4d(Hh, Ww), noise_pred);
    });
}

// transformer.cpp:692 run_full_denoising_loop_with_cfg, stopping after `run_steps` of a
// `num_steps` schedule (run_steps == num_steps is the whole loop).
//   latents [B, Cl, H, W]; enc [2B, L, Din] (uncond first); bias [2B, 1, L] or null
//   out [B, Cl, H, W]; step_index_out receives the scheduler's final step_index
int ref_denoise(void * mp, const float * latents, size_t B, size_t Hh, size_t Ww, const float * enc,
                size_t L, size_t Din, const float * bias, float guidance, size_t num_steps,
                size_t run_steps, float * out, size_t * step_index_out) {
    return guarded([&] {
        const auto & w = static_cast<RefModel *>(mp)->w;
        const size_t Cl = w.patch_embed_weight.dim_size(1);
        SanaSchedulerConfig cfg = make_sana_scheduler_config();
        SanaSchedulerState state = init_sana_scheduler_state(num_steps, cfg);
        Tensor bt = bias ? from_ptr(bias, {2 * B, 1, L}) : Tensor({1});
        Tensor lat = from_ptr(latents, {B, Cl, Hh, Ww});
        if (run_steps >= num_steps) {
            lat = run_full_denoising_loop_with_cfg(lat, from_ptr(enc, {2 * B, L, Din}), guidance,
                                                   state, cfg, w, bias ? &bt : nullptr);
        } else {
            Tensor ctx = project_caption_context(
                from_ptr(enc, {2 * B, L, Din}), w.caption.linear_1_weight, &w.caption.linear_1_bias,
                w.caption.linear_2_weight, &w.caption.linear_2_bias, w.caption_norm_weight);
            for (size_t s = 0; s < run_steps; ++s) {
                lat = run_full_denoising_step_with_cfg(lat, ctx, guidance, state, cfg, w,
                                                       bias ? &bt : nullptr);
            }
        }
        to_ptr(lat, out);
        if (step_index_out) *step_index_out = state.step_index;
    });
}

// scheduler.cpp:89 build_sana_scheduler_timesteps with the default config except flow_shift
int ref_scheduler_schedule(size_t n, float flow_shift, float * timesteps, float * sigmas) {
    return guarded([&] {
        SanaSchedulerConfig cfg = make_sana_scheduler_config();
        cfg.flow_shift = flow_shift;
        SanaSchedulerTimesteps s = build_sana_scheduler_timesteps(n, cfg);
        std::copy(s.timesteps.begin(), s.timesteps.end(), timesteps);
        std::copy(s.sigmas.begin(), s.sigmas.end(), sigmas);
    });
}

// scheduler.cpp:272 step_sana_scheduler, run over a whole sequence of model outputs:
// model_outputs [n_steps, numel]; sample [numel] is updated through all steps and the
// sample after every step is written to samples_out [n_steps, numel].
int ref_scheduler_run(size_t n_steps, float flow_shift, const float * model_outputs,
                      const float * sample, size_t numel, float * samples_out) {
    return guarded([&] {
        SanaSchedulerConfig cfg = make_sana_scheduler_config();
        cfg.flow_shift = flow_shift;
        SanaSchedulerState state = init_sana_scheduler_state(n_steps, cfg);
        Tensor x = from_ptr(sample, {numel});
        for (size_t s = 0; s < n_steps; ++s) {
            x = step_sana_scheduler(from_ptr(model_outputs + s * numel, {numel}), x, state, cfg);
            to_ptr(x, samples_out + s * numel);
        }
    });
}

// The C ABI's scheduler config as plain fields (same layout as orc_sched_config).
struct RefSchedConfig {
    int num_train_timesteps;
    float flow_shift;
    int use_flow_sigmas;
    int solver_order;
    int lower_order_final;
    int final_sigmas_zero;
    int solver_heun;
};

// init_sana_scheduler_state + step_sana_scheduler n_steps times with any config; sigmas_in
// [n_steps + 1] (or null) replaces the built schedule, for configs the builder refuses.
int ref_scheduler_run_config(const RefSchedConfig * c, size_t n_steps, const float * sigmas_in,
                             const float * model_outputs, const float * sample, size_t numel,
                             float * timesteps_out, float * sigmas_out, float * samples_out) {
    return guarded([&] {
        SanaSchedulerConfig cfg = make_sana_scheduler_config();
        cfg.num_train_timesteps = static_cast<size_t>(c->num_train_timesteps);
        cfg.flow_shift = c->flow_shift;
        cfg.use_flow_sigmas = c->use_flow_sigmas != 0;
        cfg.solver_order = static_cast<size_t>(c->solver_order);
        cfg.lower_order_final = c->lower_order_final != 0;
        cfg.final_sigmas_type = c->final_sigmas_zero ? "zero" : "sigma_min";
        cfg.solver_type = c->solver_heun ? "heun" : "midpoint";
        SanaSchedulerState state;
        if (sigmas_in) {
            state.schedule.timesteps.assign(n_steps, 0.0f);
            state.schedule.sigmas.assign(sigmas_in, sigmas_in + n_steps + 1);
        } else {
            state = init_sana_scheduler_state(n_steps, cfg);
        }
        std::copy(state.schedule.timesteps.begin(), state.schedule.timesteps.end(), timesteps_out);
        std::copy(state.schedule.sigmas.begin(), state.schedule.sigmas.end(), sigmas_out);
        Tensor x = from_ptr(sample, {numel});
        for (size_t s = 0; s < n_steps; ++s) {
            x = step_sana_scheduler(from_ptr(model_outputs + s * numel, {numel}), x, state, cfg);
            to_ptr(x, samples_out + s * numel);
        }
    });
}

// transformer.cpp:570 apply_classifier_free_guidance; noise [2B, Cl, H, W]
int ref_cfg(const float * noise, size_t B, size_t Cl, size_t Hh, size_t Ww, float g, float * out) {
    return guarded([&] {
        to_ptr(apply_classifier_free_guidance(from_ptr(noise, {2 * B, Cl, Hh, Ww}), g), out);
    });
}


// transformer_ops.cpp:545 attention_block_3d; weights [in, out]; biases may be null
int ref_attention_block(const float * x, size_t B, size_t T, size_t C, const float * wq,
                        const float * bq, const float * wk, const float * bk, const float * wv,
                        const float * bv, const float * wo, const float * bo, size_t heads,
                        float * out) {
    return guarded([&] {
        Tensor z({C});
        z.fill(0.0f);
        Tensor tbq = bq ? from_ptr(bq, {C}) : z, tbk = bk ? from_ptr(bk, {C}) : z;
        Tensor tbv = bv ? from_ptr(bv, {C}) : z, tbo = bo ? from_ptr(bo, {C}) : z;
        to_ptr(attention_block_3d(from_ptr(x, {B, T, C}), from_ptr(wq, {C, C}), bq ? &tbq : nullptr,
                                  from_ptr(wk, {C, C}), bk ? &tbk : nullptr, from_ptr(wv, {C, C}),
                                  bv ? &tbv : nullptr, from_ptr(wo, {C, C}), bo ? &tbo : nullptr,
                                  heads),
               out);
    });
}

// transformer_ops.cpp:572 cross_attention_block_3d; ctx [B, L, C]; bias [B, 1, L] or null
int ref_cross_attention_block(const float * x, size_t B, size_t T, size_t C, const float * ctx,
                              size_t L, const float * bias, const float * wq, const float * bq,
                              const float * wk, const float * bk, const float * wv,
                              const float * bv, const float * wo, const float * bo, size_t heads,
                              float * out) {
    return guarded([&] {
        Tensor z({C});
        z.fill(0.0f);
        Tensor tbq = bq ? from_ptr(bq, {C}) : z, tbk = bk ? from_ptr(bk, {C}) : z;
        Tensor tbv = bv ? from_ptr(bv, {C}) : z, tbo = bo ? from_ptr(bo, {C}) : z;
        Tensor bt = bias ? from_ptr(bias, {B, 1, L}) : Tensor({1});
        to_ptr(cross_attention_block_3d(from_ptr(x, {B, T, C}), from_ptr(ctx, {B, L, C}),
                                        bias ? &bt : nullptr, from_ptr(wq, {C, C}),
                                        bq ? &tbq : nullptr, from_ptr(wk, {C, C}),
                                        bk ? &tbk : nullptr, from_ptr(wv, {C, C}),
                                        bv ? &tbv : nullptr, from_ptr(wo, {C, C}),
                                        bo ? &tbo : nullptr, heads),
               out);
    });
}

// Scheduler pieces with an explicit state: sigmas has n_sigmas entries (the schedule's
// timesteps count is n_sigmas - 1, their values are unused by the arithmetic).
static SanaSchedulerState make_state(const float * sigmas, size_t n_sigmas, size_t step_index,
                                     size_t lower) {
    SanaSchedulerState st;
    st.schedule.sigmas.assign(sigmas, sigmas + n_sigmas);
    st.schedule.timesteps.assign(n_sigmas - 1, 0.0f);
    st.step_index = step_index;
    st.lower_order_step_count = lower;
    return st;
}

// scheduler.cpp:155 convert_sana_scheduler_model_output
int ref_scheduler_convert(const float * sigmas, size_t n_sigmas, size_t step_index,
                          const float * model_output, const float * sample, size_t numel,
                          float * out) {
    return guarded([&] {
        SanaSchedulerState st = make_state(sigmas, n_sigmas, step_index, 0);
        to_ptr(convert_sana_scheduler_model_output(from_ptr(model_output, {numel}),
                                                   from_ptr(sample, {numel}), st,
                                                   make_sana_scheduler_config()),
               out);
    });
}

// scheduler.cpp:175 first-order update (order 1, converted output m0) or scheduler.cpp:207
// second-order update (order 2, history [m1, m0] with m0 the newest)
int ref_scheduler_update(int order, const float * sigmas, size_t n_sigmas, size_t step_index,
                         const float * m0, const float * m1, const float * sample, size_t numel,
                         float * out) {
    return guarded([&] {
        SanaSchedulerState st = make_state(sigmas, n_sigmas, step_index, 1);
        SanaSchedulerConfig cfg = make_sana_scheduler_config();
        if (order == 1) {
            to_ptr(sana_scheduler_first_order_update(from_ptr(m0, {numel}), from_ptr(sample, {numel}),
                                                     st, cfg),
                   out);
        } else {
            st.previous_model_outputs.push_back(from_ptr(m1, {numel}));
            st.previous_model_outputs.push_back(from_ptr(m0, {numel}));
            to_ptr(sana_scheduler_second_order_update(from_ptr(sample, {numel}), st, cfg), out);
        }
    });
}

// scheduler.cpp:272 step_sana_scheduler with an explicit state. hist holds n_hist (<= 2)
// converted outputs, oldest first; the updated history (oldest first) is written to
// hist_out with its length in *n_hist_out, the new lower-order count in *lower_out.
int ref_scheduler_step(const float * sigmas, size_t n_sigmas, size_t step_index, size_t lower,
                       const float * hist, size_t n_hist, const float * model_output,
                       const float * sample, size_t numel, float * out, float * hist_out,
                       size_t * n_hist_out, size_t * lower_out) {
    return guarded([&] {
        SanaSchedulerState st = make_state(sigmas, n_sigmas, step_index, lower);
        for (size_t i = 0; i < n_hist; ++i) {
            st.previous_model_outputs.push_back(from_ptr(hist + i * numel, {numel}));
        }
        to_ptr(step_sana_scheduler(from_ptr(model_output, {numel}), from_ptr(sample, {numel}), st,
                                   make_sana_scheduler_config()),
               out);
        for (size_t i = 0; i < st.previous_model_outputs.size(); ++i) {
            to_ptr(st.previous_model_outputs[i], hist_out + i * numel);
        }
        *n_hist_out = st.previous_model_outputs.size();
        *lower_out = st.lower_order_step_count;
    });
}

// vae.cpp:243 run_vae_decode on SanaVaeWeights built from a pointer table: the same
// dims struct and tensor order as the oracle's orc_vae_decode (PyTorch layouts; the
// attention projections go through linear_weight_to_conv1x1 as load_vae_attention_weights
// does, vae.cpp:26-41).
struct ref_vae_block {
    int channels, has_upsample, is_res_block, layers;
};
struct ref_vae_dims {
    int latent_channels, out_channels, n_blocks, head_dim, ms_kernel;
    float scaling_factor;
    ref_vae_block blocks[8];
};

int ref_vae_decode(const ref_vae_dims * d, const float * const * t, const float * latents, size_t B, size_t h,
                   size_t w, float * out) {
    return guarded([&] {
        const size_t n = static_cast<size_t>(d->n_blocks);
        auto C = [&](size_t i) { return static_cast<size_t>(d->blocks[i].channels); };
        const size_t Cl = static_cast<size_t>(d->latent_channels), Co = static_cast<size_t>(d->out_channels);
        const size_t k = static_cast<size_t>(d->ms_kernel), hd = static_cast<size_t>(d->head_dim);
        size_t j = 0;
        SanaVaeDecoderWeights dec{
            from_ptr(t[0], {C(n - 1), Cl, 3, 3}), from_ptr(t[1], {C(n - 1)}),
            from_ptr(t[2], {C(0)}), from_ptr(t[3], {C(0)}),
            from_ptr(t[4], {Co, C(0), 3, 3}), from_ptr(t[5], {Co}), {}};
        j = 6;
        for (size_t i = 0; i < n; ++i) {
            const ref_vae_block & b = d->blocks[i];
            const size_t c = C(i);
            SanaVaeUpBlockWeights ub;
            if (b.has_upsample) {
                ub.upsample_conv_weight = from_ptr(t[j], {c, C(i + 1), 3, 3});
                ub.upsample_conv_bias = from_ptr(t[j + 1], {c});
                j += 2;
            }
            ub.is_res_block = b.is_res_block != 0;
            for (int l = 0; l < b.layers; ++l) {
                if (b.is_res_block) {
                    ub.res_blocks.push_back(SanaVaeResBlockWeights{
                        from_ptr(t[j], {c, c, 3, 3}), from_ptr(t[j + 1], {c}), from_ptr(t[j + 2], {c, c, 3, 3}),
                        from_ptr(t[j + 3], {c}), from_ptr(t[j + 4], {c})});
                    j += 5;
                } else {
                    SanaVaeAttentionWeights a{
                        linear_weight_to_conv1x1(from_ptr(t[j], {c, c})),
                        linear_weight_to_conv1x1(from_ptr(t[j + 1], {c, c})),
                        linear_weight_to_conv1x1(from_ptr(t[j + 2], {c, c})),
                        from_ptr(t[j + 3], {3 * c, 1, k, k}),
                        from_ptr(t[j + 4], {3 * c, hd, 1, 1}),
                        linear_weight_to_conv1x1(from_ptr(t[j + 5], {c, 2 * c})),
                        from_ptr(t[j + 6], {c}), from_ptr(t[j + 7], {c})};
                    SanaVaeGlumbConvWeights g{
                        from_ptr(t[j + 8], {8 * c, c, 1, 1}), from_ptr(t[j + 9], {8 * c}),
                        from_ptr(t[j + 10], {8 * c, 1, 3, 3}), from_ptr(t[j + 11], {8 * c}),
                        from_ptr(t[j + 12], {c, 4 * c, 1, 1}), from_ptr(t[j + 13], {c}), from_ptr(t[j + 14], {c})};
                    ub.attn_glumb_layers.push_back(SanaVaeAttnGlumbLayerWeights{std::move(a), std::move(g)});
                    j += 15;
                }
            }
            dec.up_blocks.push_back(std::move(ub));
        }
        SanaVaeWeights vw{std::move(dec), d->scaling_factor, 32};
        to_ptr(run_vae_decode(from_ptr(latents, {B, Cl, h, w}), vw), out);
    });
}

}  // extern "C"
