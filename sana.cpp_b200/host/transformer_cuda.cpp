// transformer.h (cconthekeyboard/sana.cpp src/transformer.h:114-155) over the C ABI: the
// denoiser step, loop and blocks run on the GPU with the weights uploaded once per weight
// struct (shim.cpp). Argument checks and their exception types follow the reference
// (transformer.cpp:496-778).
#include "transformer.h"

#include <algorithm>
#include <cmath>
#include <stdexcept>

#include "shim.h"

using sana_shim::as_int;
using sana_shim::check;
using sana_shim::handle;
using sana_shim::opt;
using sana_shim::ptr;
using sana_shim::require;

namespace {

// Rows of one [B, C] tensor split into a [B, 1, C] tensor.
Tensor slab(const std::vector<float>& all, size_t B, size_t C, size_t k) {
    Tensor t({B, 1, C});
    for (size_t b = 0; b < B; ++b)
        for (size_t i = 0; i < C; ++i) t.data()[b * C + i] = all[(b * 6 + k) * C + i];
    return t;
}

// True when the state's schedule is the one build_sana_scheduler_timesteps gives `c`.
bool built_schedule(const SanaSchedulerState& s, const sana_scheduler_config& c) {
    const size_t n = s.schedule.timesteps.size();
    if (n == 0 || n > 1024 || s.schedule.sigmas.size() != n + 1) return false;
    std::vector<float> ts(n), sg(n + 1);
    if (sana_scheduler_schedule_config(&c, static_cast<int>(n), ts.data(), sg.data()) != SANA_OK) return false;
    return ts == s.schedule.timesteps && sg == s.schedule.sigmas;
}

}  // namespace

SanaBlockModulation compute_sana_block_modulation(const Tensor& timestep, const Tensor& scale_shift_table) {
    require(timestep.rank() == 2, "timestep must be rank 2");
    require(scale_shift_table.rank() == 2, "scale_shift_table must be rank 2");
    require(scale_shift_table.dim_size(0) == 6, "scale_shift_table must have shape {6, hidden}");
    const size_t B = timestep.dim_size(0), C = scale_shift_table.dim_size(1);
    require(timestep.dim_size(1) == 6 * C, "timestep width must equal 6 * hidden");
    std::vector<float> all(B * 6 * C);
    if (B && C)
        check(sana_op_block_modulation(handle(), ptr(timestep), ptr(scale_shift_table), as_int(B, "batch"),
                                       as_int(C, "hidden"), all.data()));
    return {slab(all, B, C, 0), slab(all, B, C, 1), slab(all, B, C, 2),
            slab(all, B, C, 3), slab(all, B, C, 4), slab(all, B, C, 5)};
}

SanaBlockStageOutputs block_forward(const Tensor& input, const Tensor& context, const Tensor& timestep,
                                    const SanaBlockWeights& weights, const Tensor* encoder_attention_bias) {
    require(input.rank() == 3, "input must be rank 3");
    require(context.rank() == 3, "context must be rank 3");
    require(timestep.rank() == 2, "timestep must be rank 2");
    const size_t S = input.dim_size(0), T = input.dim_size(1), C = input.dim_size(2);
    require(context.dim_size(0) == S && context.dim_size(2) == C, "context must be [batch, tokens, hidden]");
    require(timestep.dim_size(0) == S && timestep.dim_size(1) == 6 * C, "timestep width must equal 6 * hidden");
    const size_t L = context.dim_size(1);
    if (encoder_attention_bias)
        require(encoder_attention_bias->numel() == S * L, "attention bias must be [batch, 1, context tokens]");
    sana_shim::ensure_block(weights);
    SanaBlockStageOutputs out{Tensor(input.shape()), Tensor(input.shape()), Tensor(input.shape())};
    check(sana_cuda_block_forward(handle(), 0, ptr(input), as_int(S, "batch"), as_int(T, "tokens"), ptr(context),
                                  as_int(L, "context tokens"), ptr(timestep), opt(encoder_attention_bias),
                                  out.after_self.data().data(), out.after_cross.data().data(),
                                  out.after_ff.data().data()));
    return out;
}

Tensor run_model_blocks(const Tensor& input, const Tensor& context, const Tensor& timestep,
                        const SanaDenoiserWeights& weights, size_t block_begin, size_t block_end,
                        const Tensor* encoder_attention_bias) {
    if (block_begin > block_end || block_end > weights.blocks.size())
        throw std::invalid_argument("invalid model block range");
    require(input.rank() == 3, "input must be rank 3");
    require(context.rank() == 3, "context must be rank 3");
    require(timestep.rank() == 2, "timestep must be rank 2");
    const size_t S = input.dim_size(0), T = input.dim_size(1), C = input.dim_size(2), L = context.dim_size(1);
    require(context.dim_size(0) == S && context.dim_size(2) == C, "context must be [batch, tokens, hidden]");
    require(timestep.dim_size(0) == S && timestep.dim_size(1) == 6 * C, "timestep width must equal 6 * hidden");
    if (encoder_attention_bias)
        require(encoder_attention_bias->numel() == S * L, "attention bias must be [batch, 1, context tokens]");
    if (block_begin == block_end) return input;
    sana_shim::ensure_weights(weights);
    Tensor out(input.shape());
    check(sana_cuda_run_model_blocks(handle(), ptr(input), as_int(S, "batch"), as_int(T, "tokens"), ptr(context),
                                     as_int(L, "context tokens"), ptr(timestep), opt(encoder_attention_bias),
                                     as_int(block_begin, "block"), as_int(block_end, "block"), out.data().data()));
    return out;
}

Tensor apply_classifier_free_guidance(const Tensor& noise_pred, float guidance_scale) {
    require(noise_pred.rank() == 4, "noise_pred must be rank 4");
    require(noise_pred.dim_size(0) % 2 == 0, "noise_pred batch size must be even for classifier-free guidance");
    const size_t B = noise_pred.dim_size(0) / 2;
    Tensor out({B, noise_pred.dim_size(1), noise_pred.dim_size(2), noise_pred.dim_size(3)});
    if (out.numel() == 0) return out;
    check(sana_op_cfg(handle(), ptr(noise_pred), as_int(B, "batch"), as_int(noise_pred.dim_size(1), "channels"),
                      as_int(noise_pred.dim_size(2), "height"), as_int(noise_pred.dim_size(3), "width"),
                      guidance_scale, out.data().data()));
    return out;
}

Tensor run_full_denoising_step_with_cfg(const Tensor& latents, const Tensor& context, float guidance_scale,
                                        SanaSchedulerState& scheduler_state,
                                        const SanaSchedulerConfig& scheduler_config,
                                        const SanaDenoiserWeights& denoiser_weights,
                                        const Tensor* encoder_attention_bias) {
    if (scheduler_state.step_index >= scheduler_state.schedule.timesteps.size())
        throw std::invalid_argument("scheduler step_index is out of range");
    require(context.rank() == 3, "context must be rank 3");
    require(latents.rank() == 4, "latents must be rank 4");
    require(context.dim_size(0) == latents.dim_size(0) * 2,
            "context batch size must equal 2 * latent batch size for CFG");
    if (encoder_attention_bias)
        require(encoder_attention_bias->dim_size(0) == latents.dim_size(0) * 2,
                "encoder_attention_bias batch size must equal 2 * latent batch size for CFG");
    require(scheduler_state.schedule.sigmas.size() == scheduler_state.schedule.timesteps.size() + 1,
            "scheduler sigmas must have one extra final entry");
    const sana_scheduler_config cc = sana_shim::c_config(scheduler_config);
    sana_shim::ensure_weights(denoiser_weights);
    const size_t B = latents.dim_size(0), numel = latents.numel();
    for (const Tensor& h : scheduler_state.previous_model_outputs)
        require(h.same_shape(latents), "stored model outputs must match sample shape");
    require(scheduler_state.previous_model_outputs.size() <= 2, "at most two stored model outputs are supported");
    std::vector<float> history(2 * numel);
    int n_history = static_cast<int>(scheduler_state.previous_model_outputs.size());
    for (int i = 0; i < n_history; ++i)
        std::copy(scheduler_state.previous_model_outputs[i].data().begin(),
                  scheduler_state.previous_model_outputs[i].data().end(), history.begin() + i * numel);
    Tensor out = latents;
    int step = as_int(scheduler_state.step_index, "step index");
    int lower = as_int(scheduler_state.lower_order_step_count, "lower order count");
    check(sana_cuda_denoise_step_config(
        handle(), &cc, out.data().data(), as_int(B, "batch"), as_int(latents.dim_size(2), "height"),
        as_int(latents.dim_size(3), "width"), ptr(context), as_int(context.dim_size(1), "context tokens"),
        opt(encoder_attention_bias), guidance_scale, scheduler_state.schedule.timesteps[scheduler_state.step_index],
        scheduler_state.schedule.sigmas.data(), as_int(scheduler_state.schedule.sigmas.size(), "sigmas"), &step,
        &lower, history.data(), &n_history));
    scheduler_state.step_index = static_cast<size_t>(step);
    scheduler_state.lower_order_step_count = static_cast<size_t>(lower);
    scheduler_state.previous_model_outputs.clear();
    for (int i = 0; i < n_history; ++i) {
        Tensor h(latents.shape());
        std::copy(history.begin() + i * numel, history.begin() + (i + 1) * numel, h.data().begin());
        scheduler_state.previous_model_outputs.push_back(std::move(h));
    }
    return out;
}

Tensor run_full_denoising_loop_with_cfg(const Tensor& initial_latents, const Tensor& encoder_hidden_states,
                                        float guidance_scale, SanaSchedulerState& scheduler_state,
                                        const SanaSchedulerConfig& scheduler_config,
                                        const SanaDenoiserWeights& denoiser_weights,
                                        const Tensor* encoder_attention_bias) {
    require(initial_latents.rank() == 4, "latents must be rank 4");
    require(encoder_hidden_states.rank() == 3, "encoder_hidden_states must be rank 3");
    require(encoder_hidden_states.dim_size(0) == initial_latents.dim_size(0) * 2,
            "encoder_hidden_states batch size must equal 2 * latent batch size for CFG");
    if (encoder_attention_bias)
        require(encoder_attention_bias->dim_size(0) == initial_latents.dim_size(0) * 2,
                "encoder_attention_bias batch size must equal 2 * latent batch size for CFG");
    const sana_scheduler_config cc = sana_shim::c_config(scheduler_config);
    sana_shim::ensure_weights(denoiser_weights);
    const size_t n = scheduler_state.schedule.timesteps.size();
    const size_t L = encoder_hidden_states.dim_size(1), Din = encoder_hidden_states.dim_size(2);
    if (scheduler_state.step_index == 0 && scheduler_state.previous_model_outputs.empty() &&
        scheduler_state.lower_order_step_count == 0 && built_schedule(scheduler_state, cc)) {
        // A fresh state on the config's own schedule: the whole loop runs on the device (one
        // CUDA graph from the second call with the same shapes).
        Tensor out(initial_latents.shape());
        check(sana_cuda_denoise_loop_config(handle(), &cc, ptr(initial_latents),
                                            as_int(initial_latents.dim_size(0), "batch"),
                                            as_int(initial_latents.dim_size(2), "height"),
                                            as_int(initial_latents.dim_size(3), "width"), ptr(encoder_hidden_states),
                                            as_int(L, "context tokens"), as_int(Din, "caption dim"),
                                            opt(encoder_attention_bias), guidance_scale, as_int(n, "steps"),
                                            out.data().data()));
        scheduler_state.step_index = n;
        scheduler_state.lower_order_step_count = std::min(n, scheduler_config.solver_order);
        return out;
    }
    // Any other state: project the caption once, then step (transformer.cpp:692-724).
    const size_t C = denoiser_weights.blocks[0].scale_shift_table.dim_size(1);
    Tensor context({encoder_hidden_states.dim_size(0), L, C});
    check(sana_cuda_project_caption(handle(), ptr(encoder_hidden_states),
                                    as_int(encoder_hidden_states.dim_size(0), "batch"), as_int(L, "context tokens"),
                                    as_int(Din, "caption dim"), context.data().data()));
    Tensor latents = initial_latents;
    while (scheduler_state.step_index < n)
        latents = run_full_denoising_step_with_cfg(latents, context, guidance_scale, scheduler_state,
                                                   scheduler_config, denoiser_weights, encoder_attention_bias);
    return latents;
}
