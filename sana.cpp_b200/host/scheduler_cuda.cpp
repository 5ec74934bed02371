// scheduler.h (cconthekeyboard/sana.cpp src/scheduler.h:34-65) over the C ABI: the schedule is
// built on the host (as the reference does), the per-element updates run on the device.
// Checks and their std::invalid_argument follow scheduler.cpp:8-45,89-318.
#include "scheduler.h"

#include <stdexcept>

#include "shim.h"

using sana_shim::as_int;
using sana_shim::check;
using sana_shim::handle;
using sana_shim::ptr;
using sana_shim::require;

namespace {

// validate_scheduler_config (scheduler.cpp:8-24).
void validate_config(const SanaSchedulerConfig& c) {
    if (c.solver_order == 0) throw std::invalid_argument("solver_order must be positive");
    if (c.solver_order > 2) throw std::invalid_argument("only solver_order <= 2 is supported");
    if (c.prediction_type != "flow_prediction") throw std::invalid_argument("only flow_prediction is supported");
    if (c.algorithm_type != "dpmsolver++") throw std::invalid_argument("only dpmsolver++ is supported");
    if (c.solver_type != "midpoint" && c.solver_type != "heun")
        throw std::invalid_argument("solver_type must be midpoint or heun");
}

// validate_scheduler_step_inputs (scheduler.cpp:26-41).
void validate_state(const SanaSchedulerState& s) {
    if (s.schedule.timesteps.empty()) throw std::invalid_argument("scheduler state has no timesteps");
    if (s.schedule.sigmas.size() != s.schedule.timesteps.size() + 1)
        throw std::invalid_argument("scheduler sigmas must have one extra final entry");
    if (s.step_index >= s.schedule.timesteps.size()) throw std::invalid_argument("scheduler step_index is out of range");
}

int sigma_count(const SanaSchedulerState& s) { return as_int(s.schedule.sigmas.size(), "sigma count"); }

}  // namespace

namespace sana_shim {
sana_scheduler_config c_config(const SanaSchedulerConfig& c) {
    validate_config(c);
    sana_scheduler_config r;
    sana_scheduler_config_default(&r);
    if (c.num_train_timesteps > static_cast<size_t>(2147483647))
        throw std::invalid_argument("num_train_timesteps does not fit the C ABI's int");
    r.num_train_timesteps = static_cast<int>(c.num_train_timesteps);
    r.flow_shift = c.flow_shift;
    r.use_flow_sigmas = c.use_flow_sigmas ? 1 : 0;
    r.solver_order = static_cast<int>(c.solver_order);
    r.lower_order_final = c.lower_order_final ? 1 : 0;
    r.final_sigmas_zero = c.final_sigmas_type == "zero" ? 1 : 0;
    r.solver_heun = c.solver_type == "heun" ? 1 : 0;
    return r;
}
}  // namespace sana_shim

SanaSchedulerConfig make_sana_scheduler_config() { return SanaSchedulerConfig(); }

SanaSchedulerTimesteps build_sana_scheduler_timesteps(size_t num_inference_steps, const SanaSchedulerConfig& config) {
    validate_config(config);
    if (num_inference_steps == 0) throw std::invalid_argument("num_inference_steps must be positive");
    if (!config.use_flow_sigmas) throw std::invalid_argument("only use_flow_sigmas=true is supported");
    if (config.timestep_spacing != "linspace") throw std::invalid_argument("only linspace timestep_spacing is supported");
    if (config.final_sigmas_type != "zero") throw std::invalid_argument("only zero final_sigmas_type is supported");
    if (config.num_train_timesteps == 0) throw std::invalid_argument("num_train_timesteps must be positive");
    const sana_scheduler_config cc = sana_shim::c_config(config);
    SanaSchedulerTimesteps s;
    s.timesteps.resize(num_inference_steps);
    s.sigmas.resize(num_inference_steps + 1);
    check(sana_scheduler_schedule_config(&cc, as_int(num_inference_steps, "num_inference_steps"), s.timesteps.data(),
                                         s.sigmas.data()));
    return s;
}

SanaSchedulerState init_sana_scheduler_state(size_t num_inference_steps, const SanaSchedulerConfig& config) {
    validate_config(config);
    SanaSchedulerState state;
    state.schedule = build_sana_scheduler_timesteps(num_inference_steps, config);
    state.step_index = 0;
    state.lower_order_step_count = 0;
    return state;
}

Tensor convert_sana_scheduler_model_output(const Tensor& model_output, const Tensor& sample,
                                           const SanaSchedulerState& state, const SanaSchedulerConfig& config) {
    validate_config(config);
    validate_state(state);
    require(model_output.same_shape(sample), "model_output and sample must have the same shape");
    Tensor out(sample.shape());
    if (out.numel() == 0) return out;
    check(sana_scheduler_convert(handle(), state.schedule.sigmas.data(), sigma_count(state),
                                 as_int(state.step_index, "step index"), ptr(model_output), ptr(sample),
                                 as_int(sample.numel(), "numel"), out.data().data()));
    return out;
}

Tensor sana_scheduler_first_order_update(const Tensor& converted_model_output, const Tensor& sample,
                                         const SanaSchedulerState& state, const SanaSchedulerConfig& config) {
    validate_config(config);
    validate_state(state);
    require(converted_model_output.same_shape(sample), "converted_model_output and sample must have the same shape");
    const sana_scheduler_config cc = sana_shim::c_config(config);
    Tensor out(sample.shape());
    if (out.numel() == 0) return out;
    check(sana_scheduler_update_config(handle(), &cc, 1, state.schedule.sigmas.data(), sigma_count(state),
                                       as_int(state.step_index, "step index"), ptr(converted_model_output), nullptr,
                                       ptr(sample), as_int(sample.numel(), "numel"), out.data().data()));
    return out;
}

Tensor sana_scheduler_second_order_update(const Tensor& sample, const SanaSchedulerState& state,
                                          const SanaSchedulerConfig& config) {
    validate_config(config);
    validate_state(state);
    if (state.step_index == 0)
        throw std::invalid_argument("second-order update requires at least one previous step");
    if (state.previous_model_outputs.size() < 2)
        throw std::invalid_argument("second-order update requires two model outputs");
    const Tensor& m0 = state.previous_model_outputs.back();
    const Tensor& m1 = state.previous_model_outputs[state.previous_model_outputs.size() - 2];
    require(m0.same_shape(sample) && m1.same_shape(sample), "stored model outputs must match sample shape");
    const sana_scheduler_config cc = sana_shim::c_config(config);
    Tensor out(sample.shape());
    if (out.numel() == 0) return out;
    check(sana_scheduler_update_config(handle(), &cc, 2, state.schedule.sigmas.data(), sigma_count(state),
                                       as_int(state.step_index, "step index"), ptr(m0), ptr(m1), ptr(sample),
                                       as_int(sample.numel(), "numel"), out.data().data()));
    return out;
}

Tensor step_sana_scheduler(const Tensor& model_output, const Tensor& sample, SanaSchedulerState& state,
                           const SanaSchedulerConfig& config) {
    validate_config(config);
    validate_state(state);
    require(model_output.same_shape(sample), "model_output and sample must have the same shape");
    const sana_scheduler_config cc = sana_shim::c_config(config);
    const size_t numel = sample.numel();
    for (const Tensor& h : state.previous_model_outputs)
        require(h.same_shape(sample), "stored model outputs must match sample shape");
    // the device step takes at most the last two converted outputs, oldest first
    std::vector<float> history(2 * numel);
    const size_t keep = state.previous_model_outputs.size() > 2 ? 2 : state.previous_model_outputs.size();
    const size_t first = state.previous_model_outputs.size() - keep;
    for (size_t i = 0; i < keep; ++i)
        std::copy(state.previous_model_outputs[first + i].data().begin(),
                  state.previous_model_outputs[first + i].data().end(), history.begin() + i * numel);
    int n_history = static_cast<int>(keep);
    int step = as_int(state.step_index, "step index");
    int lower = as_int(state.lower_order_step_count, "lower order count");
    Tensor out(sample.shape());
    check(sana_scheduler_step_config(handle(), &cc, state.schedule.sigmas.data(), sigma_count(state), &step, &lower,
                                     history.data(), &n_history, ptr(model_output), ptr(sample),
                                     as_int(numel, "numel"), out.data().data()));
    state.step_index = static_cast<size_t>(step);
    state.lower_order_step_count = static_cast<size_t>(lower);
    state.previous_model_outputs.clear();
    for (int i = 0; i < n_history; ++i) {
        Tensor h(sample.shape());
        std::copy(history.begin() + i * numel, history.begin() + (i + 1) * numel, h.data().begin());
        state.previous_model_outputs.push_back(std::move(h));
    }
    return out;
}
