// Tests of the C++ host layer (sana.cpp_b200/host): the reference's own API entry points,
// called as sana.cpp's code calls them, running on the GPU through the C ABI.
//
//   test_shim            known-answer tests of the reference's unit tests (fp32 check mode,
//                        the reference's tolerances), error behaviour, and bf16-mode
//                        consistency of the block / step / loop entry points
//   test_shim --no-gpu   only what needs no device: the status -> exception mapping
//
// Expected values are those asserted in cconthekeyboard/sana.cpp tests/test_tensor.cpp,
// tests/test_transformer.cpp and tests/test_scheduler_main.cpp (cited per case).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "sana_cuda.h"
#include "sana_cuda_shim.h"
#include "scheduler.h"
#include "transformer.h"
#include "transformer_ops.h"
#include "vae.h"

namespace {

int g_failed = 0, g_checked = 0;

void expect(bool ok, const std::string& what) {
    ++g_checked;
    if (!ok) {
        ++g_failed;
        std::printf("FAIL %s\n", what.c_str());
    }
}

Tensor T(std::vector<size_t> shape, std::vector<float> v) {
    Tensor t(std::move(shape));
    t.data() = std::move(v);
    return t;
}

void close(const Tensor& got, const std::vector<float>& want, float tol, const std::string& what) {
    bool ok = got.numel() == want.size();
    float worst = 0.0f;
    for (size_t i = 0; ok && i < want.size(); ++i) worst = std::max(worst, std::fabs(got.data()[i] - want[i]));
    ok = ok && worst <= tol;
    if (!ok) {
        std::string g;
        for (size_t i = 0; i < got.numel() && i < 8; ++i) g += std::to_string(got.data()[i]) + " ";
        std::printf("  %s: max|diff| %g (tol %g), got %s\n", what.c_str(), worst, tol, g.c_str());
    }
    expect(ok, what);
}

template <class E>
void throws(const std::function<void()>& f, const std::string& what) {
    bool thrown = false;
    try {
        f();
    } catch (const E&) {
        thrown = true;
    } catch (...) {
    }
    expect(thrown, what + " throws");
}

double rel_l2(const Tensor& a, const Tensor& b) {
    if (!a.same_shape(b)) return 1e30;
    double n = 0, d = 0;
    for (size_t i = 0; i < a.numel(); ++i) {
        const double x = static_cast<double>(a.data()[i]) - b.data()[i];
        n += x * x;
        d += static_cast<double>(b.data()[i]) * b.data()[i];
    }
    return std::sqrt(n / (d > 0 ? d : 1e-30));
}

Tensor eye(size_t n) {
    Tensor t({n, n});
    for (size_t i = 0; i < n; ++i) t.data()[i * n + i] = 1.0f;
    return t;
}

// --- known-answer tests of the reference, fp32 check mode ----------------------------------
void kat_tensor_ops() {
    // test_tensor.cpp:92-148
    const Tensor x = T({1, 2, 2}, {1, 3, 2, 4});
    close(x.layer_norm_3d_lastdim(0.0f), {-1, 1, -1, 1}, 0.0f, "layer_norm_3d_lastdim");
    const Tensor g = T({2}, {2, 3}), b = T({2}, {1, -1});
    close(x.layer_norm_3d_lastdim(0.0f, &g, &b), {-1, 2, -1, 2}, 0.0f, "layer_norm_3d_lastdim affine");
    close(T({1, 2, 2}, {3, 4, 0, 5}).rms_norm_3d_lastdim(0.0f, &g), {1.6970563f, 3.3941126f, 0.0f, 4.2426405f}, 1e-5f,
          "rms_norm_3d_lastdim");
    close(T({1, 2, 2}, {1, 2, 3, 4}).modulate_3d_lastdim(T({1, 1, 2}, {10, 20}), T({1, 1, 2}, {0.5f, -0.5f})),
          {11.5f, 21.0f, 14.5f, 22.0f}, 0.0f, "modulate_3d_lastdim");
}

void qkv(Tensor& q, Tensor& k, Tensor& v) {
    // test_transformer.cpp:180-210
    q = T({1, 1, 2, 2}, {1, 0, 0, 1});
    k = T({1, 1, 2, 2}, {1, 2, 3, 4});
    v = T({1, 1, 2, 2}, {10, 20, 30, 40});
}

void kat_transformer_ops() {
    Tensor q({1}), k({1}), v({1});
    qkv(q, k, v);
    // test_transformer.cpp:229-241
    const std::vector<float> att = {26.088594f, 36.088594f, 26.088594f, 36.088594f};
    close(attention_4d(q, k, v), att, 1e-5f, "attention_4d");
    close(linear_attention_4d(q, k, v), {25.0f, 35.0f, 23.333334f, 33.333332f}, 1e-5f, "linear_attention_4d");
    // attention_4d restated from its parts (transformer_ops.cpp:348-392)
    Tensor s = attention_scores_4d(q, k);
    close(s, {1, 3, 2, 4}, 0.0f, "attention_scores_4d");
    s.mul_inplace_scalar(1.0f / std::sqrt(2.0f));
    close(attention_values_4d(softmax_lastdim_4d(s), v), att, 1e-5f, "attention_4d from scores, softmax, values");
    close(softmax_lastdim_4d(T({1, 1, 1, 3}, {0.0f, std::log(2.0f), std::log(5.0f)})), {0.125f, 0.25f, 0.625f}, 1e-6f,
          "softmax_lastdim_4d");
    // split_heads_3d / merge_heads_4d (transformer_ops.cpp:83-171)
    Tensor x({2, 3, 8});
    for (size_t i = 0; i < x.numel(); ++i) x.data()[i] = static_cast<float>(i);
    const Tensor h = split_heads_3d(x, 4);
    expect(h.shape() == std::vector<size_t>({2, 4, 3, 2}), "split_heads_3d shape");
    // element [b=1, head=2, t=1, d=1] = x[1, 1, 2*2 + 1]
    expect(h.at({1, 2, 1, 1}) == x.at({1, 1, 5}), "split_heads_3d layout");
    close(merge_heads_4d(h), x.data(), 0.0f, "merge_heads_4d inverts split_heads_3d");
    // project_caption_context, test_transformer.cpp:243-280
    Tensor w1({4, 2});
    w1.at({0, 0}) = 1.0f;
    w1.at({1, 1}) = 1.0f;
    const Tensor zb({2});
    close(project_caption_context(T({1, 2, 4}, {1, 2, 3, 4, 5, 6, 7, 8}), w1, &zb, eye(2), &zb, T({2}, {1, 2})),
          {0.5590534f, 2.5980382f, 0.9053573f, 2.1728575f}, 1e-5f, "project_caption_context");
    // attention_block_3d / cross_attention_block_3d, test_transformer.cpp:310-371
    const Tensor xe = T({1, 2, 2}, {1, 0, 0, 1}), w = eye(2);
    close(attention_block_3d(xe, w, &zb, w, &zb, w, &zb, w, &zb, 1), {1, 0, 0, 1}, 1e-5f, "attention_block_3d");
    close(cross_attention_block_3d(xe, T({1, 2, 2}, {2, 0, 0, 3}), nullptr, w, &zb, w, &zb, w, &zb, w, &zb, 1),
          {1.6088594f, 0.5867110f, 0.2140836f, 2.6788745f}, 1e-5f, "cross_attention_block_3d");
}

// The one-token block of test_transformer.cpp:373-484: hidden 2, one head each, identity (or
// zero) projections, the GLUMB weights of test_tensor.cpp:273-304, gates 1 from the timestep.
SanaBlockWeights kat_block(bool residual_only) {
    const size_t C = 2;
    const Tensor proj = residual_only ? Tensor({C, C}) : eye(C);
    const Tensor zb({C});
    Tensor w_inv({4, 2, 1, 1}), w_dw({4, 1, 3, 3}), w_pt({2, 2, 1, 1});
    w_inv.at({0, 0, 0, 0}) = w_inv.at({1, 1, 0, 0}) = w_inv.at({2, 0, 0, 0}) = w_inv.at({3, 1, 0, 0}) = 1.0f;
    for (size_t c = 0; c < 4; ++c) w_dw.at({c, 0, 1, 1}) = 1.0f;
    w_pt.at({0, 0, 0, 0}) = w_pt.at({1, 1, 0, 0}) = 1.0f;
    return SanaBlockWeights{Tensor({6, C}), Tensor({0}), Tensor({0}), proj, zb, proj, zb, proj, zb, proj, zb,
                            proj, zb, proj, zb, proj, zb, proj, zb, Tensor({0}), Tensor({0}), w_inv, Tensor({4}),
                            w_dw, Tensor({4}), w_pt, 1, 1};
}

void kat_block_forward() {
    const Tensor x = T({1, 1, 2}, {1, 0}), ctx = T({1, 2, 2}, {2, 0, 0, 3});
    Tensor tmod({1, 12});
    for (size_t i : {4, 5, 10, 11}) tmod.data()[i] = 1.0f;
    close(block_forward(x, ctx, tmod, kat_block(false)).after_ff, {4.3467007f, -0.9475632f}, 1e-5f, "block_forward");
    close(block_forward(x, ctx, tmod, kat_block(true)).after_ff, {1.3607715f, 0.0313307f}, 1e-5f,
          "block_forward residual only");
    // compute_sana_block_modulation (transformer.cpp:496-542)
    Tensor table({6, 2});
    for (size_t i = 0; i < 12; ++i) table.data()[i] = 0.5f * static_cast<float>(i);
    const SanaBlockModulation m = compute_sana_block_modulation(tmod, table);
    close(m.gate_msa, {1.0f + 2.0f, 1.0f + 2.5f}, 0.0f, "compute_sana_block_modulation gate_msa");
    close(m.scale_mlp, {4.0f, 4.5f}, 0.0f, "compute_sana_block_modulation scale_mlp");
    // apply_classifier_free_guidance (transformer.cpp:570-602): uncond + g (cond - uncond)
    close(apply_classifier_free_guidance(T({2, 1, 1, 2}, {1, 2, 3, 6}), 4.5f), {1 + 4.5f * 2, 2 + 4.5f * 4}, 1e-5f,
          "apply_classifier_free_guidance");
}

void kat_scheduler() {
    // test_scheduler_main.cpp:27-41
    const SanaSchedulerConfig cfg = make_sana_scheduler_config();
    const SanaSchedulerTimesteps s4 = build_sana_scheduler_timesteps(4, cfg);
    close(T({4}, s4.timesteps), {999, 899, 749, 499}, 1e-3f, "build_sana_scheduler_timesteps timesteps");
    close(T({5}, s4.sigmas), {0.99966644f, 0.89963979f, 0.74962479f, 0.49966654f, 0.0f}, 1e-6f,
          "build_sana_scheduler_timesteps sigmas");
    // test_scheduler_main.cpp:80-115
    SanaSchedulerState st;
    st.schedule.sigmas = {0.8f, 0.5f, 0.2f, 0.0f};
    st.schedule.timesteps = {800, 500, 200};
    const Tensor mo = T({1}, {2.0f}), sample = T({1}, {4.0f});
    const Tensor conv = convert_sana_scheduler_model_output(mo, sample, st, cfg);
    close(conv, {2.4f}, 1e-6f, "convert_sana_scheduler_model_output");
    close(sana_scheduler_first_order_update(conv, sample, st, cfg), {3.4f}, 1e-5f, "first_order_update");
    close(step_sana_scheduler(mo, sample, st, cfg), {3.4f}, 1e-5f, "step_sana_scheduler");
    expect(st.previous_model_outputs.size() == 1 && std::fabs(st.previous_model_outputs[0].data()[0] - 2.4f) < 1e-6f,
           "step_sana_scheduler history");
    expect(st.lower_order_step_count == 1 && st.step_index == 1, "step_sana_scheduler counters");
    SanaSchedulerState s2;
    s2.schedule.sigmas = {0.8f, 0.5f, 0.2f, 0.1f, 0.09f, 0.08f, 0.07f, 0.06f, 0.05f, 0.04f, 0.03f, 0.02f, 0.015f,
                          0.01f, 0.005f, 0.001f, 0.0f};
    s2.schedule.timesteps.assign(16, 1.0f);
    s2.step_index = 1;
    s2.lower_order_step_count = 1;
    s2.previous_model_outputs = {T({1}, {2.4f}), T({1}, {2.0f})};
    close(sana_scheduler_second_order_update(T({1}, {3.4f}), s2, cfg), {2.44f}, 1e-5f, "second_order_update");
    step_sana_scheduler(T({1}, {3.1f}), T({1}, {3.4f}), s2, cfg);
    expect(s2.previous_model_outputs.size() == 2 && s2.lower_order_step_count == 2 && s2.step_index == 2,
           "step_sana_scheduler second step state");
}

// Scheduler configurations other than the default (scheduler.cpp:71-81,207-318): heun and
// midpoint second order, solver_order 1, lower_order_final off, variance-preserving sigmas,
// other num_train_timesteps. Expected values: the reference build's step_sana_scheduler on
// the same inputs (tests/golden/make_golden.py scheduler -> scheduler_configs.inc).
#include "scheduler_configs.inc"

SanaSchedulerConfig sched_case_config(int i) {
    const int* c = kSchedCfg + 9 * i;
    SanaSchedulerConfig cfg = make_sana_scheduler_config();
    cfg.num_train_timesteps = static_cast<size_t>(c[0]);
    cfg.flow_shift = static_cast<float>(c[1]) / 1000.0f;
    cfg.use_flow_sigmas = c[2] != 0;
    cfg.solver_order = static_cast<size_t>(c[3]);
    cfg.lower_order_final = c[4] != 0;
    cfg.final_sigmas_type = c[5] ? "zero" : "sigma_min";
    cfg.solver_type = c[6] ? "heun" : "midpoint";
    return cfg;
}

// Host only: the schedules build_sana_scheduler_timesteps makes for every buildable case.
void scheduler_config_schedules() {
    for (int i = 0; i < kSchedCases; ++i) {
        const int* c = kSchedCfg + 9 * i;
        if (c[8]) continue;
        const size_t n = static_cast<size_t>(c[7]);
        const SanaSchedulerTimesteps s = build_sana_scheduler_timesteps(n, sched_case_config(i));
        const float* want = kSchedSchedule + kSchedSgOff[i];
        bool same = s.timesteps.size() == n && s.sigmas.size() == n + 1;
        for (size_t j = 0; same && j < n; ++j) same = s.timesteps[j] == want[j];
        for (size_t j = 0; same && j <= n; ++j) same = s.sigmas[j] == want[n + j];
        expect(same, "build_sana_scheduler_timesteps config case " + std::to_string(i));
    }
    SanaSchedulerConfig vp = make_sana_scheduler_config();
    vp.use_flow_sigmas = false;
    throws<std::invalid_argument>([&] { build_sana_scheduler_timesteps(4, vp); }, "schedule without flow sigmas");
    SanaSchedulerConfig zero_train = make_sana_scheduler_config();
    zero_train.num_train_timesteps = 0;
    throws<std::invalid_argument>([&] { build_sana_scheduler_timesteps(4, zero_train); }, "num_train_timesteps 0");
}

// On the device: every case stepped through step_sana_scheduler, each step's sample within
// 1e-6 of the reference's (relative to the sample's largest magnitude).
void scheduler_config_steps() {
    for (int i = 0; i < kSchedCases; ++i) {
        const int* c = kSchedCfg + 9 * i;
        const size_t n = static_cast<size_t>(c[7]), numel = static_cast<size_t>(kSchedNumel);
        const SanaSchedulerConfig cfg = sched_case_config(i);
        SanaSchedulerState st;
        st.schedule.timesteps.assign(kSchedSchedule + kSchedSgOff[i], kSchedSchedule + kSchedSgOff[i] + n);
        st.schedule.sigmas.assign(kSchedSchedule + kSchedSgOff[i] + n, kSchedSchedule + kSchedSgOff[i] + 2 * n + 1);
        Tensor x = T({numel}, std::vector<float>(kSchedSample0 + i * numel, kSchedSample0 + (i + 1) * numel));
        const float* mo = kSchedModelOut + kSchedMoOff[i];
        const float* want_all = kSchedSamples + kSchedMoOff[i];
        double worst = 0.0;
        for (size_t s = 0; s < n; ++s) {
            x = step_sana_scheduler(T({numel}, std::vector<float>(mo + s * numel, mo + (s + 1) * numel)), x, st, cfg);
            double scale = 1e-30, diff = 0.0;
            for (size_t j = 0; j < numel; ++j) {
                scale = std::max(scale, static_cast<double>(std::fabs(want_all[s * numel + j])));
                diff = std::max(diff, static_cast<double>(std::fabs(x.data()[j] - want_all[s * numel + j])));
            }
            worst = std::max(worst, diff / scale);
        }
        const bool ok = worst <= 1e-6 && st.step_index == n &&
                        st.previous_model_outputs.size() == std::min<size_t>(n, cfg.solver_order) &&
                        st.lower_order_step_count == std::min<size_t>(n, cfg.solver_order);
        if (!ok) std::printf("  scheduler config case %d: worst relative diff %g\n", i, worst);
        expect(ok, "step_sana_scheduler config case " + std::to_string(i));
    }
}

void errors() {
    // the reference's std::invalid_argument contracts (test_transformer.cpp:511-619)
    throws<std::invalid_argument>([] { split_heads_3d(Tensor({1, 2, 6}), 4); }, "split_heads_3d bad heads");
    throws<std::invalid_argument>([] { split_heads_3d(Tensor({1, 2, 6}), 0); }, "split_heads_3d zero heads");
    throws<std::invalid_argument>([] { merge_heads_4d(Tensor({1, 2, 6})); }, "merge_heads_4d rank");
    throws<std::invalid_argument>([] { apply_classifier_free_guidance(Tensor({3, 1, 2, 2}), 1.0f); },
                                  "apply_classifier_free_guidance odd batch");
    throws<std::invalid_argument>([] { softmax_lastdim_4d(Tensor({2, 3})); }, "softmax_lastdim_4d rank");
    throws<std::invalid_argument>(
        [] { compute_sana_block_modulation(Tensor({1, 12}), Tensor({5, 2})); }, "compute_sana_block_modulation table");
    const SanaDenoiserWeights none{SanaCaptionWeights{Tensor({0}), Tensor({0}), Tensor({0}), Tensor({0})}, {},
                                   Tensor({0}), Tensor({0}), Tensor({0}), Tensor({0}), Tensor({0}), Tensor({0}),
                                   Tensor({0}), Tensor({0}), Tensor({0}), Tensor({0}), Tensor({0}), Tensor({0})};
    throws<std::invalid_argument>(
        [&] { run_model_blocks(Tensor({1, 1, 2}), Tensor({1, 1, 2}), Tensor({1, 12}), none, 0, 1); },
        "run_model_blocks range");
    SanaSchedulerState st = init_sana_scheduler_state(2, make_sana_scheduler_config());
    st.step_index = 2;
    throws<std::invalid_argument>([&] { step_sana_scheduler(Tensor({1}), Tensor({1}), st, make_sana_scheduler_config()); },
                                  "step_sana_scheduler step_index");
    SanaSchedulerState fresh = init_sana_scheduler_state(4, make_sana_scheduler_config());
    throws<std::invalid_argument>(
        [&] { sana_scheduler_second_order_update(Tensor({1}), fresh, make_sana_scheduler_config()); },
        "second order update at step 0");
    SanaSchedulerConfig bad = make_sana_scheduler_config();
    bad.solver_order = 3;
    throws<std::invalid_argument>([&] { build_sana_scheduler_timesteps(4, bad); }, "solver_order 3");
    throws<std::invalid_argument>([] { build_sana_scheduler_timesteps(0, make_sana_scheduler_config()); },
                                  "zero inference steps");
}

// --- bf16 mode: a small random model through the block / step / loop entry points --------
struct Rng {
    std::mt19937 g{1234};
    std::normal_distribution<float> n{0.0f, 1.0f};
    Tensor t(std::vector<size_t> shape, float scale) {
        Tensor x(std::move(shape));
        for (float& v : x.data()) v = scale * n(g);
        return x;
    }
};

SanaDenoiserWeights small_model(Rng& r, size_t C, size_t nb, size_t Cl, size_t Din, size_t E) {
    std::vector<SanaBlockWeights> blocks;
    for (size_t i = 0; i < nb; ++i) {
        blocks.push_back(SanaBlockWeights{
            r.t({6, C}, 0.1f), r.t({C}, 0.1f), r.t({C}, 0.1f), r.t({C, C}, 0.1f), r.t({C}, 0.02f), r.t({C, C}, 0.1f),
            r.t({C}, 0.02f), r.t({C, C}, 0.1f), r.t({C}, 0.02f), r.t({C, C}, 0.1f), r.t({C}, 0.02f), r.t({C, C}, 0.1f),
            r.t({C}, 0.02f), r.t({C, C}, 0.1f), r.t({C}, 0.02f), r.t({C, C}, 0.1f), r.t({C}, 0.02f), r.t({C, C}, 0.1f),
            r.t({C}, 0.02f), r.t({C}, 0.1f), r.t({C}, 0.1f), r.t({E, C, 1, 1}, 0.1f), r.t({E}, 0.02f),
            r.t({E, 1, 3, 3}, 0.2f), r.t({E}, 0.02f), r.t({C, E / 2, 1, 1}, 0.1f), 4, 2});
    }
    Tensor norm = r.t({C}, 0.1f);
    for (float& v : norm.data()) v += 1.0f;
    return SanaDenoiserWeights{
        SanaCaptionWeights{r.t({Din, C}, 0.1f), r.t({C}, 0.02f), r.t({C, C}, 0.1f), r.t({C}, 0.02f)},
        blocks,
        r.t({C, Cl, 1, 1}, 0.2f), r.t({C}, 0.02f),            // patch embed
        r.t({256, C}, 0.05f), r.t({C}, 0.02f),                 // time embedding linear 1
        r.t({C, C}, 0.1f), r.t({C}, 0.02f),                    // time embedding linear 2
        r.t({C, 6 * C}, 0.1f), r.t({6 * C}, 0.02f),            // t_block
        norm, r.t({2, C}, 0.1f),                               // caption norm, final table
        r.t({C, Cl}, 0.1f), r.t({Cl}, 0.02f)};                 // proj_out
}

void bf16_consistency() {
    Rng r;
    const size_t C = 64, nb = 2, Cl = 4, Din = 48, E = 160, L = 12, side = 8;
    const SanaDenoiserWeights w = small_model(r, C, nb, Cl, Din, E);
    const Tensor lat = r.t({1, Cl, side, side}, 1.0f), enc = r.t({2, L, Din}, 1.0f);
    Tensor bias({2, 1, L});
    for (size_t j = 5; j < L; ++j) bias.data()[j] = -10000.0f;  // uncond row: 5 valid keys

    // run_model_blocks against the chained block_forward of each block
    const Tensor x = r.t({2, side * side, C}, 1.0f), ctx = r.t({2, L, C}, 1.0f), tmod = r.t({2, 6 * C}, 0.1f);
    const Tensor all = run_model_blocks(x, ctx, tmod, w, 0, nb, &bias);
    Tensor chained = x;
    for (size_t b = 0; b < nb; ++b) chained = block_forward(chained, ctx, tmod, w.blocks[b], &bias).after_ff;
    const double e_blocks = rel_l2(all, chained);
    std::printf("  run_model_blocks vs chained block_forward: rel L2 %.2e\n", e_blocks);
    expect(e_blocks < 1e-2, "run_model_blocks matches chained block_forward");
    expect(run_model_blocks(x, ctx, tmod, w, 1, 1, &bias).data() == x.data(), "run_model_blocks empty range");

    // the device loop (fresh state) against the reference loop of single steps
    const SanaSchedulerConfig cfg = make_sana_scheduler_config();
    SanaSchedulerState fused = init_sana_scheduler_state(4, cfg);
    const Tensor out_loop = run_full_denoising_loop_with_cfg(lat, enc, 4.5f, fused, cfg, w, &bias);
    expect(fused.step_index == 4 && fused.lower_order_step_count == 2, "loop advances the scheduler state");
    SanaSchedulerState stepped = init_sana_scheduler_state(4, cfg);
    const Tensor context = project_caption_context(enc, w.caption.linear_1_weight, &w.caption.linear_1_bias,
                                                   w.caption.linear_2_weight, &w.caption.linear_2_bias,
                                                   w.caption_norm_weight);
    Tensor lat_s = lat;
    while (stepped.step_index < 4) lat_s = run_full_denoising_step_with_cfg(lat_s, context, 4.5f, stepped, cfg, w, &bias);
    const double e_loop = rel_l2(out_loop, lat_s);
    std::printf("  device loop vs stepped loop: rel L2 %.2e\n", e_loop);
    expect(e_loop < 2e-2, "run_full_denoising_loop_with_cfg matches run_full_denoising_step_with_cfg");
    expect(stepped.previous_model_outputs.size() == 2, "stepped state keeps two model outputs");
    // a started state takes the step-by-step path and continues where it stopped
    SanaSchedulerState half = init_sana_scheduler_state(4, cfg);
    Tensor lat_h = lat;
    for (int i = 0; i < 2; ++i) lat_h = run_full_denoising_step_with_cfg(lat_h, context, 4.5f, half, cfg, w, &bias);
    const Tensor out_h = run_full_denoising_loop_with_cfg(lat_h, enc, 4.5f, half, cfg, w, &bias);
    const double e_half = rel_l2(out_h, lat_s);
    std::printf("  resumed loop vs stepped loop: rel L2 %.2e\n", e_half);
    expect(e_half < 2e-2 && half.step_index == 4, "loop resumes a started state");
}

// run_vae_decode through the reference's SanaVaeWeights structure: the same image as the C
// ABI given the documented tensor table, the validators' std::invalid_argument contracts,
// and a fresh upload after invalidate_weights().
void vae_decode_entry_point() {
    std::mt19937 g{77};
    std::normal_distribution<float> nd(0.0f, 1.0f);
    auto rnd = [&](std::vector<size_t> shape, float scale, float offset = 0.0f) {
        Tensor t(std::move(shape));
        for (float& v : t.data()) v = offset + scale * nd(g);
        return t;
    };
    const size_t Cl = 8, ch[3] = {16, 32, 64};
    SanaVaeWeights w{SanaVaeDecoderWeights{rnd({ch[2], Cl, 3, 3}, 0.02f), rnd({ch[2]}, 0.02f), rnd({ch[0]}, 0.1f, 1.0f),
                                           rnd({ch[0]}, 0.1f), rnd({3, ch[0], 3, 3}, 0.02f), rnd({3}, 0.02f), {}},
                     0.5f, 32};
    SanaVaeDecoderWeights& d = w.decoder;
    for (int i = 0; i < 3; ++i) {
        const size_t c = ch[i];
        SanaVaeUpBlockWeights b;
        if (i < 2) {
            b.upsample_conv_weight = rnd({c, ch[i + 1], 3, 3}, 0.02f);
            b.upsample_conv_bias = rnd({c}, 0.02f);
            b.is_res_block = true;
            for (int l = 0; l < 1 + i; ++l)
                b.res_blocks.push_back({rnd({c, c, 3, 3}, 0.02f), rnd({c}, 0.02f), rnd({c, c, 3, 3}, 0.02f),
                                        rnd({c}, 0.1f, 1.0f), rnd({c}, 0.1f)});
        } else {
            for (int l = 0; l < 2; ++l) {
                SanaVaeAttnGlumbLayerWeights layer{
                    {rnd({c, c, 1, 1}, 0.02f), rnd({c, c, 1, 1}, 0.02f), rnd({c, c, 1, 1}, 0.02f),
                     rnd({3 * c, 1, 5, 5}, 0.02f), rnd({3 * c, 32, 1, 1}, 0.02f), rnd({c, 2 * c, 1, 1}, 0.02f),
                     rnd({c}, 0.1f, 1.0f), rnd({c}, 0.1f)},
                    {rnd({8 * c, c, 1, 1}, 0.02f), rnd({8 * c}, 0.02f), rnd({8 * c, 1, 3, 3}, 0.02f),
                     rnd({8 * c}, 0.02f), rnd({c, 4 * c, 1, 1}, 0.02f), rnd({c}, 0.1f, 1.0f), rnd({c}, 0.1f)}};
                b.attn_glumb_layers.push_back(std::move(layer));
            }
        }
        d.up_blocks.push_back(std::move(b));
    }
    const Tensor lat = rnd({2, Cl, 4, 6}, 1.0f);
    const Tensor img = run_vae_decode(lat, w);
    expect(img.rank() == 4 && img.dim_size(0) == 2 && img.dim_size(1) == 3 && img.dim_size(2) == 16 &&
               img.dim_size(3) == 24,
           "run_vae_decode output shape [2, 3, 16, 24]");

    // the C ABI on its own handle, tensors in include/sana_cuda.h's documented order
    std::vector<const float*> table;
    auto add = [&](const Tensor& t) { table.push_back(t.data().data()); };
    for (const Tensor* t : {&d.conv_in_weight, &d.conv_in_bias, &d.norm_out_weight, &d.norm_out_bias,
                            &d.conv_out_weight, &d.conv_out_bias})
        add(*t);
    sana_vae_dims dims{};
    dims.latent_channels = static_cast<int>(Cl);
    dims.out_channels = 3;
    dims.n_blocks = 3;
    dims.head_dim = 32;
    dims.ms_kernel = 5;
    dims.scaling_factor = 0.5f;
    for (int i = 0; i < 3; ++i) {
        const SanaVaeUpBlockWeights& b = d.up_blocks[i];
        dims.blocks[i] = {static_cast<int>(ch[i]), i < 2 ? 1 : 0, i < 2 ? 1 : 0,
                          static_cast<int>(i < 2 ? b.res_blocks.size() : b.attn_glumb_layers.size())};
        if (i < 2) {
            add(*b.upsample_conv_weight);
            add(*b.upsample_conv_bias);
            for (const SanaVaeResBlockWeights& r : b.res_blocks)
                for (const Tensor* t : {&r.conv1_weight, &r.conv1_bias, &r.conv2_weight, &r.norm_weight, &r.norm_bias})
                    add(*t);
        } else {
            for (const SanaVaeAttnGlumbLayerWeights& l : b.attn_glumb_layers)
                for (const Tensor* t : {&l.attention.to_q_weight_conv1x1, &l.attention.to_k_weight_conv1x1,
                                        &l.attention.to_v_weight_conv1x1, &l.attention.proj_in_weight,
                                        &l.attention.proj_out_weight, &l.attention.to_out_weight_conv1x1,
                                        &l.attention.norm_out_weight, &l.attention.norm_out_bias,
                                        &l.glumb.conv_inverted_weight, &l.glumb.conv_inverted_bias,
                                        &l.glumb.conv_depth_weight, &l.glumb.conv_depth_bias,
                                        &l.glumb.conv_point_weight, &l.glumb.norm_weight, &l.glumb.norm_bias})
                    add(*t);
        }
    }
    sana_cuda_ctx* h = nullptr;
    bool ok = sana_cuda_create(0, SANA_MODE_F32, &h) == SANA_OK;
    ok = ok && sana_cuda_vae_upload(h, &dims, table.data()) == SANA_OK;
    Tensor direct({2, 3, 16, 24});
    ok = ok && sana_cuda_vae_decode(h, lat.data().data(), 2, 4, 6, direct.data().data()) == SANA_OK;
    if (h) sana_cuda_destroy(h);
    expect(ok && direct.data() == img.data(), "run_vae_decode equals the C ABI on the documented table");

    // the validators and shape contracts (vae.cpp:172-208, 247-254)
    throws<std::invalid_argument>([&] { run_vae_decode(Tensor({2, Cl, 4}), w); }, "vae latents of rank 3");
    throws<std::invalid_argument>([&] { run_vae_decode(Tensor({1, Cl + 1, 2, 2}), w); }, "vae latent channels");
    SanaVaeWeights bad = w;
    bad.decoder.conv_in_bias = Tensor({ch[2] + 1});
    throws<std::invalid_argument>([&] { validate_vae_weights(bad); }, "vae conv_in bias shape");
    bad = w;
    bad.scaling_factor = 0.0f;
    throws<std::invalid_argument>([&] { run_vae_decode(lat, bad); }, "vae scaling factor");

    // weights changed in place: the cached upload is refreshed after invalidate_weights()
    SanaVaeWeights w2 = w;
    const Tensor before = run_vae_decode(lat, w2);
    for (float& v : w2.decoder.conv_out_bias.data()) v += 1.0f;
    sana_cuda_shim::invalidate_weights();
    const Tensor after = run_vae_decode(lat, w2);
    double shift = 0.0;
    for (size_t i = 0; i < after.numel(); ++i) shift += after.data()[i] - before.data()[i];
    expect(std::fabs(shift / static_cast<double>(after.numel()) - 1.0) < 1e-4, "vae upload refreshed after invalidate");
}

}  // namespace

int main(int argc, char** argv) {
    const bool no_gpu = argc > 1 && std::strcmp(argv[1], "--no-gpu") == 0;
    if (no_gpu) {
        // No device: the first call fails to create a handle and reports it as an exception.
        throws<std::runtime_error>([] { linear_attention_4d(Tensor({1, 1, 1, 1}), Tensor({1, 1, 1, 1}),
                                                            Tensor({1, 1, 1, 1})); },
                                   "call without a CUDA device");
        // shape errors are found before any device work
        throws<std::invalid_argument>([] { split_heads_3d(Tensor({1, 2, 6}), 4); }, "split_heads_3d bad heads");
        scheduler_config_schedules();
    } else {
        sana_cuda_shim::configure(0, SANA_MODE_F32);
        kat_tensor_ops();
        kat_transformer_ops();
        kat_block_forward();
        kat_scheduler();
        scheduler_config_schedules();
        scheduler_config_steps();
        errors();
        vae_decode_entry_point();
        sana_cuda_shim::configure(0, SANA_MODE_BF16);
        bf16_consistency();
    }
    std::printf("%d checks, %d failed\n", g_checked, g_failed);
    return g_failed == 0 ? 0 : 1;
}
