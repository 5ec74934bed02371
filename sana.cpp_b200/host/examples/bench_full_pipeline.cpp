// The reference's full-pipeline benchmark (cconthekeyboard/sana.cpp tests/bench_full_pipeline.cpp)
// on the CUDA host layer: the same call sequence through the reference's own API —
// conditioning, run_full_denoising_loop_with_cfg, run_vae_decode — with the same timing
// summary. The Gemma-2 encoder (llama.cpp) is not part of this build: "encoder" here is the
// encoder's output contract (sana_prompt_pair_assemble: uncond first, row-0 + tail slice,
// -10000 mask) applied to synthetic hidden states. Weights are random-initialised with the
// real shapes (Sana-0.6B, DC-AE f32c32), linear weights in the loaders' [in, out] layout.
//
//   bench_full_pipeline [warmup] [iters] [--small]
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "sana_cuda.h"
#include "scheduler.h"
#include "transformer.h"
#include "vae.h"

namespace {

using Clock = std::chrono::steady_clock;
double elapsed_ms(Clock::time_point a, Clock::time_point b) {
    return std::chrono::duration<double, std::milli>(b - a).count();
}

// Uniform values with standard deviation `stdev` (xorshift64*), `offset` added.
struct Fill {
    uint64_t s = 0x9e3779b97f4a7c15ull;
    Tensor operator()(std::vector<size_t> shape, float stdev, float offset = 0.0f) {
        Tensor t(std::move(shape));
        const float a = stdev * 1.7320508f;
        for (float& v : t.data()) {
            s ^= s >> 12;
            s ^= s << 25;
            s ^= s >> 27;
            const uint64_t r = s * 0x2545f4914f6cdd1dull;
            v = offset + a * (static_cast<float>(r >> 40) * (2.0f / 16777216.0f) - 1.0f);
        }
        return t;
    }
};

struct Dims {
    size_t blocks, C, Cl, Din, E, self_heads, cross_heads, L, pos_rows;
    std::vector<size_t> vae_channels;
    std::vector<bool> vae_res;
    size_t vae_layers, latent_hw;
};

SanaDenoiserWeights make_denoiser(const Dims& d, Fill& f) {
    const size_t C = d.C, E = d.E;
    SanaDenoiserWeights w{SanaCaptionWeights{f({d.Din, C}, 0.02f), f({C}, 0.02f), f({C, C}, 0.02f), f({C}, 0.02f)},
                          {},
                          f({C, d.Cl, 1, 1}, 0.02f), f({C}, 0.02f),
                          f({256, C}, 0.02f), f({C}, 0.02f), f({C, C}, 0.02f), f({C}, 0.02f),
                          f({C, 6 * C}, 0.02f), f({6 * C}, 0.02f),
                          f({C}, 0.0f, 1.0f), f({2, C}, 1.0f / std::sqrt(static_cast<float>(C))),
                          f({C, d.Cl}, 0.02f), f({d.Cl}, 0.02f)};
    for (size_t b = 0; b < d.blocks; ++b) {
        w.blocks.push_back(SanaBlockWeights{
            f({6, C}, 1.0f / std::sqrt(static_cast<float>(C))), Tensor({0}), Tensor({0}),
            f({C, C}, 0.02f), f({C}, 0.02f), f({C, C}, 0.02f), f({C}, 0.02f), f({C, C}, 0.02f), f({C}, 0.02f),
            f({C, C}, 0.02f), f({C}, 0.02f),
            f({C, C}, 0.02f), f({C}, 0.02f), f({C, C}, 0.02f), f({C}, 0.02f), f({C, C}, 0.02f), f({C}, 0.02f),
            f({C, C}, 0.02f), f({C}, 0.02f), Tensor({0}), Tensor({0}),
            f({E, C, 1, 1}, 0.02f), f({E}, 0.02f), f({E, 1, 3, 3}, 0.02f), f({E}, 0.02f),
            f({C, E / 2, 1, 1}, 0.02f), d.self_heads, d.cross_heads});
    }
    return w;
}

SanaVaeWeights make_vae(const Dims& d, Fill& f) {
    const std::vector<size_t>& ch = d.vae_channels;
    const size_t n = ch.size();
    SanaVaeWeights w{SanaVaeDecoderWeights{f({ch[n - 1], d.Cl, 3, 3}, 0.02f), f({ch[n - 1]}, 0.02f),
                                           f({ch[0]}, 0.1f, 1.0f), f({ch[0]}, 0.1f), f({3, ch[0], 3, 3}, 0.02f),
                                           f({3}, 0.02f), {}},
                     0.41407f, 32};
    for (size_t i = 0; i < n; ++i) {
        const size_t c = ch[i];
        SanaVaeUpBlockWeights b;
        if (i + 1 < n) {
            b.upsample_conv_weight = f({c, ch[i + 1], 3, 3}, 0.02f);
            b.upsample_conv_bias = f({c}, 0.02f);
            b.is_res_block = d.vae_res[i];
        }
        for (size_t l = 0; l < d.vae_layers; ++l) {
            if (b.is_res_block) {
                b.res_blocks.push_back({f({c, c, 3, 3}, 0.02f), f({c}, 0.02f), f({c, c, 3, 3}, 0.02f),
                                        f({c}, 0.1f, 1.0f), f({c}, 0.1f)});
            } else {
                b.attn_glumb_layers.push_back(
                    {{f({c, c, 1, 1}, 0.02f), f({c, c, 1, 1}, 0.02f), f({c, c, 1, 1}, 0.02f), f({3 * c, 1, 5, 5}, 0.02f),
                      f({3 * c, 32, 1, 1}, 0.02f), f({c, 2 * c, 1, 1}, 0.02f), f({c}, 0.1f, 1.0f), f({c}, 0.1f)},
                     {f({8 * c, c, 1, 1}, 0.02f), f({8 * c}, 0.02f), f({8 * c, 1, 3, 3}, 0.02f), f({8 * c}, 0.02f),
                      f({c, 4 * c, 1, 1}, 0.02f), f({c}, 0.1f, 1.0f), f({c}, 0.1f)}});
            }
        }
        w.decoder.up_blocks.push_back(std::move(b));
    }
    return w;
}

struct PipelineRunResult {
    Tensor decoded_image;
    double encoder_ms = 0.0;
    double transformer_ms = 0.0;
    double vae_ms = 0.0;
    double total_ms = 0.0;
};

PipelineRunResult run_pipeline_once(const Dims& d, const Tensor& negative_states, const Tensor& positive_states,
                                    float guidance_scale, const Tensor& initial_latent, size_t num_steps,
                                    const SanaSchedulerConfig& scheduler_config,
                                    const SanaDenoiserWeights& denoiser_weights, const SanaVaeWeights& vae_weights) {
    const auto total_start = Clock::now();

    const auto encoder_start = Clock::now();
    Tensor embeddings({2, d.L, d.Din});
    Tensor attention_bias({2, 1, d.L});
    char err[256] = {0};
    // real tokens: 8 in the negative prompt, 40 in the instruction-prefixed positive one
    const size_t neg_real = d.L < 8 ? d.L : 8, pos_real = d.pos_rows < 40 ? d.pos_rows : 40;
    if (sana_prompt_pair_assemble(negative_states.data().data(), d.L, neg_real, positive_states.data().data(),
                                  d.pos_rows, pos_real, d.Din, d.L, embeddings.data().data(),
                                  attention_bias.data().data(), err, sizeof(err)) != SANA_OK)
        throw std::invalid_argument(err);
    const auto encoder_end = Clock::now();

    const auto transformer_start = Clock::now();
    SanaSchedulerState scheduler_state = init_sana_scheduler_state(num_steps, scheduler_config);
    Tensor final_latents = run_full_denoising_loop_with_cfg(initial_latent, embeddings, guidance_scale,
                                                            scheduler_state, scheduler_config, denoiser_weights,
                                                            &attention_bias);
    const auto transformer_end = Clock::now();

    const auto vae_start = Clock::now();
    Tensor decoded_image = run_vae_decode(final_latents, vae_weights);
    const auto vae_end = Clock::now();

    const auto total_end = Clock::now();
    return PipelineRunResult{std::move(decoded_image), elapsed_ms(encoder_start, encoder_end),
                             elapsed_ms(transformer_start, transformer_end), elapsed_ms(vae_start, vae_end),
                             elapsed_ms(total_start, total_end)};
}

void print_run(const char* label, int index, const PipelineRunResult& r) {
    std::cout << label << " " << index << ": " << r.total_ms << " ms"
              << " (encoder=" << r.encoder_ms << " transformer=" << r.transformer_ms << " vae=" << r.vae_ms << ")\n"
              << std::flush;
}

}  // namespace

int main(int argc, char** argv) {
    int warmup = 0, iters = 1;
    bool small = false;
    std::vector<std::string> pos;
    for (int i = 1; i < argc; ++i) {
        if (std::strcmp(argv[i], "--small") == 0) small = true;
        else pos.push_back(argv[i]);
    }
    if (pos.size() >= 1) warmup = std::stoi(pos[0]);
    if (pos.size() >= 2) iters = std::stoi(pos[1]);
    if (warmup < 0) throw std::invalid_argument("warmup must be non-negative");
    if (iters <= 0) throw std::invalid_argument("iters must be positive");

    // Sana-0.6B at 1024 px (infer_main.cpp:366-374) or a small structure for a quick check
    const Dims d = small ? Dims{2, 128, 8, 64, 320, 4, 2, 16, 20, {64, 64, 128}, {true, true, false}, 1, 8}
                         : Dims{28, 1152, 32, 2304, 5760, 36, 16, 300, 324,
                                {128, 256, 512, 512, 1024, 1024}, {true, true, true, false, false, false}, 3, 32};
    const size_t num_steps = 20;
    const float guidance_scale = 4.5f;

    const auto weights_load_start = Clock::now();
    Fill fill;
    const SanaDenoiserWeights denoiser_weights = make_denoiser(d, fill);
    const SanaVaeWeights vae_weights = make_vae(d, fill);
    const Tensor negative_states = fill({d.L, d.Din}, 1.0f);
    const Tensor positive_states = fill({d.pos_rows, d.Din}, 1.0f);
    const auto weights_load_end = Clock::now();
    const double weights_load_ms = elapsed_ms(weights_load_start, weights_load_end);

    Tensor initial_latent({1, d.Cl, d.latent_hw, d.latent_hw});
    if (sana_randn_torch_cpu(initial_latent.data().data(), initial_latent.numel(), 42) != SANA_OK)
        throw std::runtime_error("randn_torch_cpu failed");
    const SanaSchedulerConfig scheduler_config = make_sana_scheduler_config();

    std::cout << "warming up full pipeline (" << warmup << " runs, " << num_steps << " steps each)\n" << std::flush;
    for (int i = 0; i < warmup; ++i)
        print_run("warmup", i + 1,
                  run_pipeline_once(d, negative_states, positive_states, guidance_scale, initial_latent, num_steps,
                                    scheduler_config, denoiser_weights, vae_weights));

    std::cout << "benchmarking full pipeline (" << iters << " runs)\n" << std::flush;
    double total_encoder_ms = 0.0, total_transformer_ms = 0.0, total_vae_ms = 0.0, total_total_ms = 0.0;
    bool finite = true;
    for (int i = 0; i < iters; ++i) {
        PipelineRunResult r = run_pipeline_once(d, negative_states, positive_states, guidance_scale, initial_latent,
                                                num_steps, scheduler_config, denoiser_weights, vae_weights);
        for (float v : r.decoded_image.data()) finite = finite && std::isfinite(v);
        total_encoder_ms += r.encoder_ms;
        total_transformer_ms += r.transformer_ms;
        total_vae_ms += r.vae_ms;
        total_total_ms += r.total_ms;
        print_run("run", i + 1, r);
    }

    const double count = static_cast<double>(iters);
    std::cout << "\n=== timing summary ===\n";
    std::cout << "weights_load_ms:    " << weights_load_ms << " (synthetic)\n";
    std::cout << "warmup_iters:       " << warmup << "\n";
    std::cout << "iters:              " << iters << "\n";
    std::cout << "total_ms:           " << total_total_ms << "\n";
    std::cout << "avg_ms:             " << (total_total_ms / count) << "\n";
    std::cout << "encoder_ms_avg:     " << (total_encoder_ms / count) << " (output contract only)\n";
    std::cout << "transformer_ms_avg: " << (total_transformer_ms / count) << " (" << num_steps << " steps)\n";
    std::cout << "vae_ms_avg:         " << (total_vae_ms / count) << "\n";
    std::cout << "image_finite:       " << (finite ? "yes" : "no") << "\n";
    return finite ? 0 : 1;
}
