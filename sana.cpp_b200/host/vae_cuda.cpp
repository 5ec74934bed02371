// run_vae_decode and the VAE validators (vae.h) over the C ABI: the SanaVaeWeights structure
// becomes a sana_vae_dims descriptor and a tensor table (include/sana_cuda.h's VAE order), kept
// uploaded while the caller passes the same tensors.
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "shim.h"
#include "vae.h"

namespace {

std::mutex g_vae_mu;
std::vector<std::pair<const void*, size_t>> g_vae_key;
unsigned g_vae_epoch = 0;

void need(bool ok, const char* message) {
    if (!ok) throw std::invalid_argument(message);
}

// Output channels of an up block: its upsample conv's, else its first layer's.
size_t block_channels(const SanaVaeUpBlockWeights& b) {
    if (b.upsample_conv_weight) return b.upsample_conv_weight->dim_size(0);
    if (b.is_res_block && !b.res_blocks.empty()) return b.res_blocks[0].conv1_weight.dim_size(0);
    if (!b.attn_glumb_layers.empty()) return b.attn_glumb_layers[0].attention.to_q_weight_conv1x1.dim_size(0);
    throw std::invalid_argument("vae up block has no layers");
}

}  // namespace

void validate_vae_decoder_weights(const SanaVaeDecoderWeights& w) {
    need(w.conv_in_weight.rank() == 4, "vae decoder conv_in.weight must be rank 4");
    need(w.conv_in_bias.rank() == 1, "vae decoder conv_in.bias must be rank 1");
    need(w.norm_out_weight.rank() == 1, "vae decoder norm_out.weight must be rank 1");
    need(w.norm_out_bias.rank() == 1, "vae decoder norm_out.bias must be rank 1");
    need(w.conv_out_weight.rank() == 4, "vae decoder conv_out.weight must be rank 4");
    need(w.conv_out_bias.rank() == 1, "vae decoder conv_out.bias must be rank 1");
    need(!w.up_blocks.empty(), "vae decoder must contain at least one up block");
    need(w.conv_in_weight.dim_size(0) == w.conv_in_bias.dim_size(0),
         "vae decoder conv_in bias shape must match output channels");
    need(w.norm_out_weight.dim_size(0) == w.norm_out_bias.dim_size(0), "vae decoder norm_out bias shape must match");
    need(w.conv_out_weight.dim_size(0) == w.conv_out_bias.dim_size(0),
         "vae decoder conv_out bias shape must match output channels");
    need(w.norm_out_weight.dim_size(0) == w.conv_out_weight.dim_size(1),
         "vae decoder norm_out channels must match conv_out input channels");
}

void validate_vae_weights(const SanaVaeWeights& w) {
    validate_vae_decoder_weights(w.decoder);
    need(w.scaling_factor > 0.0f, "vae scaling_factor must be positive");
    need(w.spatial_compression_ratio != 0, "vae spatial_compression_ratio must be positive");
}

Tensor run_vae_decode(const Tensor& latents, const SanaVaeWeights& weights) {
    using sana_shim::as_int;
    validate_vae_weights(weights);
    need(latents.rank() == 4, "vae decode latents must be rank 4");
    const SanaVaeDecoderWeights& d = weights.decoder;
    need(latents.dim_size(1) == d.conv_in_weight.dim_size(1), "vae decode latent channels must match decoder conv_in input");
    need(d.up_blocks.size() <= 8, "vae decoder has more than 8 up blocks");

    sana_vae_dims dims{};
    dims.latent_channels = as_int(d.conv_in_weight.dim_size(1), "latent channels");
    dims.out_channels = as_int(d.conv_out_weight.dim_size(0), "output channels");
    dims.n_blocks = as_int(d.up_blocks.size(), "up block count");
    dims.head_dim = 32;  // run_vae_decode's attention_head_dim (vae.cpp:292)
    dims.ms_kernel = 5;
    dims.scaling_factor = weights.scaling_factor;
    std::vector<const float*> table;
    std::vector<std::pair<const void*, size_t>> key;
    auto add = [&](const Tensor& t) {
        table.push_back(sana_shim::ptr(t));
        key.emplace_back(sana_shim::ptr(t), t.numel());
    };
    for (const Tensor* t : {&d.conv_in_weight, &d.conv_in_bias, &d.norm_out_weight, &d.norm_out_bias,
                            &d.conv_out_weight, &d.conv_out_bias})
        add(*t);
    for (size_t i = 0; i < d.up_blocks.size(); ++i) {
        const SanaVaeUpBlockWeights& b = d.up_blocks[i];
        sana_vae_block& db = dims.blocks[i];
        db.channels = as_int(block_channels(b), "block channels");
        db.has_upsample = b.upsample_conv_weight.has_value() ? 1 : 0;
        db.is_res_block = b.is_res_block ? 1 : 0;
        db.layers = as_int(b.is_res_block ? b.res_blocks.size() : b.attn_glumb_layers.size(), "layer count");
        if (db.has_upsample) {
            need(b.upsample_conv_bias.has_value(), "vae upsample conv has no bias");
            add(*b.upsample_conv_weight);
            add(*b.upsample_conv_bias);
        }
        if (b.is_res_block) {
            for (const SanaVaeResBlockWeights& r : b.res_blocks)
                for (const Tensor* t : {&r.conv1_weight, &r.conv1_bias, &r.conv2_weight, &r.norm_weight, &r.norm_bias})
                    add(*t);
        } else {
            for (const SanaVaeAttnGlumbLayerWeights& l : b.attn_glumb_layers) {
                const SanaVaeAttentionWeights& a = l.attention;
                const SanaVaeGlumbConvWeights& g = l.glumb;
                need(a.proj_in_weight.rank() == 4, "vae attention proj_in.weight must be rank 4");
                dims.ms_kernel = as_int(a.proj_in_weight.dim_size(2), "multiscale kernel");
                for (const Tensor* t : {&a.to_q_weight_conv1x1, &a.to_k_weight_conv1x1, &a.to_v_weight_conv1x1,
                                        &a.proj_in_weight, &a.proj_out_weight, &a.to_out_weight_conv1x1,
                                        &a.norm_out_weight, &a.norm_out_bias, &g.conv_inverted_weight,
                                        &g.conv_inverted_bias, &g.conv_depth_weight, &g.conv_depth_bias,
                                        &g.conv_point_weight, &g.norm_weight, &g.norm_bias})
                    add(*t);
            }
        }
    }
    key.emplace_back(nullptr, static_cast<size_t>(dims.ms_kernel) * 1000003u +
                                  static_cast<size_t>(weights.scaling_factor * 1e6f));

    sana_cuda_ctx* h = sana_shim::handle();
    {
        std::lock_guard<std::mutex> lock(g_vae_mu);
        const unsigned epoch = sana_shim::weights_epoch();
        if (key != g_vae_key || epoch != g_vae_epoch) {
            g_vae_key.clear();
            sana_shim::check(sana_cuda_vae_upload(h, &dims, table.data()));
            g_vae_key = key;
            g_vae_epoch = epoch;
        }
    }
    const size_t up = size_t{1} << (dims.n_blocks - 1);
    const int B = as_int(latents.dim_size(0), "batch"), lh = as_int(latents.dim_size(2), "latent height"),
              lw = as_int(latents.dim_size(3), "latent width");
    Tensor out({latents.dim_size(0), d.conv_out_weight.dim_size(0), latents.dim_size(2) * up, latents.dim_size(3) * up});
    sana_shim::check(sana_cuda_vae_decode(h, latents.data().data(), B, lh, lw, out.data().data()));
    return out;
}
