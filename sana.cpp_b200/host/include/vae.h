// The reference's VAE decoder API (cconthekeyboard/sana.cpp src/vae.h:11-92): the weight
// structs, with the same members in the same order so that weights built by the reference's
// own load_vae_weights pass straight through, and the decode entry points, implemented by
// host/vae_cuda.cpp over the C ABI of include/sana_cuda.h. The GGUF index helpers
// (find_vae_decoder_up_block_prefixes, load_vae_weights) stay the reference's own code and
// are not declared here.
#pragma once

#include <optional>
#include <vector>

#include "tensor.h"

struct SanaVaeResBlockWeights {
    Tensor conv1_weight;
    Tensor conv1_bias;
    Tensor conv2_weight;
    Tensor norm_weight;
    Tensor norm_bias;
};

struct SanaVaeAttentionWeights {
    Tensor to_q_weight_conv1x1;
    Tensor to_k_weight_conv1x1;
    Tensor to_v_weight_conv1x1;
    Tensor proj_in_weight;
    Tensor proj_out_weight;
    Tensor to_out_weight_conv1x1;
    Tensor norm_out_weight;
    Tensor norm_out_bias;
};

struct SanaVaeGlumbConvWeights {
    Tensor conv_inverted_weight;
    Tensor conv_inverted_bias;
    Tensor conv_depth_weight;
    Tensor conv_depth_bias;
    Tensor conv_point_weight;
    Tensor norm_weight;
    Tensor norm_bias;
};

struct SanaVaeAttnGlumbLayerWeights {
    SanaVaeAttentionWeights attention;
    SanaVaeGlumbConvWeights glumb;
};

struct SanaVaeUpBlockWeights {
    std::optional<Tensor> upsample_conv_weight;
    std::optional<Tensor> upsample_conv_bias;
    bool is_res_block = false;
    std::vector<SanaVaeResBlockWeights> res_blocks;
    std::vector<SanaVaeAttnGlumbLayerWeights> attn_glumb_layers;
};

struct SanaVaeDecoderWeights {
    Tensor conv_in_weight;
    Tensor conv_in_bias;
    Tensor norm_out_weight;
    Tensor norm_out_bias;
    Tensor conv_out_weight;
    Tensor conv_out_bias;
    std::vector<SanaVaeUpBlockWeights> up_blocks;
};

struct SanaVaeWeights {
    SanaVaeDecoderWeights decoder;
    float scaling_factor = 1.0f;
    size_t spatial_compression_ratio = 32;
};

// validate_vae_decoder_weights / validate_vae_weights (vae.cpp:172-208): std::invalid_argument
// with the reference's messages.
void validate_vae_decoder_weights(const SanaVaeDecoderWeights& weights);
void validate_vae_weights(const SanaVaeWeights& weights);

// run_vae_decode (vae.cpp:243-325) on the GPU: latents [B, latent, h, w] -> image
// [B, out, h * 2^u, w * 2^u], u = the number of upsampling up blocks.
Tensor run_vae_decode(const Tensor& latents, const SanaVaeWeights& weights);
