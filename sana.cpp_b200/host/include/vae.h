// The reference's VAE decoder API (cconthekeyboard/sana.cpp src/vae.h:11-92): the weight
// structs, with the same members in the same order so that weights built by the reference's
// own load_vae_weights pass straight through, and the decode entry points, implemented by
// host/vae_cuda.cpp over the C ABI of include/sana_cuda.h, and the loaders
// (find_vae_decoder_up_block_prefixes, load_vae_weights), implemented by host/loaders.cpp on
// top of weights_io.h.
#pragma once

#include <optional>
#include <string>
#include <unordered_map>
#include <vector>

#include "tensor.h"
#include "weights_io.h"

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

// "decoder.up_blocks.<i>" prefixes ordered by i (vae.cpp:88-136).
std::vector<std::string> find_vae_decoder_up_block_prefixes(
    const std::unordered_map<std::string, SavedWeightInfo>& index);
// vae.cpp:12-86, 138-160: an up block has an upsample conv when "<prefix>.0.conv.weight"
// exists, then three layers; it holds ResBlocks only when it has the upsample conv and its
// first layer has conv1 (otherwise attention + GLUMBConv layers); attention linear weights
// become [out, in, 1, 1].
SanaVaeWeights load_vae_weights(const std::string& weights_dir,
                                const std::unordered_map<std::string, SavedWeightInfo>& index, float scaling_factor,
                                size_t spatial_compression_ratio);

// validate_vae_decoder_weights / validate_vae_weights (vae.cpp:172-208): std::invalid_argument
// with the reference's messages.
void validate_vae_decoder_weights(const SanaVaeDecoderWeights& weights);
void validate_vae_weights(const SanaVaeWeights& weights);

// run_vae_decode (vae.cpp:243-325) on the GPU: latents [B, latent, h, w] -> image
// [B, out, h * 2^u, w * 2^u], u = the number of upsampling up blocks.
Tensor run_vae_decode(const Tensor& latents, const SanaVaeWeights& weights);
