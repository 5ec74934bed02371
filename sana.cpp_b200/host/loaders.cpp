// The weight loaders and validators of transformer.h and vae.h: the reference's
// load_*_weights / find_*_prefixes / validate_* (transformer.cpp:166-488, 780-881;
// vae.cpp:12-160), which build the host weight structs from a weight index by the tensors'
// diffusers names. The names, the block discovery rules, the checks and their messages are
// the reference's (the file formats and the front ends depend on them); reading goes through
// weights_io.h.
#include <algorithm>
#include <map>
#include <set>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "transformer.h"
#include "vae.h"

namespace {

using Index = std::unordered_map<std::string, SavedWeightInfo>;

// "<prefix>.<suffix>", or the bare suffix for an empty prefix (transformer.cpp:26-31).
std::string joined(const std::string& prefix, const std::string& suffix) {
    return prefix.empty() ? suffix : prefix + "." + suffix;
}

bool all_digits(const std::string& s) {
    return !s.empty() && std::all_of(s.begin(), s.end(), [](char c) { return c >= '0' && c <= '9'; });
}

// "stem.<digits>" -> (stem, value); false when the text after the last dot is not a number
// (transformer.cpp:33-56).
bool trailing_index(const std::string& prefix, std::string* stem, size_t* value) {
    const size_t dot = prefix.rfind('.');
    if (dot == std::string::npos || !all_digits(prefix.substr(dot + 1))) return false;
    *stem = prefix.substr(0, dot);
    *value = static_cast<size_t>(std::stoull(prefix.substr(dot + 1)));
    return true;
}

void fail_if(bool bad, const char* message) {
    if (bad) throw std::runtime_error(message);
}

void invalid_if(bool bad, const char* message) {
    if (bad) throw std::invalid_argument(message);
}

Tensor filled(size_t n, float value) {
    Tensor t({n});
    t.fill(value);
    return t;
}

// A [out, in] linear weight as the [out, in, 1, 1] conv weight of the VAE's attention
// (linear_weight_to_conv1x1, vae_ops.cpp:592-599).
Tensor as_conv1x1(const Tensor& w) {
    invalid_if(w.rank() != 2, "linear_weight_to_conv1x1 expects rank-2 weight");
    Tensor out({w.dim_size(0), w.dim_size(1), 1, 1});
    out.data() = w.data();
    return out;
}

}  // namespace

SanaCaptionWeights load_caption_weights(const std::string& dir, const Index& index) {
    return SanaCaptionWeights{
        load_linear_weight_tensor(dir, index, "caption_projection.linear_1.weight"),
        load_weight_tensor(dir, index, "caption_projection.linear_1.bias"),
        load_linear_weight_tensor(dir, index, "caption_projection.linear_2.weight"),
        load_weight_tensor(dir, index, "caption_projection.linear_2.bias"),
    };
}

SanaBlockWeights load_block_weights(const std::string& dir, const Index& index, const std::string& prefix,
                                    size_t self_num_heads, size_t cross_num_heads) {
    invalid_if(self_num_heads == 0, "self_num_heads must be greater than 0");
    invalid_if(cross_num_heads == 0, "cross_num_heads must be greater than 0");
    auto plain = [&](const char* suffix) { return load_weight_tensor(dir, index, joined(prefix, suffix)); };
    auto linear = [&](const char* suffix) { return load_linear_weight_tensor(dir, index, joined(prefix, suffix)); };

    Tensor table = plain("scale_shift_table");
    Tensor q = linear("attn1.to_q.weight"), k = linear("attn1.to_k.weight"), v = linear("attn1.to_v.weight");
    Tensor o = linear("attn1.to_out.0.weight"), ob = plain("attn1.to_out.0.bias");
    Tensor cq = linear("attn2.to_q.weight"), cqb = plain("attn2.to_q.bias");
    Tensor ck = linear("attn2.to_k.weight"), ckb = plain("attn2.to_k.bias");
    Tensor cv = linear("attn2.to_v.weight"), cvb = plain("attn2.to_v.bias");
    Tensor co = linear("attn2.to_out.0.weight"), cob = plain("attn2.to_out.0.bias");
    Tensor fi = plain("ff.conv_inverted.weight"), fib = plain("ff.conv_inverted.bias");
    Tensor fd = plain("ff.conv_depth.weight"), fdb = plain("ff.conv_depth.bias");
    Tensor fp = plain("ff.conv_point.weight");

    // transformer.cpp:317-376, in the reference's order
    fail_if(table.rank() != 2 || table.dim_size(0) != 6, "scale_shift_table must have shape {6, hidden}");
    fail_if(q.rank() != 2 || k.rank() != 2 || v.rank() != 2 || o.rank() != 2, "attn1 projection weights must be rank 2");
    fail_if(ob.rank() != 1, "attn1 output bias must be rank 1");
    fail_if(cq.rank() != 2 || ck.rank() != 2 || cv.rank() != 2 || co.rank() != 2,
            "attn2 projection weights must be rank 2");
    fail_if(cqb.rank() != 1 || ckb.rank() != 1 || cvb.rank() != 1 || cob.rank() != 1, "attn2 biases must be rank 1");
    fail_if(fi.rank() != 4 || fd.rank() != 4 || fp.rank() != 4, "ff conv weights must be rank 4");
    fail_if(fib.rank() != 1 || fdb.rank() != 1, "ff conv biases must be rank 1");
    const size_t hidden = q.dim_size(1);
    fail_if(table.dim_size(1) != hidden, "scale_shift_table hidden size must match attention hidden size");
    fail_if(hidden % self_num_heads != 0, "self attention hidden size must be divisible by self_num_heads");
    fail_if(hidden % cross_num_heads != 0, "cross attention hidden size must be divisible by cross_num_heads");
    fail_if(cq.dim_size(1) != hidden || co.dim_size(0) != hidden, "attn2 hidden size must match block hidden size");
    fail_if(cqb.dim_size(0) != hidden || cob.dim_size(0) != hidden,
            "attn2 q/out bias size must match block hidden size");
    fail_if(fi.dim_size(1) != hidden || fp.dim_size(0) != hidden, "ff hidden size must match block hidden size");
    const size_t expanded = fi.dim_size(0);
    fail_if(fib.dim_size(0) != expanded || fd.dim_size(0) != expanded || fdb.dim_size(0) != expanded,
            "ff expanded channel sizes must match");
    fail_if(fp.dim_size(1) * 2 != expanded, "ff point conv input channels must match split GLUMB width");

    // The checkpoints carry no self-attention q/k/v biases and no norm affines: zeros and
    // ones (transformer.cpp:377-412).
    const Tensor zeros = filled(hidden, 0.0f), ones = filled(hidden, 1.0f);
    return SanaBlockWeights{table, ones, zeros, q,   zeros, k,   zeros, v,   zeros, o,    ob,   cq, cqb, ck, ckb,
                            cv,    cvb,  co,    cob, ones,  zeros, fi, fib, fd,  fdb, fp, self_num_heads,
                            cross_num_heads};
}

std::vector<std::string> find_block_prefixes(const Index& index) {
    const std::string suffix = ".scale_shift_table";
    std::set<std::string> found;
    for (const auto& entry : index)
        if (ends_with(entry.first, suffix)) found.insert(entry.first.substr(0, entry.first.size() - suffix.size()));
    std::vector<std::string> prefixes(found.begin(), found.end());
    // numeric order among "<stem>.<n>" of one stem, text order otherwise (transformer.cpp:414-437)
    std::sort(prefixes.begin(), prefixes.end(), [](const std::string& a, const std::string& b) {
        std::string sa, sb;
        size_t ia = 0, ib = 0;
        if (trailing_index(a, &sa, &ia) && trailing_index(b, &sb, &ib) && sa == sb) return ia < ib;
        return a < b;
    });
    return prefixes;
}

std::vector<SanaBlockWeights> load_model_block_weights(const std::string& dir, const Index& index,
                                                       size_t self_num_heads, size_t cross_num_heads) {
    const std::vector<std::string> prefixes = find_block_prefixes(index);
    invalid_if(prefixes.empty(), "weight index does not contain any prefixed model blocks");
    std::vector<SanaBlockWeights> blocks;
    blocks.reserve(prefixes.size());
    for (const std::string& p : prefixes)
        blocks.push_back(load_block_weights(dir, index, p, self_num_heads, cross_num_heads));
    return blocks;
}

SanaDenoiserWeights load_denoiser_weights(const std::string& block_dir, const Index& block_index,
                                          const std::string& caption_dir, const Index& caption_index,
                                          const std::string& denoiser_dir, const Index& denoiser_index,
                                          size_t self_num_heads, size_t cross_num_heads) {
    SanaCaptionWeights caption = load_caption_weights(caption_dir, caption_index);
    std::vector<SanaBlockWeights> blocks =
        load_model_block_weights(block_dir, block_index, self_num_heads, cross_num_heads);
    auto plain = [&](const char* name) { return load_weight_tensor(denoiser_dir, denoiser_index, name); };
    auto linear = [&](const char* name) { return load_linear_weight_tensor(denoiser_dir, denoiser_index, name); };
    SanaDenoiserWeights w{
        std::move(caption),
        std::move(blocks),
        plain("patch_embed.proj.weight"),
        plain("patch_embed.proj.bias"),
        linear("time_embed.emb.timestep_embedder.linear_1.weight"),
        plain("time_embed.emb.timestep_embedder.linear_1.bias"),
        linear("time_embed.emb.timestep_embedder.linear_2.weight"),
        plain("time_embed.emb.timestep_embedder.linear_2.bias"),
        linear("time_embed.linear.weight"),
        plain("time_embed.linear.bias"),
        plain("caption_norm.weight"),
        plain("scale_shift_table"),
        linear("proj_out.weight"),
        plain("proj_out.bias"),
    };
    validate_denoiser_weights(w);
    return w;
}

void validate_model_block_sequence(const std::vector<SanaBlockWeights>& blocks) {
    invalid_if(blocks.empty(), "model must contain at least one block");
    const size_t hidden = blocks[0].scale_shift_table.dim_size(1);
    for (const SanaBlockWeights& b : blocks) {
        invalid_if(b.scale_shift_table.rank() != 2 || b.scale_shift_table.dim_size(0) != 6,
                   "each block scale_shift_table must have shape {6, hidden}");
        invalid_if(b.scale_shift_table.dim_size(1) != hidden, "all model blocks must use the same hidden size");
        invalid_if(b.q_weight.rank() != 2 || b.q_weight.dim_size(0) != hidden || b.q_weight.dim_size(1) != hidden,
                   "each block q_weight must have shape {hidden, hidden}");
        invalid_if(b.cross_out_bias.rank() != 1 || b.cross_out_bias.dim_size(0) != hidden,
                   "each block cross_out_bias must match hidden size");
        invalid_if(b.ff_point_weight.rank() != 4 || b.ff_point_weight.dim_size(0) != hidden,
                   "each block ff_point_weight output channels must match hidden size");
    }
}

void validate_denoiser_weights(const SanaDenoiserWeights& w) {
    validate_model_block_sequence(w.blocks);
    const SanaCaptionWeights& c = w.caption;
    invalid_if(c.linear_1_weight.rank() != 2 || c.linear_2_weight.rank() != 2 || c.linear_1_bias.rank() != 1 ||
                   c.linear_2_bias.rank() != 1,
               "caption weights must use expected linear tensor ranks");
    invalid_if(c.linear_1_weight.dim_size(1) != c.linear_1_bias.dim_size(0) ||
                   c.linear_2_weight.dim_size(0) != c.linear_2_bias.dim_size(0),
               "caption weight dimensions must be internally consistent");
    const size_t hidden = w.blocks[0].scale_shift_table.dim_size(1);
    invalid_if(c.linear_2_weight.dim_size(1) != hidden, "caption output hidden size must match model block hidden size");

    auto shape_is = [](const Tensor& t, std::vector<size_t> want) { return t.shape() == want; };
    const size_t latent = w.patch_embed_weight.dim_size(1);
    invalid_if(!shape_is(w.patch_embed_weight, {hidden, latent, 1, 1}),
               "patch_embed_weight must have shape {hidden, latent_channels, 1, 1}");
    invalid_if(!shape_is(w.patch_embed_bias, {hidden}), "patch_embed_bias must match hidden size");
    invalid_if(!shape_is(w.time_embed_linear_1_weight, {256, hidden}),
               "time_embed_linear_1_weight must have shape {256, hidden}");
    invalid_if(!shape_is(w.time_embed_linear_1_bias, {hidden}), "time_embed_linear_1_bias must match hidden size");
    invalid_if(!shape_is(w.time_embed_linear_2_weight, {hidden, hidden}),
               "time_embed_linear_2_weight must have shape {hidden, hidden}");
    invalid_if(!shape_is(w.time_embed_linear_2_bias, {hidden}), "time_embed_linear_2_bias must match hidden size");
    invalid_if(!shape_is(w.time_projection_weight, {hidden, 6 * hidden}),
               "time_projection_weight must have shape {hidden, 6 * hidden}");
    invalid_if(!shape_is(w.time_projection_bias, {6 * hidden}), "time_projection_bias must match 6 * hidden");
    invalid_if(!shape_is(w.caption_norm_weight, {hidden}), "caption_norm_weight must match hidden size");
    invalid_if(!shape_is(w.final_scale_shift_table, {2, hidden}),
               "final_scale_shift_table must have shape {2, hidden}");
    invalid_if(!shape_is(w.proj_out_weight, {hidden, latent}), "proj_out_weight must have shape {hidden, latent_channels}");
    invalid_if(!shape_is(w.proj_out_bias, {latent}), "proj_out_bias must match latent channel count");
}

std::vector<std::string> find_vae_decoder_up_block_prefixes(const Index& index) {
    const std::string head = "decoder.up_blocks.";
    std::map<size_t, std::string> ordered;
    for (const auto& entry : index) {
        const std::string& name = entry.first;
        if (name.compare(0, head.size(), head) != 0) continue;
        const size_t dot = name.find('.', head.size());
        if (dot == std::string::npos) continue;
        const std::string number = name.substr(head.size(), dot - head.size());
        if (!all_digits(number)) continue;
        ordered.emplace(static_cast<size_t>(std::stoull(number)), head + number);
    }
    std::vector<std::string> prefixes;
    for (const auto& entry : ordered) prefixes.push_back(entry.second);
    return prefixes;
}

namespace {

SanaVaeUpBlockWeights load_up_block(const std::string& dir, const Index& index, const std::string& prefix) {
    auto t = [&](const std::string& name) { return load_weight_tensor(dir, index, name); };
    SanaVaeUpBlockWeights block;
    const bool upsample = index.count(prefix + ".0.conv.weight") != 0;
    const size_t first = upsample ? 1 : 0;
    if (upsample) {
        block.upsample_conv_weight = t(prefix + ".0.conv.weight");
        block.upsample_conv_bias = t(prefix + ".0.conv.bias");
        block.is_res_block = index.count(prefix + "." + std::to_string(first) + ".conv1.weight") != 0;
    }
    for (size_t layer = first; layer < first + 3; ++layer) {
        const std::string p = prefix + "." + std::to_string(layer);
        if (block.is_res_block) {
            block.res_blocks.push_back(SanaVaeResBlockWeights{t(p + ".conv1.weight"), t(p + ".conv1.bias"),
                                                              t(p + ".conv2.weight"), t(p + ".norm.weight"),
                                                              t(p + ".norm.bias")});
            continue;
        }
        SanaVaeAttentionWeights attn{as_conv1x1(t(p + ".attn.to_q.weight")),
                                     as_conv1x1(t(p + ".attn.to_k.weight")),
                                     as_conv1x1(t(p + ".attn.to_v.weight")),
                                     t(p + ".attn.to_qkv_multiscale.0.proj_in.weight"),
                                     t(p + ".attn.to_qkv_multiscale.0.proj_out.weight"),
                                     as_conv1x1(t(p + ".attn.to_out.weight")),
                                     t(p + ".attn.norm_out.weight"),
                                     t(p + ".attn.norm_out.bias")};
        SanaVaeGlumbConvWeights glumb{t(p + ".conv_out.conv_inverted.weight"), t(p + ".conv_out.conv_inverted.bias"),
                                      t(p + ".conv_out.conv_depth.weight"),    t(p + ".conv_out.conv_depth.bias"),
                                      t(p + ".conv_out.conv_point.weight"),    t(p + ".conv_out.norm.weight"),
                                      t(p + ".conv_out.norm.bias")};
        block.attn_glumb_layers.push_back(SanaVaeAttnGlumbLayerWeights{std::move(attn), std::move(glumb)});
    }
    return block;
}

}  // namespace

SanaVaeWeights load_vae_weights(const std::string& dir, const Index& index, float scaling_factor,
                                size_t spatial_compression_ratio) {
    auto t = [&](const char* name) { return load_weight_tensor(dir, index, name); };
    SanaVaeDecoderWeights decoder{t("decoder.conv_in.weight"),  t("decoder.conv_in.bias"),
                                  t("decoder.norm_out.weight"), t("decoder.norm_out.bias"),
                                  t("decoder.conv_out.weight"), t("decoder.conv_out.bias"),
                                  {}};
    for (const std::string& prefix : find_vae_decoder_up_block_prefixes(index))
        decoder.up_blocks.push_back(load_up_block(dir, index, prefix));
    return SanaVaeWeights{std::move(decoder), scaling_factor, spatial_compression_ratio};
}
