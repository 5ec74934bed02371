// Driver for tests/test_frontends.py: the weight loaders (transformer.h / vae.h), weights_io.h and
// the encoder contract of gemma_encoder.h, called the way the reference's front ends call them.
// Loaded tensors are written back as .npy for the test to compare with what it wrote; failures
// are printed as "<exception type>: <message>" and exit 0, so the test reads the error contract.
//
//   test_frontend denoiser <model.gguf> <caption.gguf> <denoiser.gguf> <self_heads> <cross_heads> <outdir>
//   test_frontend vae <vae.gguf> <outdir>
//   test_frontend npy_copy <in.npy> <out.npy>
//   test_frontend index_tensor <index path> <weights_dir> <name> <out.npy> [linear]
//   test_frontend prompt <prompt> <negative> <max_sequence_length> <gemma path> <outdir>
//   test_frontend select <in.npy> <keep> <out.npy>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <stdexcept>
#include <string>

#include "gemma_encoder.h"
#include "transformer.h"
#include "vae.h"
#include "weights_io.h"

namespace {

void save(const Tensor& t, const std::string& dir, const std::string& name) { save_npy_tensor(t, dir + "/" + name + ".npy"); }

int denoiser(char** a) {
    const std::string m = a[0], c = a[1], d = a[2], out = a[5];
    const SanaDenoiserWeights w = load_denoiser_weights(m, load_weight_index(m), c, load_weight_index(c), d,
                                                        load_weight_index(d), std::stoul(a[3]), std::stoul(a[4]));
    save(w.caption.linear_1_weight, out, "caption.linear_1_weight");
    save(w.caption.linear_1_bias, out, "caption.linear_1_bias");
    save(w.caption.linear_2_weight, out, "caption.linear_2_weight");
    save(w.caption.linear_2_bias, out, "caption.linear_2_bias");
    save(w.patch_embed_weight, out, "patch_embed_weight");
    save(w.patch_embed_bias, out, "patch_embed_bias");
    save(w.time_embed_linear_1_weight, out, "time_embed_linear_1_weight");
    save(w.time_embed_linear_1_bias, out, "time_embed_linear_1_bias");
    save(w.time_embed_linear_2_weight, out, "time_embed_linear_2_weight");
    save(w.time_embed_linear_2_bias, out, "time_embed_linear_2_bias");
    save(w.time_projection_weight, out, "time_projection_weight");
    save(w.time_projection_bias, out, "time_projection_bias");
    save(w.caption_norm_weight, out, "caption_norm_weight");
    save(w.final_scale_shift_table, out, "final_scale_shift_table");
    save(w.proj_out_weight, out, "proj_out_weight");
    save(w.proj_out_bias, out, "proj_out_bias");
    std::ofstream meta(out + "/meta.txt");
    meta << w.blocks.size() << "\n";
    for (size_t i = 0; i < w.blocks.size(); ++i) {
        const SanaBlockWeights& b = w.blocks[i];
        const std::string p = "blocks." + std::to_string(i) + ".";
        meta << b.self_num_heads << " " << b.cross_num_heads << "\n";
        const std::pair<const char*, const Tensor*> fields[] = {
            {"scale_shift_table", &b.scale_shift_table}, {"attn_norm_gamma", &b.attn_norm_gamma},
            {"attn_norm_beta", &b.attn_norm_beta},       {"q_weight", &b.q_weight},
            {"q_bias", &b.q_bias},                       {"k_weight", &b.k_weight},
            {"k_bias", &b.k_bias},                       {"v_weight", &b.v_weight},
            {"v_bias", &b.v_bias},                       {"out_weight", &b.out_weight},
            {"out_bias", &b.out_bias},                   {"cross_q_weight", &b.cross_q_weight},
            {"cross_q_bias", &b.cross_q_bias},           {"cross_k_weight", &b.cross_k_weight},
            {"cross_k_bias", &b.cross_k_bias},           {"cross_v_weight", &b.cross_v_weight},
            {"cross_v_bias", &b.cross_v_bias},           {"cross_out_weight", &b.cross_out_weight},
            {"cross_out_bias", &b.cross_out_bias},       {"mlp_norm_gamma", &b.mlp_norm_gamma},
            {"mlp_norm_beta", &b.mlp_norm_beta},         {"ff_inverted_weight", &b.ff_inverted_weight},
            {"ff_inverted_bias", &b.ff_inverted_bias},   {"ff_depth_weight", &b.ff_depth_weight},
            {"ff_depth_bias", &b.ff_depth_bias},         {"ff_point_weight", &b.ff_point_weight}};
        for (const auto& f : fields) save(*f.second, out, p + f.first);
    }
    return 0;
}

int vae(char** a) {
    const std::string path = a[0], out = a[1];
    const SanaVaeWeights w = load_vae_weights(path, load_weight_index(path), 0.41407f, 32);
    validate_vae_weights(w);
    const SanaVaeDecoderWeights& d = w.decoder;
    save(d.conv_in_weight, out, "conv_in_weight");
    save(d.conv_out_weight, out, "conv_out_weight");
    save(d.norm_out_bias, out, "norm_out_bias");
    std::ofstream meta(out + "/meta.txt");
    meta << d.up_blocks.size() << " " << w.scaling_factor << " " << w.spatial_compression_ratio << "\n";
    for (size_t i = 0; i < d.up_blocks.size(); ++i) {
        const SanaVaeUpBlockWeights& b = d.up_blocks[i];
        const std::string p = "up." + std::to_string(i) + ".";
        meta << (b.upsample_conv_weight ? 1 : 0) << " " << (b.is_res_block ? 1 : 0) << " " << b.res_blocks.size()
             << " " << b.attn_glumb_layers.size() << "\n";
        if (b.upsample_conv_weight) save(*b.upsample_conv_weight, out, p + "upsample_conv_weight");
        if (!b.res_blocks.empty()) save(b.res_blocks.back().conv2_weight, out, p + "last.conv2_weight");
        if (!b.attn_glumb_layers.empty()) {
            const SanaVaeAttnGlumbLayerWeights& l = b.attn_glumb_layers.back();
            save(l.attention.to_q_weight_conv1x1, out, p + "last.to_q_weight_conv1x1");
            save(l.attention.proj_in_weight, out, p + "last.proj_in_weight");
            save(l.glumb.conv_point_weight, out, p + "last.conv_point_weight");
        }
    }
    return 0;
}

int run(int argc, char** argv) {
    if (argc < 2) throw std::invalid_argument("no command");
    const std::string cmd = argv[1];
    char** a = argv + 2;
    const int n = argc - 2;
    if (cmd == "denoiser" && n == 6) return denoiser(a);
    if (cmd == "vae" && n == 2) return vae(a);
    if (cmd == "npy_copy" && n == 2) {
        save_npy_tensor(load_npy_tensor(a[0]), a[1]);
        return 0;
    }
    if (cmd == "index_tensor" && (n == 4 || n == 5)) {
        const auto index = load_weight_index(a[0]);
        const Tensor t = n == 5 ? load_linear_weight_tensor(a[1], index, a[2]) : load_weight_tensor(a[1], index, a[2]);
        save_npy_tensor(t, a[3]);
        return 0;
    }
    if (cmd == "prompt" && n == 5) {
        GemmaEncoderConfig config;
        config.gguf_path = a[3];
        GemmaEncoder encoder(config);
        const GemmaPromptPair pair = encode_prompt_pair(encoder, a[0], a[1], std::stoul(a[2]));
        save(pair.embeddings, a[4], "embeddings");
        save(pair.attention_bias, a[4], "bias");
        return 0;
    }
    if (cmd == "select" && n == 3) {
        save_npy_tensor(select_rows_first_and_last(load_npy_tensor(a[0]), std::stoul(a[1])), a[2]);
        return 0;
    }
    throw std::invalid_argument("unknown command or wrong argument count: " + cmd);
}

}  // namespace

int main(int argc, char** argv) {
    try {
        return run(argc, argv);
    } catch (const std::invalid_argument& e) {
        std::cout << "invalid_argument: " << e.what() << "\n";
    } catch (const std::runtime_error& e) {
        std::cout << "runtime_error: " << e.what() << "\n";
    }
    return 0;
}
