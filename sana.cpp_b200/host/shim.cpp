// The process-wide handle and the weight cache behind the reference API entry points.
#include "shim.h"

#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "sana_cuda_shim.h"
#include "transformer.h"

namespace sana_shim {
namespace {

std::mutex g_mu;
sana_cuda_ctx* g_ctx = nullptr;
int g_device = -1, g_mode = -1;  // -1: from the environment

// What the handle currently holds: the (address, size) of every tensor of the weights it was
// given, with their head counts; kind 1 = a SanaDenoiserWeights, 2 = a single block.
struct Key {
    int kind = 0;
    std::vector<std::pair<const void*, size_t>> t;
    bool operator==(const Key& o) const { return kind == o.kind && t == o.t; }
};
Key g_key;
unsigned g_epoch = 1;  // bumped whenever cached device weights may be stale (new handle, invalidate)

int env_int(const char* name, int def) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoi(v) : def;
}
int env_mode() {
    const char* v = std::getenv("SANA_CUDA_MODE");
    if (v && (std::strcmp(v, "f32") == 0 || std::strcmp(v, "fp32") == 0)) return SANA_MODE_F32;
    return SANA_MODE_BF16;
}

void add(Key& k, const Tensor& t) { k.t.emplace_back(t.numel() ? t.data().data() : nullptr, t.numel()); }

const Tensor* block_tensors(const SanaBlockWeights& b, int i) {
    const Tensor* all[26] = {&b.scale_shift_table, &b.attn_norm_gamma, &b.attn_norm_beta, &b.q_weight, &b.q_bias,
                             &b.k_weight, &b.k_bias, &b.v_weight, &b.v_bias, &b.out_weight, &b.out_bias,
                             &b.cross_q_weight, &b.cross_q_bias, &b.cross_k_weight, &b.cross_k_bias,
                             &b.cross_v_weight, &b.cross_v_bias, &b.cross_out_weight, &b.cross_out_bias,
                             &b.mlp_norm_gamma, &b.mlp_norm_beta, &b.ff_inverted_weight, &b.ff_inverted_bias,
                             &b.ff_depth_weight, &b.ff_depth_bias, &b.ff_point_weight};
    return all[i];
}

// Element counts of a block's tensors (reference layout), 0 where the tensor is optional.
void check_block(const SanaBlockWeights& b, size_t C, size_t E) {
    const size_t need[26] = {6 * C, C, C, C * C, C, C * C, C, C * C, C, C * C, C, C * C, C,
                             C * C, C, C * C, C, C * C, C, C, C, E * C, E, E * 9, E, C * (E / 2)};
    const bool optional[26] = {false, true, true, false, true, false, true, false, true, false, true, false, true,
                               false, true, false, true, false, true, true, true, false, true, false, true, false};
    for (int i = 0; i < 26; ++i) {
        const size_t n = block_tensors(b, i)->numel();
        if (n == need[i] || (optional[i] && n == 0)) continue;
        throw std::invalid_argument("block weight " + std::to_string(i) + " has " + std::to_string(n) +
                                    " elements, expected " + std::to_string(need[i]));
    }
    if (b.self_num_heads == 0 || C % b.self_num_heads != 0)
        throw std::invalid_argument("self attention hidden size must be divisible by self_num_heads");
    if (b.cross_num_heads == 0 || C % b.cross_num_heads != 0)
        throw std::invalid_argument("cross attention hidden size must be divisible by cross_num_heads");
}

void upload(const sana_dims& d, const std::vector<const float*>& model, const std::vector<const float*>& blocks) {
    check(sana_cuda_upload_weights(handle(), &d, model.data(), blocks.data(), SANA_LAYOUT_REFERENCE));
}

}  // namespace

sana_cuda_ctx* handle() {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_ctx) {
        const int device = g_device >= 0 ? g_device : env_int("SANA_CUDA_DEVICE", 0);
        const int m = g_mode >= 0 ? g_mode : env_mode();
        sana_cuda_ctx* c = nullptr;
        const int rc = sana_cuda_create(device, m, &c);
        if (rc != SANA_OK) {
            const std::string msg = c ? sana_cuda_last_error(c) : "sana_cuda_create failed";
            if (c) sana_cuda_destroy(c);
            throw std::runtime_error(msg);
        }
        g_ctx = c;
        g_mode = m;
        g_key = Key();
        ++g_epoch;
    }
    return g_ctx;
}

int mode() {
    handle();
    return g_mode;
}

unsigned weights_epoch() {
    std::lock_guard<std::mutex> lock(g_mu);
    return g_epoch;
}

void check(int rc) {
    if (rc == SANA_OK) return;
    const std::string msg = g_ctx ? sana_cuda_last_error(g_ctx) : "no CUDA handle";
    if (rc == SANA_ERR_INVALID) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

const float* ptr(const Tensor& t) { return t.numel() ? t.data().data() : nullptr; }
const float* opt(const Tensor* t) { return t ? ptr(*t) : nullptr; }

int as_int(size_t v, const char* what) {
    if (v > static_cast<size_t>(INT_MAX)) throw std::invalid_argument(std::string(what) + " is too large");
    return static_cast<int>(v);
}

void require(bool ok, const char* message) {
    if (!ok) throw std::invalid_argument(message);
}

void ensure_weights(const SanaDenoiserWeights& w) {
    require(!w.blocks.empty(), "denoiser weights have no blocks");
    Key k;
    k.kind = 1;
    for (const Tensor* t : {&w.caption.linear_1_weight, &w.caption.linear_1_bias, &w.caption.linear_2_weight,
                            &w.caption.linear_2_bias, &w.patch_embed_weight, &w.patch_embed_bias,
                            &w.time_embed_linear_1_weight, &w.time_embed_linear_1_bias,
                            &w.time_embed_linear_2_weight, &w.time_embed_linear_2_bias, &w.time_projection_weight,
                            &w.time_projection_bias, &w.caption_norm_weight, &w.final_scale_shift_table,
                            &w.proj_out_weight, &w.proj_out_bias})
        add(k, *t);
    for (const SanaBlockWeights& b : w.blocks) {
        for (int i = 0; i < 26; ++i) add(k, *block_tensors(b, i));
        k.t.emplace_back(nullptr, b.self_num_heads * 1000003u + b.cross_num_heads);
    }
    handle();
    if (g_key == k) return;

    const SanaBlockWeights& b0 = w.blocks[0];
    require(b0.scale_shift_table.rank() == 2 && b0.scale_shift_table.dim_size(0) == 6,
            "scale_shift_table must have shape {6, hidden}");
    require(w.patch_embed_weight.rank() == 4, "patch_embed_weight must be rank 4");
    require(w.caption.linear_1_weight.rank() == 2, "caption linear_1_weight must be rank 2");
    require(b0.ff_inverted_weight.rank() >= 1, "ff_inverted_weight must not be empty");
    const size_t C = b0.scale_shift_table.dim_size(1);
    const size_t Cl = w.patch_embed_weight.dim_size(1);
    const size_t Din = w.caption.linear_1_weight.dim_size(0);
    const size_t E = b0.ff_inverted_weight.dim_size(0);
    for (const SanaBlockWeights& b : w.blocks) {
        check_block(b, C, E);
        require(b.self_num_heads == b0.self_num_heads && b.cross_num_heads == b0.cross_num_heads,
                "all blocks must have the same head counts");
    }
    const size_t need[16] = {Din * C, C, C * C, C, C * Cl, C, 256 * C, C, C * C, C, C * 6 * C, 6 * C, C, 2 * C,
                             C * Cl, Cl};
    std::vector<const float*> model;
    for (size_t i = 0; i < 16; ++i) {
        const std::pair<const void*, size_t>& e = k.t[i];
        if (e.second != need[i])
            throw std::invalid_argument("denoiser weight " + std::to_string(i) + " has " + std::to_string(e.second) +
                                        " elements, expected " + std::to_string(need[i]));
        model.push_back(static_cast<const float*>(e.first));
    }
    std::vector<const float*> blocks;
    for (const SanaBlockWeights& b : w.blocks)
        for (int i = 0; i < 26; ++i) blocks.push_back(ptr(*block_tensors(b, i)));
    sana_dims d{as_int(w.blocks.size(), "block count"), as_int(C, "hidden size"), as_int(Cl, "latent channels"),
                as_int(Din, "caption dim"), as_int(E, "ff width"), as_int(b0.self_num_heads, "self heads"),
                as_int(b0.cross_num_heads, "cross heads")};
    g_key = Key();
    upload(d, model, blocks);
    g_key = k;
}

void ensure_block(const SanaBlockWeights& b) {
    Key k;
    k.kind = 2;
    for (int i = 0; i < 26; ++i) add(k, *block_tensors(b, i));
    k.t.emplace_back(nullptr, b.self_num_heads * 1000003u + b.cross_num_heads);
    handle();
    if (g_key == k) return;
    require(b.scale_shift_table.rank() == 2 && b.scale_shift_table.dim_size(0) == 6,
            "scale_shift_table must have shape {6, hidden}");
    require(b.ff_inverted_weight.rank() >= 1, "ff_inverted_weight must not be empty");
    const size_t C = b.scale_shift_table.dim_size(1), E = b.ff_inverted_weight.dim_size(0);
    check_block(b, C, E);
    // The model-level tensors are not used by block_forward; zeros of a one-channel model
    // stand in for them.
    static std::vector<float> zeros;
    const size_t need[16] = {C, C, C * C, C, C, C, 256 * C, C, C * C, C, 6 * C * C, 6 * C, C, 2 * C, C, 1};
    size_t most = 0;
    for (size_t n : need) most = n > most ? n : most;
    if (zeros.size() < most) zeros.assign(most, 0.0f);
    std::vector<const float*> model(16, zeros.data());
    std::vector<const float*> blocks;
    for (int i = 0; i < 26; ++i) blocks.push_back(ptr(*block_tensors(b, i)));
    sana_dims d{1, as_int(C, "hidden size"), 1, 1, as_int(E, "ff width"), as_int(b.self_num_heads, "self heads"),
                as_int(b.cross_num_heads, "cross heads")};
    g_key = Key();
    upload(d, model, blocks);
    g_key = k;
}

}  // namespace sana_shim

namespace sana_cuda_shim {

void configure(int device, int mode) {
    std::lock_guard<std::mutex> lock(sana_shim::g_mu);
    if (sana_shim::g_ctx) sana_cuda_destroy(sana_shim::g_ctx);
    sana_shim::g_ctx = nullptr;
    sana_shim::g_device = device;
    sana_shim::g_mode = mode;
    sana_shim::g_key = sana_shim::Key();
    ++sana_shim::g_epoch;
}

void invalidate_weights() {
    std::lock_guard<std::mutex> lock(sana_shim::g_mu);
    sana_shim::g_key = sana_shim::Key();
    ++sana_shim::g_epoch;
}

}  // namespace sana_cuda_shim
