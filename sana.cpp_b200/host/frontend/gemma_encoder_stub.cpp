// gemma_encoder.h without a text encoder. The reference encodes prompts with Gemma-2-2B through
// llama.cpp (gemma_encoder.cpp:79-150); this host layer carries neither, so the hidden states
// here are synthetic. What stays the reference's is the contract around the encoder
// (gemma_encoder.cpp:156-244), which is what the denoiser sees:
//   * the positive prompt is encoded behind an instruction prefix, padded to
//     prefix_tokens + max_sequence_length - 2 rows, then cut to row 0 plus the last
//     max_sequence_length - 1 rows; the negative prompt is padded to max_sequence_length;
//   * a text longer than its padded length is refused (no truncation);
//   * embeddings [2, L, hidden] negative first, bias [2, 1, L] = (1 - mask) * -10000 over the
//     real tokens that survive the cut (sana_prompt_pair_assemble).
// Stand-ins: a token is the beginning-of-sequence id, then one id per whitespace-separated
// word (an FNV-1a hash of the word); the instruction prefix is 24 tokens (the beginning id and
// 23 fixed ids); the hidden states of a padded sequence are torch.randn(rows, 2304) seeded with
// an FNV-1a hash of its token ids, so equal prompts give equal states.
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "gemma_encoder.h"
#include "sana_cuda.h"

struct GemmaEncoder::Impl {
    std::string gguf_path;
    size_t hidden = 2304;  // Gemma-2-2B's embedding width, the caption projection's input
};

GemmaEncoder::GemmaEncoder(const GemmaEncoderConfig& config) : impl(std::make_unique<Impl>()) {
    // the reference fails here when the model file cannot be loaded (gemma_encoder.cpp:90-94)
    if (!std::ifstream(config.gguf_path, std::ios::binary))
        throw std::runtime_error("failed to load Gemma-2 GGUF: " + config.gguf_path);
    impl->gguf_path = config.gguf_path;
}

GemmaEncoder::~GemmaEncoder() = default;

namespace {

constexpr int32_t kBeginId = 2;
constexpr int32_t kPadId = 0;
constexpr size_t kPrefixTokens = 24;

uint64_t fnv1a(const void* data, size_t n, uint64_t h = 1469598103934665603ull) {
    const unsigned char* p = static_cast<const unsigned char*>(data);
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
}

std::vector<int32_t> tokens_of(const std::string& text, bool with_prefix) {
    std::vector<int32_t> ids{kBeginId};
    if (with_prefix)
        for (size_t i = 1; i < kPrefixTokens; ++i) ids.push_back(static_cast<int32_t>(100 + i));
    std::istringstream words(text);
    std::string w;
    while (words >> w) ids.push_back(static_cast<int32_t>(1000 + fnv1a(w.data(), w.size()) % 200000));
    return ids;
}

// Pads with kPadId to `length`; returns the real-token count.
size_t pad_to(std::vector<int32_t>& ids, size_t length) {
    const size_t real = ids.size();
    if (real > length) throw std::invalid_argument("tokenized text exceeds padded_length; truncation not implemented");
    ids.resize(length, kPadId);
    return real;
}

std::vector<float> hidden_states(const std::vector<int32_t>& ids, size_t hidden) {
    std::vector<float> out(ids.size() * hidden);
    if (sana_randn_torch_cpu(out.data(), out.size(), fnv1a(ids.data(), ids.size() * sizeof(int32_t))) != SANA_OK)
        throw std::runtime_error("synthetic hidden states failed");
    return out;
}

}  // namespace

GemmaPromptPair encode_prompt_pair(GemmaEncoder& encoder, const std::string& prompt, const std::string& negative_prompt,
                                   size_t max_sequence_length) {
    const size_t hidden = encoder.impl->hidden;
    const size_t L = max_sequence_length;
    const size_t positive_rows = kPrefixTokens + L - 2;

    // positive branch first, as the reference orders its failures
    std::vector<int32_t> pos = tokens_of(prompt, true);
    const size_t pos_real = pad_to(pos, positive_rows);
    const std::vector<float> pos_states = hidden_states(pos, hidden);
    if (L == 0 || L > positive_rows)
        throw std::invalid_argument("select_rows_first_and_last: keep must be in (0, rows]");
    std::vector<int32_t> neg = tokens_of(negative_prompt, false);
    const size_t neg_real = pad_to(neg, L);
    const std::vector<float> neg_states = hidden_states(neg, hidden);

    GemmaPromptPair pair{Tensor({2, L, hidden}), Tensor({2, 1, L})};
    char err[256] = {0};
    const int rc = sana_prompt_pair_assemble(neg_states.data(), L, neg_real, pos_states.data(), positive_rows, pos_real,
                                             hidden, L, pair.embeddings.data().data(),
                                             pair.attention_bias.data().data(), err, sizeof err);
    if (rc == SANA_ERR_INVALID) throw std::invalid_argument(err);
    if (rc != SANA_OK) throw std::runtime_error(err[0] ? err : "sana_prompt_pair_assemble failed");
    return pair;
}

Tensor select_rows_first_and_last(const Tensor& input, size_t keep) {
    if (input.rank() != 2) throw std::invalid_argument("select_rows_first_and_last expects a rank-2 tensor");
    Tensor out({keep, input.dim_size(1)});
    char err[256] = {0};
    const int rc = sana_select_rows_first_and_last(input.data().data(), input.dim_size(0), input.dim_size(1), keep,
                                                   out.data().data(), err, sizeof err);
    if (rc == SANA_ERR_INVALID) throw std::invalid_argument(err);
    if (rc != SANA_OK) throw std::runtime_error("select_rows_first_and_last failed");
    return out;
}
