// The reference's text-encoder API (cconthekeyboard/sana.cpp src/gemma_encoder.h:1-48) with the
// same names and signatures, so that its front ends compile unchanged. The reference runs
// Gemma-2-2B through llama.cpp, which this host layer does not carry: host/frontend/
// gemma_encoder_stub.cpp keeps the contract around the encoder (the padded token counts, the
// positive branch's first-and-last-rows slice, negative-first batch order and the
// (1 - mask) * -10000 bias, through sana_prompt_pair_assemble) and replaces the hidden states
// with seeded synthetic ones of Gemma-2-2B's width (2304). Its timings say nothing about a text
// encoder.
#pragma once

#include <cstdint>
#include <memory>
#include <string>

#include "tensor.h"

struct GemmaEncoderConfig {
    std::string gguf_path;
    size_t max_sequence_length = 300;
    int32_t n_threads = 4;
};

struct GemmaEncoder {
    explicit GemmaEncoder(const GemmaEncoderConfig& config);
    ~GemmaEncoder();
    GemmaEncoder(const GemmaEncoder&) = delete;
    GemmaEncoder& operator=(const GemmaEncoder&) = delete;

    struct Impl;
    std::unique_ptr<Impl> impl;
};

// Negative prompt first, then positive.
struct GemmaPromptPair {
    Tensor embeddings;      // [2, max_sequence_length, hidden]
    Tensor attention_bias;  // [2, 1, max_sequence_length], (1 - mask) * -10000
};

GemmaPromptPair encode_prompt_pair(GemmaEncoder& encoder, const std::string& prompt, const std::string& negative_prompt,
                                   size_t max_sequence_length = 300);

// Row 0 of a rank-2 tensor followed by its last keep-1 rows.
Tensor select_rows_first_and_last(const Tensor& input, size_t keep);
