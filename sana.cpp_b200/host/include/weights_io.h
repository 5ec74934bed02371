// The reference's weight-file API (cconthekeyboard/sana.cpp src/weights_io.h:1-56), declared with
// the same names, members and signatures so that its front ends (src/infer_main.cpp,
// tests/bench_full_pipeline.cpp) compile unchanged against this host layer. Implemented by
// host/frontend/weights_io.cpp: GGUF files are indexed through the C ABI's sana_gguf_* reader
// (no ggml), the legacy npy + JSON index by its own parser.
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

#include "tensor.h"

struct TensorComparison {
    float max_abs_diff;
    float mean_abs_diff;
};

enum class WeightFormat {
    Npy,
    Gguf,
};

struct SavedWeightInfo {
    std::string file;  // npy: file name inside the weights directory; gguf: the .gguf path
    std::vector<size_t> shape;
    std::string dtype;
    WeightFormat format = WeightFormat::Npy;
    size_t offset = 0;  // gguf: file offset of the tensor's data
};

bool ends_with(const std::string& value, const std::string& suffix);

// ".gguf" paths: every tensor of the file (weights_io.cpp:134-164); anything else: the JSON
// index {"name": {"file": ..., "shape": [...], "dtype": ...}, ...} (weights_io.cpp:171-322).
std::unordered_map<std::string, SavedWeightInfo> load_weight_index(const std::string& path);
Tensor load_weight_tensor(const std::string& weights_dir, const std::unordered_map<std::string, SavedWeightInfo>& index,
                          const std::string& name);
// load_weight_tensor of a rank-2 [out, in] weight, returned transposed to [in, out].
Tensor load_linear_weight_tensor(const std::string& weights_dir,
                                 const std::unordered_map<std::string, SavedWeightInfo>& index,
                                 const std::string& name);
Tensor load_npy_tensor(const std::string& path);
void save_npy_tensor(const Tensor& tensor, const std::string& path);
TensorComparison compare_tensor_to_reference(const Tensor& actual, const std::string& path);
Tensor slice_batch_3d(const Tensor& input, size_t batch_index);
TensorComparison compare_batch_slice_to_reference(const Tensor& actual, const std::string& path, size_t batch_index);
TensorComparison compare_block_output_to_reference(const Tensor& actual, const std::string& path, size_t batch_index);
