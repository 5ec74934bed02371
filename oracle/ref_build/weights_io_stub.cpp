// Test infrastructure only (oracle side). Stands in for the three symbols of the
// reference's weights_io.cpp that transformer.cpp links against. The real file needs
// ggml (fetched over the network by the reference's CMake), which is absent here;
// the synthetic-weight harness builds SanaDenoiserWeights directly in memory, so the
// loaders are never called. Any call throws, so a path that reached them fails loudly.
//
// Declarations come from the reference's weights_io.h (weights_io.h:30-42).
#include "weights_io.h"

#include <stdexcept>

bool ends_with(const std::string & value, const std::string & suffix) {
    return value.size() >= suffix.size() &&
           value.compare(value.size() - suffix.size(), suffix.size(), suffix) == 0;
}

Tensor load_weight_tensor(
    const std::string &,
    const std::unordered_map<std::string, SavedWeightInfo> &,
    const std::string & name
) {
    throw std::runtime_error("oracle build has no weight files: " + name);
}

Tensor load_linear_weight_tensor(
    const std::string &,
    const std::unordered_map<std::string, SavedWeightInfo> &,
    const std::string & name
) {
    throw std::runtime_error("oracle build has no weight files: " + name);
}
