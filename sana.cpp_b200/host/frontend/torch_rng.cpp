// torch_rng.h over the C ABI's sana_randn_torch_cpu (the reference's torch_rng.cpp:35-68
// restated in csrc and pinned to torch's own output).
#include <stdexcept>

#include "sana_cuda.h"
#include "torch_rng.h"

Tensor randn_torch_cpu(const std::vector<size_t>& shape, uint64_t seed) {
    Tensor t(shape);
    if (t.numel() < 16) throw std::invalid_argument("randn_torch_cpu requires at least 16 elements");
    if (sana_randn_torch_cpu(t.data().data(), t.numel(), seed) != SANA_OK)
        throw std::runtime_error("randn_torch_cpu failed");
    return t;
}
