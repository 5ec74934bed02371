// The reference's seeded latent generator (cconthekeyboard/sana.cpp src/torch_rng.h:1-14):
// torch.randn(shape) on a CPU torch.Generator seeded with `seed`, bit-identical, at least 16
// elements (std::invalid_argument otherwise, torch_rng.cpp:39-41). Implemented by
// host/frontend/torch_rng.cpp over the C ABI's sana_randn_torch_cpu.
#pragma once

#include <cstdint>
#include <vector>

#include "tensor.h"

Tensor randn_torch_cpu(const std::vector<size_t>& shape, uint64_t seed);
