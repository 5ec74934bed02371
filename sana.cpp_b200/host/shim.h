// Shared plumbing of the C++ host layer: the process-wide C-ABI handle, status -> exception
// mapping (SANA_ERR_INVALID -> std::invalid_argument, as the reference throws for argument
// and shape errors; anything else -> std::runtime_error) and the device weight cache.
#pragma once

#include <stdexcept>
#include <string>

#include "sana_cuda.h"
#include "tensor.h"

struct SanaDenoiserWeights;
struct SanaBlockWeights;
struct SanaSchedulerConfig;

namespace sana_shim {

sana_cuda_ctx* handle();
int mode();
// Changes whenever device copies of weights may no longer match the caller's tensors (a new
// handle, configure(), invalidate_weights()); caches compare it with the value they saw.
unsigned weights_epoch();
void check(int rc);
// Data pointer of a tensor, nullptr when it holds no elements.
const float* ptr(const Tensor& t);
// Data pointer of an optional tensor: nullptr when absent or empty.
const float* opt(const Tensor* t);
// A size as the C ABI's int; std::invalid_argument when it does not fit.
int as_int(size_t v, const char* what);
void require(bool ok, const char* message);

// Makes the handle's uploaded weights those of `w` (all blocks) / of the single block `b`.
void ensure_weights(const SanaDenoiserWeights& w);
void ensure_block(const SanaBlockWeights& b);

// The config as the C ABI's struct, after validate_scheduler_config's checks
// (scheduler.cpp:8-24; std::invalid_argument otherwise).
sana_scheduler_config c_config(const SanaSchedulerConfig& c);

}  // namespace sana_shim
