// Controls of the C++ host layer that have no counterpart in the reference (which has no
// device state): which GPU and precision the reference API entry points run on, and when the
// device copy of the weights must be refreshed.
#pragma once

namespace sana_cuda_shim {

// Device and mode (SANA_MODE_BF16 = 0: bf16 operands on the tensor cores, the default;
// SANA_MODE_F32 = 1: fp32 everywhere, the parity check mode). Takes effect for the next call;
// without it the environment decides (SANA_CUDA_DEVICE, SANA_CUDA_MODE = bf16 | f32).
void configure(int device, int mode);

// The entry points keep one device copy of the last SanaDenoiserWeights (or SanaBlockWeights)
// and of the last SanaVaeWeights they were given, recognised by the addresses and sizes of
// their tensors. A caller that overwrites weight values in place calls this so that the next
// call uploads them again.
void invalidate_weights();

}  // namespace sana_cuda_shim
