// Dense projections of the denoiser: C[M, N] = A[M, K] . B[N, K]^T with a fused epilogue.
//
// A is the activation (row-major, row stride lda elements), B the weight in PyTorch
// [out, in] layout (row stride ldb). The reference computes the same products as
// gemm_row_major over [in, out] weights (common_ops.cpp:13-65, linear_3d_lastdim :177,
// conv2d_1x1 :322); the weight cache stores the transpose so both operands are K-major.
#pragma once

#include "common.cuh"

namespace sana {

enum Activation : int { kActNone = 0, kActSilu = 1, kActGelu = 2 };

// What happens to an fp32 accumulator value v at (row r, column n):
//   v += bias[n]                                   (bias optional)
//   v  = act(v)                                    (none / SiLU / GELU-tanh)
//   v  = resid[r, n] + gate[r / rows_per_gate, n] * v   (residual mode; gate optional = 1)
//   out[r, n] = v   (bf16 or fp32), and optionally out2[r, n] = act2(v) (bf16 or fp32)
// This fuses, per projection, the bias add of gemm_row_major, the activations that follow
// it (silu_inplace, gelu_tanh_inplace), the AdaLN gate (mul_inplace_broadcast_lastdim,
// tensor.cpp:130) and the residual add (add_inplace, tensor.cpp:101) of block_forward.
struct Epilogue {
    const float* bias = nullptr;
    int act = kActNone;
    void* out = nullptr;
    int out_bf16 = 1;
    long long ldo = 0;
    const float* resid = nullptr;
    long long ldr = 0;
    const float* gate = nullptr;
    long long gate_ld = 0;
    int rows_per_gate = 1;
    void* out2 = nullptr;
    int out2_bf16 = 1;
    long long ldo2 = 0;
    int act2 = kActNone;
};

// Implicit convolution as the A operand (tensor-core pair kernel only): A is an NHWC bf16
// image batch [M / (H * W), H, W, C] and row m of the product is pixel m. K = kh * kw * C with
// k = t * C + c, tap t = ty * kw + tx reading the pixel at offset (oy + ty, ox + tx), zero
// outside the image. A 3x3 "same" convolution is kh = kw = 3, oy = ox = -1. The weight B is
// [N, kh * kw * C] in the same tap-major order. Needs C % 64 == 0 and 128-row tiles that
// are rectangles of whole image rows: W % 128 == 0, or 128 % W == 0 with (H * W) % 128 == 0.
//
// pair = 1 makes each product row a pair of horizontally adjacent pixels (2x, 2x + 1), so an
// N = 128-channel convolution becomes an N = 256 product: W and C then describe the image
// as super-pixels of two pixels (W = pixel width / 2, C = 2 * channels), K = kh * kw * (C / 2)
// with tap column e = ox + tx relative to the row's first pixel reading pixel 2x + e, and
// the weight rows [0, N/2) / [N/2, N) are the even / odd pixel's outputs.
struct ConvA {
    int H = 0, W = 0, C = 0;
    int kh = 3, kw = 3, oy = -1, ox = -1;
    int pair = 0;
};

struct GemmProblem {
    const void* A = nullptr;
    int a_bf16 = 1;
    long long lda = 0;
    const void* B = nullptr;
    int b_bf16 = 1;
    long long ldb = 0;
    int M = 0, N = 0, K = 0;
    Epilogue ep;
    ConvA conv;  // conv.H == 0: A is a plain row-major matrix
    // Set by the denoiser and VAE paths: bf16 operands must take the tensor-core kernel
    // unless the shape itself rules it out (K % 8 != 0 or N < 16, tiny test models); a
    // problem refused only for its pointers or strides is an error, not a slow fallback.
    int require_tc = 0;
};

// True when the tcgen05 kernel can run the problem (bf16 operands, TMA-legal strides).
bool gemm_tc_supported(const GemmProblem& p);
// True when the problem's shape alone (K % 8 == 0, N >= 16) allows the tensor-core kernel.
bool gemm_tc_shape_ok(const GemmProblem& p);
// The same for an implicit-convolution problem (p.conv set).
bool gemm_conv_supported(const GemmProblem& p);
// tcgen05 / TMEM / TMA tensor-core path (gemm_tc.cu). err: device error word.
void gemm_tc(const GemmProblem& p, int* err, cudaStream_t stream, int num_sms);
// Generic CUDA-core path for any shape or operand type (gemm_simt.cu): fp32 check mode,
// tiny shapes and odd strides.
void gemm_simt(const GemmProblem& p, cudaStream_t stream);
// Dispatch: tensor cores when supported and not disabled, else the generic path.
void gemm(const GemmProblem& p, int* err, cudaStream_t stream, int num_sms, bool allow_tc = true);

// Process-wide counts of gemm() dispatches to each path (host-side launch accounting).
void gemm_counts(long long* tc, long long* simt);

}  // namespace sana
