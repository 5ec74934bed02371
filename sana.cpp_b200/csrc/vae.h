// The DC-AE VAE decoder the reference runs after the denoiser (vae.h, vae.cpp:243-325,
// vae_ops.cpp), on the device: NHWC activations (pixel rows, channels contiguous), so every
// 1x1 convolution and projection is a GEMM over pixel rows and each 3x3 convolution is one
// over tap-major patches, on the same tensor-core GEMM as the denoiser.
#pragma once

#include <vector>

#include "engine.h"

namespace sana {

struct VaeBlockDims {
    int channels = 0, has_upsample = 0, is_res_block = 0, layers = 0;
};

// Mirrors SanaVaeWeights' structure (vae.h:43-73): up block i has `channels` outputs, an
// optional nearest-2x upsample conv from block i+1's channels, then `layers` ResBlocks or
// attention + GLUMBConv layers. head_dim is the attention head size (32 in
// run_vae_decode, vae.cpp:292), ms_kernel the multiscale depthwise size (3 or 5).
struct VaeDims {
    int latent_channels = 0, out_channels = 0, n_blocks = 0, head_dim = 32, ms_kernel = 5;
    float scaling_factor = 1.0f;
    VaeBlockDims blocks[8];
};

// Tensors per VaeDims in upload order (the order of include/sana_cuda.h's VAE table).
size_t vae_tensor_count(const VaeDims& d);
// validate_vae_weights (vae.cpp:172-208) on the dims: std::invalid_argument with its messages.
void vae_validate(const VaeDims& d);

class VaeDecoder {
   public:
    explicit VaeDecoder(Engine& eng) : eng_(eng) {}

    // Host fp32 tensors in PyTorch layouts, order as vae_tensor_count describes.
    void upload(const VaeDims& d, const float* const* tensors);
    bool has_weights() const { return have_; }
    const VaeDims& dims() const { return d_; }
    // run_vae_decode on device buffers: latents [B, latent, h, w] fp32 NCHW -> out
    // [B, out, h * 2^u, w * 2^u] fp32 NCHW, u = upsampling blocks. Asynchronous on the
    // engine's stream.
    void decode(const float* lat_d, int B, int h, int w, float* out_d);
    // The same on host buffers (copies in, decode, copies out, synchronizes, checks the
    // device error word).
    void decode_host(const float* lat, int B, int h, int w, float* out);
    // Launches of the last decode (host-side count of this decoder's kernels and GEMMs).
    int last_launches() const { return launches_; }

   private:
    struct Layer {
        DevBuf c1w, c1b, c2w;                    // ResBlock: conv weights [C, 9, C] (act type)
        DevBuf c1w2, c1b2, c2w2;                 // bf16, C <= 128: pixel-pair forms [2C, 12, C], [2C]
        DevBuf wqkv, msdw, msgw, wout;           // attention: [3C, C], [3C/32, k*k, 32] f32, [3C/32, 32, 32] f32, [C, 2C]
        DevBuf winv, binv, wdw, bdw, wpt;        // GLUMBConv: [8C, C], [8C], [8C, 9] f32, [8C], [C, 4C]
        DevBuf n1w, n1b, n2w, n2b;               // RMSNorm weight / bias (ResBlock: n1 only)
    };
    struct Block {
        DevBuf upw, upb;  // [C, 9, C_next] (act type), [C]
        DevBuf upw4;      // bf16: the four sub-pixel parity weights [4, C, 4, C_next]
        DevBuf upw4p, upb2;  // bf16, C <= 128: their pixel-pair forms [4, 2C, 6, C_next], bias [2C]
        std::vector<Layer> layers;
    };

    template <class T> void upload_impl(const float* const* t);
    template <class T> void decode_impl(const float* lat_d, int B, int h, int w, float* out_d);
    template <class T>
    void conv3x3(const T* in, int B, int H, int W, int Cin, bool upsample, const DevBuf& w, const float* bias,
                 int Cout, int act, T* out);
    template <class T>
    void upsample_conv(const T* in, int B, int H, int W, int Cin, const Block& blk, int Cout, T* out);
    // implicit convolution on the tensor cores when the shape tiles (bf16 only)
    bool implicit_ok(int H, int W, int Cin) const;
    // pair: two horizontally adjacent pixels per product row (ConvA::pair); w then holds the
    // pair weights and bias the doubled bias
    template <class T>
    void conv_gemm(const T* in, int B, int H, int W, int Cin, int kh, int kw, int oy, int ox, const void* w,
                   const float* bias, int Cout, int act, T* out, bool pair = false);
    bool pair_ok(int H, int W, int Cin, int Cout) const;
    template <class T>
    void gemm_rows(const T* A, long long M, int K, const DevBuf& w, const float* bias, int N, int act, T* out);
    void ensure_workspace(int B, int h, int w);

    Engine& eng_;
    VaeDims d_{};
    bool have_ = false;
    int launches_ = 0;
    DevBuf cin_w_, cin_b_, nout_w_, nout_b_, cout_w_, cout_b_;
    std::vector<Block> blocks_;
    // workspace (grown on demand): residual stream ping-pong, conv patches, branch buffers
    DevBuf x_, y_, g_, col_, qkv_, ms_, merged_, inv_, glu_, partial_, par_;
    long long ws_key_ = -1;
    DevBuf lat_in_, img_out_;  // host-path staging
};

}  // namespace sana
