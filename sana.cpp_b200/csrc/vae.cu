// The DC-AE VAE decoder on the device (vae.cpp:243-325, vae_ops.cpp). Activations are NHWC
// rows [pixels, channels] in the engine's activation type (bf16, or fp32 in check mode).
//
//   conv_in (3x3 over latents / scaling_factor, + the repeated-channel shortcut)
//   for each up block, innermost first:
//     [nearest-2x upsample conv 3x3 + the pixel-shuffled channel shortcut]
//     ResBlock:  x + RMSNorm(conv3x3(silu(conv3x3(x) + b)))
//     or EfficientViT layer:
//       x + RMSNorm(to_out(linear attention over qkv heads and the multiscale heads))
//       x + RMSNorm(conv_point(dw3x3 GLU(silu(conv_inverted(x) + b))))
//   RMSNorm(+bias), ReLU, conv_out 3x3 -> NCHW fp32
//
// 3x3 convolutions are implicit GEMMs on the tensor-core kernel: its producer loads each
// tap's shifted pixel tile straight from the NHWC image with 4-D TMA boxes (zero fill at
// the borders), weights reordered to [Cout, 9, Cin] at upload. A nearest-2x upsample
// followed by a 3x3 conv is computed as four 2x2 convolutions on the low-resolution image,
// one per output parity (the 3x3 taps that land on the same source pixel summed at
// upload), and a shuffle kernel interleaves them and adds the channel shortcut: 4/9 of the
// FLOPs, no upsampled copy. Shapes the implicit path cannot tile (and the fp32 check mode)
// gather tap-major patches [pixels, 9 * Cin] for a plain GEMM instead. The
// q/k/v projection rows are permuted at upload in groups of head_dim channels so that the
// reference's reading of the concatenated [q | k | v] (head g takes channels
// [3 g d, 3 g d + 3 d) as its q, k, v; vae_ops.cpp:686-714) becomes the plain
// [q heads | k heads | v heads] layout of the linear-attention kernel; the multiscale
// depthwise and grouped weights move with their channels.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "vae.h"

namespace sana {

namespace {

inline int blocks_for(long long n, int threads = 256) { return static_cast<int>((n + threads - 1) / threads); }

// conv_in: 3x3 "same" over latents * inv_sf (NCHW fp32), + bias, + the repeated-channel
// shortcut out[c] += scaled[c / (C / Cl)] (vae.cpp:210-241, vae_ops.cpp:455-493).
// w: [9, Cl, C] fp32 (consecutive output channels read consecutive weights). out: NHWC [B*H*W, C].
// A block computes kCinPix consecutive pixels for every output channel: their scaled 3x3
// neighbourhoods ([9 * Cl][kCinPix], zero outside the image) sit in shared memory and each
// weight is read once for all of them. Cl <= 64, C <= 1024.
constexpr int kCinPix = 4;
template <class T>
__global__ void __launch_bounds__(256) vae_conv_in_kernel(const float* __restrict__ lat, int B, int Cl, int H, int W,
                                                          const float* __restrict__ w, const float* __restrict__ bias,
                                                          float inv_sf, int C, T* __restrict__ out) {
    __shared__ __align__(16) float s_lat[9 * 64][kCinPix];
    const long long P = static_cast<long long>(B) * H * W;
    const long long p0 = static_cast<long long>(blockIdx.x) * kCinPix;
    const int K = 9 * Cl;
    for (int i = threadIdx.x; i < K * kCinPix; i += blockDim.x) {
        const int k = i % kCinPix, t = i / kCinPix;
        const int tap = t / Cl, c = t % Cl;
        const long long p = p0 + k;
        float v = 0.f;
        if (p < P) {
            const int x = static_cast<int>(p % W), y = static_cast<int>((p / W) % H);
            const int b = static_cast<int>(p / (static_cast<long long>(W) * H));
            const int iy = y + tap / 3 - 1, ix = x + tap % 3 - 1;
            if (iy >= 0 && iy < H && ix >= 0 && ix < W)
                v = lat[((static_cast<long long>(b) * Cl + c) * H + iy) * W + ix] * inv_sf;
        }
        s_lat[t][k] = v;
    }
    __syncthreads();
    const int rep = C / Cl;
    for (int oc = threadIdx.x; oc < C; oc += blockDim.x) {
        float acc[kCinPix];
#pragma unroll
        for (int k = 0; k < kCinPix; ++k) acc[k] = bias[oc];
#pragma unroll 8  // several weight loads in flight per thread
        for (int t = 0; t < K; ++t) {
            const float wv = w[static_cast<long long>(t) * C + oc];
#pragma unroll
            for (int k4 = 0; k4 < kCinPix; k4 += 4) {
                const float4 a = *reinterpret_cast<const float4*>(&s_lat[t][k4]);
                acc[k4] = fmaf(wv, a.x, acc[k4]);
                acc[k4 + 1] = fmaf(wv, a.y, acc[k4 + 1]);
                acc[k4 + 2] = fmaf(wv, a.z, acc[k4 + 2]);
                acc[k4 + 3] = fmaf(wv, a.w, acc[k4 + 3]);
            }
        }
#pragma unroll
        for (int k = 0; k < kCinPix; ++k) {
            const long long p = p0 + k;
            if (p >= P) break;
            const int x = static_cast<int>(p % W), y = static_cast<int>((p / W) % H);
            const int b = static_cast<int>(p / (static_cast<long long>(W) * H));
            const float sc = lat[((static_cast<long long>(b) * Cl + oc / rep) * H + y) * W + x] * inv_sf;
            out[p * C + oc] = from_f<T>(acc[k] + sc);
        }
    }
}

// Tap-major 3x3 patches of an NHWC image for a "same" convolution at output size
// (H << up) x (W << up): col[p, tap, c] = in at output pixel p shifted by the tap, read
// through the nearest-2x upsample when up = 1, zero outside. V channels per thread.
template <class T, int V>
__global__ void im2col3x3_kernel(const T* __restrict__ in, int B, int H, int W, int C, int up,
                                 T* __restrict__ col) {
    const int Ho = H << up, Wo = W << up, CV = C / V;
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long n = static_cast<long long>(B) * Ho * Wo * 9 * CV;
    if (i >= n) return;
    const int cv = static_cast<int>(i % CV);
    const long long r = i / CV;
    const int tap = static_cast<int>(r % 9);
    const long long p = r / 9;
    const int x = static_cast<int>(p % Wo);
    const int y = static_cast<int>((p / Wo) % Ho);
    const int b = static_cast<int>(p / (static_cast<long long>(Wo) * Ho));
    const int yy = y + tap / 3 - 1, xx = x + tap % 3 - 1;
    using Vec = typename std::conditional<V * sizeof(T) == 16, uint4, T>::type;
    Vec v;
    if (yy < 0 || yy >= Ho || xx < 0 || xx >= Wo) {
        if constexpr (V * sizeof(T) == 16) v = make_uint4(0u, 0u, 0u, 0u);
        else v = from_f<T>(0.0f);
    } else {
        const long long src = ((static_cast<long long>(b) * H + (yy >> up)) * W + (xx >> up)) * C + cv * V;
        v = *reinterpret_cast<const Vec*>(in + src);
    }
    *reinterpret_cast<Vec*>(col + i * V) = v;
}

// The upsample shortcut (vae_ops.cpp:392-453): out[b, 2y+i, 2x+j, oc] +=
// in[b, y, x, (4 oc + 2 i + j) / (4 Cout / Cin)].
template <class T>
__global__ void up_shortcut_kernel(T* __restrict__ out, const T* __restrict__ in, int B, int H, int W, int Cin,
                                   int Cout) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int Ho = 2 * H, Wo = 2 * W;
    const long long n = static_cast<long long>(B) * Ho * Wo * Cout;
    if (i >= n) return;
    const int oc = static_cast<int>(i % Cout);
    const long long p = i / Cout;
    const int xo = static_cast<int>(p % Wo);
    const int yo = static_cast<int>((p / Wo) % Ho);
    const int b = static_cast<int>(p / (static_cast<long long>(Wo) * Ho));
    const int rep = 4 * Cout / Cin;
    const int ic = (4 * oc + 2 * (yo & 1) + (xo & 1)) / rep;
    const float s = to_f(in[((static_cast<long long>(b) * H + (yo >> 1)) * W + (xo >> 1)) * Cin + ic]);
    out[i] = from_f<T>(to_f(out[i]) + s);
}

// Interleaves the four parity outputs par[ij] ([B*H*W, Cout] each, ij = 2 i + j) of a
// sub-pixel upsample conv into out[b, 2y+i, 2x+j, :] and adds the upsample shortcut of
// up_shortcut_kernel. 8 channels per thread (16-byte parity loads and output stores);
// blockIdx.y is the image.
__global__ void shuffle_shortcut_kernel(const bf16* __restrict__ par, const bf16* __restrict__ in, int B, int H,
                                        int W, int Cin, int Cout, bf16* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int CV = Cout / 8, Wo = 2 * W;
    if (i >= 4 * H * W * CV) return;
    const int b = blockIdx.y;
    const int oc0 = (i % CV) * 8;
    const int p = i / CV;
    const int xo = p % Wo, yo = p / Wo;
    const int ij = 2 * (yo & 1) + (xo & 1);
    const long long lo = static_cast<long long>(b) * H * W + (yo >> 1) * W + (xo >> 1);
    const long long plane = static_cast<long long>(B) * H * W * Cout;
    const uint4 raw = *reinterpret_cast<const uint4*>(par + ij * plane + lo * Cout + oc0);
    const bf16* e = reinterpret_cast<const bf16*>(&raw);
    const bf16* sc = in + lo * Cin;
    const int rep = 4 * Cout / Cin;
    uint4 o;
    bf16* oe = reinterpret_cast<bf16*>(&o);
    if (rep == 4) {  // Cin == Cout: the shortcut channel is oc itself
        const uint4 sraw = *reinterpret_cast<const uint4*>(sc + oc0);
        const bf16* se = reinterpret_cast<const bf16*>(&sraw);
#pragma unroll
        for (int k = 0; k < 8; ++k) oe[k] = __float2bfloat16_rn(__bfloat162float(e[k]) + __bfloat162float(se[k]));
    } else if (rep == 2) {  // Cin == 2 Cout: channel 2 oc + (ij >> 1), every other one of 16
        const uint4 s0 = *reinterpret_cast<const uint4*>(sc + 2 * oc0);
        const uint4 s1 = *reinterpret_cast<const uint4*>(sc + 2 * oc0 + 8);
        const bf16* se0 = reinterpret_cast<const bf16*>(&s0);
        const bf16* se1 = reinterpret_cast<const bf16*>(&s1);
        const int odd = ij >> 1;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const bf16 v = k < 4 ? se0[2 * k + odd] : se1[2 * (k - 4) + odd];
            oe[k] = __float2bfloat16_rn(__bfloat162float(e[k]) + __bfloat162float(v));
        }
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
            oe[k] = __float2bfloat16_rn(__bfloat162float(e[k]) + __bfloat162float(sc[(4 * (oc0 + k) + ij) / rep]));
    }
    *reinterpret_cast<uint4*>(out + (static_cast<long long>(b) * 4 * H * W + p) * Cout + oc0) = o;
}

// rms_norm_4d_channelwise (vae_ops.cpp:495-575) over each pixel row, then the residual
// add (add_inplace) or ReLU (vae.cpp:313-319): out = x / sqrt(mean(x^2) + eps) * w + b
// (+ resid | relu). One warp per row.
template <class T>
__global__ void rms_rows_kernel(const T* __restrict__ x, long long rows, int C, const float* __restrict__ w,
                                const float* __restrict__ b, float eps, const T* __restrict__ resid, int relu,
                                T* __restrict__ out) {
    const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const T* xr = x + row * C;
    float ss = 0.f;
    for (int c = lane; c < C; c += 32) {
        const float v = to_f(xr[c]);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(C)) + eps);
    T* orow = out + row * C;
    const T* rr = resid ? resid + row * C : nullptr;
    for (int c = lane; c < C; c += 32) {
        float v = to_f(xr[c]) * inv * w[c] + b[c];
        if (rr) v += to_f(rr[c]);
        if (relu) v = fmaxf(v, 0.0f);
        orow[c] = from_f<T>(v);
    }
}

// The same with each lane holding ITER chunks of VPL consecutive channels of RPW rows in
// registers (C == 32 * VPL * ITER; bf16 rows), all loads of a warp's rows issued before
// the reductions.
template <int VPL, int ITER, int RPW>
__global__ void rms_rows_vec_kernel(const bf16* __restrict__ x, long long rows, int C, const float* __restrict__ w,
                                    const float* __restrict__ b, float eps, const bf16* __restrict__ resid, int relu,
                                    bf16* __restrict__ out) {
    using Vec = typename std::conditional<VPL == 8, uint4, uint2>::type;
    const long long row0 = (static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32) * RPW;
    const int lane = threadIdx.x & 31;
    if (row0 >= rows) return;
    Vec xv[RPW][ITER], rv[RPW][ITER];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int it = 0; it < ITER; ++it) {
            const long long row = row0 + r < rows ? row0 + r : rows - 1;
            const int c0 = (it * 32 + lane) * VPL;
            xv[r][it] = *reinterpret_cast<const Vec*>(x + row * C + c0);
            if (resid) rv[r][it] = *reinterpret_cast<const Vec*>(resid + row * C + c0);
        }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        if (row0 + r >= rows) break;
        float ss = 0.f;
#pragma unroll
        for (int it = 0; it < ITER; ++it) {
            const bf16* e = reinterpret_cast<const bf16*>(&xv[r][it]);
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const float v = __bfloat162float(e[k]);
                ss = fmaf(v, v, ss);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(C)) + eps);
#pragma unroll
        for (int it = 0; it < ITER; ++it) {
            const int c0 = (it * 32 + lane) * VPL;
            const bf16* e = reinterpret_cast<const bf16*>(&xv[r][it]);
            const bf16* re = reinterpret_cast<const bf16*>(&rv[r][it]);
            Vec o;
            bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                float y = __bfloat162float(e[k]) * inv * w[c0 + k] + b[c0 + k];
                if (resid) y += __bfloat162float(re[k]);
                if (relu) y = fmaxf(y, 0.0f);
                oe[k] = __float2bfloat16_rn(y);
            }
            *reinterpret_cast<Vec*>(out + (row0 + r) * C + c0) = o;
        }
    }
}

// The multiscale branch (vae_ops.cpp:681-682): depthwise K x K (no bias) then the grouped
// 1x1 over groups of 32 channels, fused per (16 x 8 pixel tile, group). qkv / out:
// [pixels, C3] rows (C3 % 8 == 0, 16-byte aligned); weights fp32 per group of 32 channels
// (in the permuted group order of the qkv columns), channel-fastest so a warp's loads are
// coalesced: dw [C3 / 32, K*K, 32], gw [C3 / 32, 32 inputs, 32 outputs]. Depthwise: thread (channel c,
// column pair) slides down its two columns, each input row read once for the 8 outputs
// it feeds; grouped: thread (output channel o) over 16 pixels with 16-byte broadcast reads.
constexpr int kMsTileX = 16, kMsTileY = 8, kMsPix = kMsTileX * kMsTileY;
template <class T, int K>
__global__ void __launch_bounds__(256) ms_branch_kernel(const T* __restrict__ qkv, int B, int H, int W, int C3,
                                                        const float* __restrict__ dw, const float* __restrict__ gw,
                                                        T* __restrict__ out) {
    constexpr int R = K / 2, HX = kMsTileX + K - 1, HY = kMsTileY + K - 1;
    constexpr int kVec = 16 / sizeof(T);  // channels per 16-byte load
    __shared__ float s_in[HX * HY][33];
    __shared__ __align__(16) float s_d[kMsPix][32];
    const int tiles_x = (W + kMsTileX - 1) / kMsTileX;
    const int tx0 = (blockIdx.x % tiles_x) * kMsTileX, ty0 = (blockIdx.x / tiles_x) * kMsTileY;
    const int g = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
    const int c = tid & 31, col = tid >> 5;
    const long long img = static_cast<long long>(b) * H * W;
    for (int i = tid; i < HX * HY * (32 / kVec); i += blockDim.x) {
        const int cv = i % (32 / kVec), pix = i / (32 / kVec);
        const int y = ty0 - R + pix / HX, x = tx0 - R + pix % HX;
        float* dst = &s_in[pix][cv * kVec];
        if (y >= 0 && y < H && x >= 0 && x < W) {
            const uint4 raw = *reinterpret_cast<const uint4*>(qkv + (img + static_cast<long long>(y) * W + x) * C3 +
                                                              g * 32 + cv * kVec);
            const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
            for (int k = 0; k < kVec; ++k) dst[k] = to_f(e[k]);
        } else {
#pragma unroll
            for (int k = 0; k < kVec; ++k) dst[k] = 0.f;
        }
    }
    float wk[K * K];
#pragma unroll
    for (int k = 0; k < K * K; ++k) wk[k] = dw[(static_cast<long long>(g) * K * K + k) * 32 + c];
    __syncthreads();
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int px = col + 8 * half;
        float acc[kMsTileY];
#pragma unroll
        for (int py = 0; py < kMsTileY; ++py) acc[py] = 0.f;
#pragma unroll
        for (int r = 0; r < HY; ++r) {
            float v[K];
#pragma unroll
            for (int kx = 0; kx < K; ++kx) v[kx] = s_in[r * HX + px + kx][c];
#pragma unroll
            for (int py = 0; py < kMsTileY; ++py) {
                const int ky = r - py;
                if (ky >= 0 && ky < K) {
#pragma unroll
                    for (int kx = 0; kx < K; ++kx) acc[py] = fmaf(v[kx], wk[ky * K + kx], acc[py]);
                }
            }
        }
#pragma unroll
        for (int py = 0; py < kMsTileY; ++py) s_d[py * kMsTileX + px][c] = acc[py];
    }
    float gk[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) gk[k] = gw[(static_cast<long long>(g) * 32 + k) * 32 + c];
    __syncthreads();
#pragma unroll 2
    for (int j = 0; j < kMsPix / 8; ++j) {
        const int p = j * 8 + col, y = ty0 + p / kMsTileX, x = tx0 + p % kMsTileX;
        const float4* dp = reinterpret_cast<const float4*>(s_d[p]);
        float acc = 0.f;
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4) {
            const float4 d4 = dp[k4];
            acc = fmaf(gk[4 * k4], d4.x, acc);
            acc = fmaf(gk[4 * k4 + 1], d4.y, acc);
            acc = fmaf(gk[4 * k4 + 2], d4.z, acc);
            acc = fmaf(gk[4 * k4 + 3], d4.w, acc);
        }
        if (y < H && x < W) out[(img + static_cast<long long>(y) * W + x) * C3 + g * 32 + c] = from_f<T>(acc);
    }
}

// conv_out, bf16 rows, C % 8 == 0: a block computes an 8 x 128-pixel tile (thread: one row,
// pixels x0 + lane + 32 k, k < 4), staging the tile's halo 8 channels at a time in shared
// memory ([10 rows][130 px] x 16 bytes: a warp's reads are consecutive pixels, no bank
// conflicts); the four output channels' weights of each (tap, channel) are one float4 in
// shared memory, read once per (tap, channel) for all four pixels. blockIdx.z is the image.
constexpr int kCoTileX = 128, kCoTileY = 8, kCoHaloX = kCoTileX + 2, kCoHaloY = kCoTileY + 2;
template <bool kFourth>  // a fourth output channel (Co == 4); RGB skips its FMAs
__global__ void __launch_bounds__(256) vae_conv_out_bf16_kernel(const bf16* __restrict__ in, int H, int W, int C,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ bias, int Co,
                                                                float* __restrict__ out) {
    extern __shared__ float4 s_w4[];                        // [9][C]
    __shared__ uint4 s_in[kCoHaloY * kCoHaloX];            // 8 channels per pixel
    for (int i = threadIdx.x; i < 9 * C; i += blockDim.x) {
        const int tap = i / C, c = i % C;
        float v[4];
#pragma unroll
        for (int o = 0; o < 4; ++o) v[o] = o < Co ? w[(static_cast<long long>(o) * 9 + tap) * C + c] : 0.f;
        s_w4[i] = make_float4(v[0], v[1], v[2], v[3]);
    }
    const int x0 = blockIdx.x * kCoTileX, y0 = blockIdx.y * kCoTileY, b = blockIdx.z;
    const int lane = threadIdx.x & 31, row = threadIdx.x >> 5;
    const bf16* img = in + static_cast<long long>(b) * H * W * C;
    float4 acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < C; c0 += 8) {
        __syncthreads();  // the previous chunk's reads are done (and the weights are staged)
        for (int i = threadIdx.x; i < kCoHaloY * kCoHaloX; i += blockDim.x) {
            const int y = y0 - 1 + i / kCoHaloX, x = x0 - 1 + i % kCoHaloX;
            s_in[i] = (y >= 0 && y < H && x >= 0 && x < W)
                          ? *reinterpret_cast<const uint4*>(img + (static_cast<long long>(y) * W + x) * C + c0)
                          : make_uint4(0u, 0u, 0u, 0u);
        }
        __syncthreads();
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
            const int dy = tap / 3, dx = tap % 3;
            float v[4][8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint4 raw = s_in[(row + dy) * kCoHaloX + lane + 32 * k + dx];
                const bf16* e = reinterpret_cast<const bf16*>(&raw);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[k][j] = __bfloat162float(e[j]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 wv = s_w4[tap * C + c0 + j];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    acc[k].x = fmaf(wv.x, v[k][j], acc[k].x);
                    acc[k].y = fmaf(wv.y, v[k][j], acc[k].y);
                    acc[k].z = fmaf(wv.z, v[k][j], acc[k].z);
                    if constexpr (kFourth) acc[k].w = fmaf(wv.w, v[k][j], acc[k].w);
                }
            }
        }
    }
    const int y = y0 + row;
    if (y >= H) return;
    const long long plane = static_cast<long long>(H) * W;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int x = x0 + lane + 32 * k;
        if (x >= W) continue;
        float* o0 = out + static_cast<long long>(b) * Co * plane + static_cast<long long>(y) * W + x;
        o0[0] = acc[k].x + bias[0];
        if (Co > 1) o0[plane] = acc[k].y + bias[1];
        if (Co > 2) o0[2 * plane] = acc[k].z + bias[2];
        if (Co > 3) o0[3 * plane] = acc[k].w + bias[3];
    }
}

// conv_out (vae.cpp:320-324): 3x3 "same" from NHWC rows [pixels, C] to NCHW fp32 with few
// output channels (Co <= 4). A warp walks kConvOutPix consecutive pixels; lane l holds
// channels [l * CPL, l * CPL + CPL) (those below C; C <= 32 * CPL), so each tap's row is one coalesced
// load; the four output sums are reduced across the warp per pixel. Weights are staged in
// shared memory as [9][4][CPL][32 lanes] fp32 (zero past Co or C), so a lane's reads are
// consecutive words across the warp (no bank conflicts).
constexpr int kConvOutPix = 8;
template <class T, int CPL>
__global__ void __launch_bounds__(256) vae_conv_out_kernel(const T* __restrict__ in, int B, int H, int W, int C,
                                                           const float* __restrict__ w, const float* __restrict__ bias,
                                                           int Co, float* __restrict__ out) {
    extern __shared__ float s_w[];  // [9][4][CPL][32]
    for (int i = threadIdx.x; i < 9 * 4 * CPL * 32; i += blockDim.x) {
        const int l = i & 31, j = (i >> 5) % CPL, o = (i / (32 * CPL)) % 4, tap = i / (128 * CPL);
        const int c = l * CPL + j;
        s_w[i] = (o < Co && c < C) ? w[(static_cast<long long>(o) * 9 + tap) * C + c] : 0.f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int P = H * W, b = blockIdx.y;
    const int p0 = (blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * kConvOutPix;
    for (int k = 0; k < kConvOutPix; ++k) {
        const int p = p0 + k;
        if (p >= P) break;
        const int x = p % W, y = p / W;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int tap = 0; tap < 9; ++tap) {
            const int iy = y + tap / 3 - 1, ix = x + tap % 3 - 1;
            if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
            const T* src = in + ((static_cast<long long>(b) * H + iy) * W + ix) * C + lane * CPL;
            if (lane * CPL >= C) continue;
            float v[CPL];
#pragma unroll
            for (int j = 0; j < CPL; ++j) v[j] = to_f(src[j]);
            const float* wt = s_w + tap * 128 * CPL + lane;
#pragma unroll
            for (int o = 0; o < 4; ++o)
#pragma unroll
                for (int j = 0; j < CPL; ++j) acc[o] = fmaf(wt[(o * CPL + j) * 32], v[j], acc[o]);
        }
#pragma unroll
        for (int o = 0; o < 4; ++o)
#pragma unroll
            for (int sh = 16; sh > 0; sh >>= 1) acc[o] += __shfl_xor_sync(0xffffffffu, acc[o], sh);
        if (lane < Co) {
            float r = acc[0];
#pragma unroll
            for (int o = 1; o < 4; ++o)
                if (lane == o) r = acc[o];
            out[((static_cast<long long>(b) * Co + lane) * H + y) * W + x] = r + bias[lane];
        }
    }
}

// --- host-side weight preparation -------------------------------------------------------

uint16_t bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

template <class T>
void put(DevBuf& dst, const std::vector<float>& src) {
    dst.ensure(src.size() * sizeof(T));
    if (sizeof(T) == 4) {
        SANA_CUDA(cudaMemcpy(dst.get(), src.data(), src.size() * 4, cudaMemcpyHostToDevice));
    } else {
        std::vector<uint16_t> h(src.size());
        for (size_t i = 0; i < src.size(); ++i) h[i] = bf16_bits(src[i]);
        SANA_CUDA(cudaMemcpy(dst.get(), h.data(), h.size() * 2, cudaMemcpyHostToDevice));
    }
}

std::vector<float> copy_of(const float* p, size_t n) { return std::vector<float>(p, p + n); }

// [Cout, Cin, 3, 3] -> [Cout, 9, Cin]
std::vector<float> tap_major(const float* w, int Cout, int Cin) {
    std::vector<float> r(static_cast<size_t>(Cout) * 9 * Cin);
    for (int o = 0; o < Cout; ++o)
        for (int c = 0; c < Cin; ++c)
            for (int t = 0; t < 9; ++t) r[(static_cast<size_t>(o) * 9 + t) * Cin + c] = w[(static_cast<size_t>(o) * Cin + c) * 9 + t];
    return r;
}

// [Cout, Cin, 3, 3] -> four [Cout, 4, Cin] weights of the sub-pixel upsample conv: parity
// (i, j) reads low-resolution rows y + i - 1 + a and columns x + j - 1 + c (a, c in {0, 1});
// its weight sums the 3x3 taps that fall on that source pixel after the nearest-2x
// upsample (rows: i = 0 -> {0}, {1, 2}; i = 1 -> {0, 1}, {2}; columns likewise).
std::vector<float> parity_weights(const float* w, int Cout, int Cin) {
    static const int lo[2][2] = {{0, 1}, {0, 2}}, hi[2][2] = {{0, 2}, {1, 2}};  // [parity][a] -> tap range
    std::vector<float> r(static_cast<size_t>(4) * Cout * 4 * Cin, 0.f);
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j)
            for (int o = 0; o < Cout; ++o)
                for (int a = 0; a < 2; ++a)
                    for (int c2 = 0; c2 < 2; ++c2)
                        for (int c = 0; c < Cin; ++c) {
                            float sum = 0.f;
                            for (int ky = lo[i][a]; ky <= hi[i][a]; ++ky)
                                for (int kx = lo[j][c2]; kx <= hi[j][c2]; ++kx)
                                    sum += w[((static_cast<size_t>(o) * Cin + c) * 3 + ky) * 3 + kx];
                            r[((static_cast<size_t>(2 * i + j) * Cout + o) * 4 + (2 * a + c2)) * Cin + c] = sum;
                        }
    return r;
}

// Per group of 32 rows of `rows` ([groups * 32, n]): the [32, n] block transposed to [n, 32].
std::vector<float> group_transpose(const std::vector<float>& rows, size_t n) {
    std::vector<float> r(rows.size());
    const size_t groups = rows.size() / (32 * n);
    for (size_t g = 0; g < groups; ++g)
        for (size_t c = 0; c < 32; ++c)
            for (size_t k = 0; k < n; ++k) r[(g * n + k) * 32 + c] = rows[(g * 32 + c) * n + k];
    return r;
}

// Pixel-pair weights of a 3x3 "same" conv ([Cout, Cin, 3, 3] -> [2 Cout, 3, 4, Cin]): rows
// [0, Cout) the even pixel's outputs, [Cout, 2 Cout) the odd one's; tap column tx reads the
// pixel at offset tx - 1 from the even pixel, i.e. kernel column tx for the even pixel and
// tx - 1 for the odd one (zero where the column falls outside the kernel).
std::vector<float> pair_conv3x3(const float* w, int Cout, int Cin) {
    std::vector<float> r(static_cast<size_t>(2) * Cout * 12 * Cin, 0.f);
    for (int n = 0; n < 2 * Cout; ++n) {
        const int o = n % Cout, shift = n / Cout;
        for (int ty = 0; ty < 3; ++ty)
            for (int tx = 0; tx < 4; ++tx) {
                const int kx = tx - shift;
                if (kx < 0 || kx > 2) continue;
                for (int c = 0; c < Cin; ++c)
                    r[((static_cast<size_t>(n) * 3 + ty) * 4 + tx) * Cin + c] =
                        w[((static_cast<size_t>(o) * Cin + c) * 3 + ty) * 3 + kx];
            }
    }
    return r;
}

// Pixel-pair form of the four sub-pixel weights ([4, Cout, 4, Cin] -> [4, 2 Cout, 2, 3, Cin]):
// tap column tx is the even pixel's column tx and the odd pixel's tx - 1.
std::vector<float> pair_parity(const std::vector<float>& w4, int Cout, int Cin) {
    std::vector<float> r(static_cast<size_t>(4) * 2 * Cout * 6 * Cin, 0.f);
    for (int ij = 0; ij < 4; ++ij)
        for (int n = 0; n < 2 * Cout; ++n) {
            const int o = n % Cout, shift = n / Cout;
            for (int ty = 0; ty < 2; ++ty)
                for (int tx = 0; tx < 3; ++tx) {
                    const int kx = tx - shift;
                    if (kx < 0 || kx > 1) continue;
                    for (int c = 0; c < Cin; ++c)
                        r[(((static_cast<size_t>(ij) * 2 * Cout + n) * 2 + ty) * 3 + tx) * Cin + c] =
                            w4[((static_cast<size_t>(ij) * Cout + o) * 4 + ty * 2 + kx) * Cin + c];
                }
        }
    return r;
}

std::vector<float> twice(const float* b, size_t n) {
    std::vector<float> r(2 * n);
    std::copy(b, b + n, r.begin());
    std::copy(b, b + n, r.begin() + static_cast<long>(n));
    return r;
}

// [C, Cl, 3, 3] -> [9, Cl, C]
std::vector<float> conv_in_layout(const float* w, int C, int Cl) {
    std::vector<float> r(static_cast<size_t>(9) * Cl * C);
    for (int o = 0; o < C; ++o)
        for (int c = 0; c < Cl; ++c)
            for (int t = 0; t < 9; ++t) r[(static_cast<size_t>(t) * Cl + c) * C + o] = w[(static_cast<size_t>(o) * Cl + c) * 9 + t];
    return r;
}

// Row groups of the concatenated [q | k | v] (3 * heads groups of d rows) in the order
// q-parts of every head, k-parts, v-parts: new group j takes old group 3 (j % heads) + j / heads.
std::vector<float> permute_groups(const std::vector<float>& rows, int heads, int d, size_t row_len) {
    std::vector<float> r(rows.size());
    for (int j = 0; j < 3 * heads; ++j) {
        const int old = 3 * (j % heads) + j / heads;
        std::memcpy(&r[static_cast<size_t>(j) * d * row_len], &rows[static_cast<size_t>(old) * d * row_len],
                    static_cast<size_t>(d) * row_len * sizeof(float));
    }
    return r;
}

template <class T>
void launch_im2col(const T* in, int B, int H, int W, int C, int up, T* col, cudaStream_t st) {
    constexpr int V = 16 / static_cast<int>(sizeof(T));
    const long long pix = static_cast<long long>(B) * (H << up) * (W << up);
    if (C % V == 0) {
        im2col3x3_kernel<T, V><<<blocks_for(pix * 9 * (C / V)), 256, 0, st>>>(in, B, H, W, C, up, col);
    } else {
        im2col3x3_kernel<T, 1><<<blocks_for(pix * 9 * C), 256, 0, st>>>(in, B, H, W, C, up, col);
    }
    SANA_CUDA(cudaGetLastError());
}

}  // namespace

size_t vae_tensor_count(const VaeDims& d) {
    size_t n = 6;
    for (int i = 0; i < d.n_blocks; ++i) {
        const VaeBlockDims& b = d.blocks[i];
        n += (b.has_upsample ? 2 : 0) + static_cast<size_t>(b.layers) * (b.is_res_block ? 5 : 15);
    }
    return n;
}

void vae_validate(const VaeDims& d) {
    if (d.n_blocks < 1 || d.n_blocks > 8) throw InvalidArg("vae decoder must contain at least one up block");
    if (!(d.scaling_factor > 0.0f)) throw InvalidArg("vae scaling_factor must be positive");
    if (d.latent_channels < 1 || d.latent_channels > 64 || d.out_channels < 1 || d.out_channels > 4)
        throw InvalidArg("vae decoder latent channels must be in [1, 64] and output channels in [1, 4]");
    if (d.head_dim != 32) throw InvalidArg("vae attention head dim must be 32");
    if (d.ms_kernel != 3 && d.ms_kernel != 5)
        throw InvalidArg("depthwise_conv2d_same only supports 3x3 or 5x5 kernels");
    if (d.blocks[0].channels > 256) throw InvalidArg("vae decoder conv_out supports at most 256 input channels");
    const int Cin = d.blocks[d.n_blocks - 1].channels;
    if (Cin % d.latent_channels != 0)
        throw InvalidArg("vae decoder conv_in output channels must be divisible by latent channels");
    for (int i = 0; i < d.n_blocks; ++i) {
        const VaeBlockDims& b = d.blocks[i];
        if (b.channels < 8 || b.channels % 8 != 0 || b.layers < 0)
            throw InvalidArg("vae up block channels must be a positive multiple of 8");
        if (b.has_upsample && i == d.n_blocks - 1) throw InvalidArg("the innermost vae up block has no upsample");
        if (!b.has_upsample && i < d.n_blocks - 1)
            throw InvalidArg("every vae up block but the innermost starts with an upsample");
        if (b.has_upsample && (4 * b.channels) % d.blocks[i + 1].channels != 0)
            throw InvalidArg("VAE upsample shortcut channel ratio is invalid");
        if (!b.is_res_block && b.layers > 0 && b.channels % d.head_dim != 0)
            throw InvalidArg("VAE attention inner_dim must be divisible by attention_head_dim");
    }
}

void VaeDecoder::upload(const VaeDims& d, const float* const* tensors) {
    vae_validate(d);
    for (size_t i = 0; i < vae_tensor_count(d); ++i)
        if (!tensors[i]) throw InvalidArg("vae weight table has a missing tensor");
    d_ = d;
    have_ = false;
    if (eng_.mode() == kModeBf16) upload_impl<bf16>(tensors);
    else upload_impl<float>(tensors);
    SANA_CUDA(cudaDeviceSynchronize());
    ws_key_ = -1;
    have_ = true;
}

template <class T>
void VaeDecoder::upload_impl(const float* const* t) {
    const VaeDims& d = d_;
    const int n = d.n_blocks, Cl = d.latent_channels, C0 = d.blocks[0].channels, Cn = d.blocks[n - 1].channels;
    const int k = d.ms_kernel, hd = d.head_dim;
    put<float>(cin_w_, conv_in_layout(t[0], Cn, Cl));
    put<float>(cin_b_, copy_of(t[1], Cn));
    put<float>(nout_w_, copy_of(t[2], C0));
    put<float>(nout_b_, copy_of(t[3], C0));
    put<float>(cout_w_, tap_major(t[4], d.out_channels, C0));
    put<float>(cout_b_, copy_of(t[5], d.out_channels));
    blocks_.clear();
    blocks_.resize(n);
    size_t j = 6;
    for (int i = 0; i < n; ++i) {
        const VaeBlockDims& bd = d.blocks[i];
        Block& blk = blocks_[i];
        const int C = bd.channels;
        const size_t CC = static_cast<size_t>(C);
        if (bd.has_upsample) {
            put<T>(blk.upw, tap_major(t[j], C, d.blocks[i + 1].channels));
            if (sizeof(T) == 2) {
                const int Cin = d.blocks[i + 1].channels;
                const std::vector<float> w4 = parity_weights(t[j], C, Cin);
                put<T>(blk.upw4, w4);
                if (C <= 128) {
                    put<T>(blk.upw4p, pair_parity(w4, C, Cin));
                    put<float>(blk.upb2, twice(t[j + 1], CC));
                }
            }
            put<float>(blk.upb, copy_of(t[j + 1], CC));
            j += 2;
        }
        blk.layers.resize(bd.layers);
        for (int l = 0; l < bd.layers; ++l) {
            Layer& L = blk.layers[l];
            if (bd.is_res_block) {
                put<T>(L.c1w, tap_major(t[j], C, C));
                put<float>(L.c1b, copy_of(t[j + 1], CC));
                put<T>(L.c2w, tap_major(t[j + 2], C, C));
                if (sizeof(T) == 2 && C <= 128) {
                    put<T>(L.c1w2, pair_conv3x3(t[j], C, C));
                    put<float>(L.c1b2, twice(t[j + 1], CC));
                    put<T>(L.c2w2, pair_conv3x3(t[j + 2], C, C));
                }
                put<float>(L.n1w, copy_of(t[j + 3], CC));
                put<float>(L.n1b, copy_of(t[j + 4], CC));
                j += 5;
            } else {
                const int heads = C / hd;
                std::vector<float> qkv(3 * CC * CC);
                for (int m = 0; m < 3; ++m) std::memcpy(&qkv[m * CC * CC], t[j + m], CC * CC * sizeof(float));
                put<T>(L.wqkv, permute_groups(qkv, heads, hd, CC));
                put<float>(L.msdw, group_transpose(permute_groups(copy_of(t[j + 3], 3 * CC * k * k), heads, hd,
                                                                  static_cast<size_t>(k * k)),
                                                   static_cast<size_t>(k * k)));
                put<float>(L.msgw, group_transpose(permute_groups(copy_of(t[j + 4], 3 * CC * hd), heads, hd,
                                                                  static_cast<size_t>(hd)),
                                                   static_cast<size_t>(hd)));
                put<T>(L.wout, copy_of(t[j + 5], CC * 2 * CC));
                put<float>(L.n1w, copy_of(t[j + 6], CC));
                put<float>(L.n1b, copy_of(t[j + 7], CC));
                put<T>(L.winv, copy_of(t[j + 8], 8 * CC * CC));
                put<float>(L.binv, copy_of(t[j + 9], 8 * CC));
                put<float>(L.wdw, copy_of(t[j + 10], 8 * CC * 9));
                put<float>(L.bdw, copy_of(t[j + 11], 8 * CC));
                put<T>(L.wpt, copy_of(t[j + 12], CC * 4 * CC));
                put<float>(L.n2w, copy_of(t[j + 13], CC));
                put<float>(L.n2b, copy_of(t[j + 14], CC));
                j += 15;
            }
        }
    }
}

void VaeDecoder::ensure_workspace(int B, int h, int w) {
    // the patch buffer's size depends on which shapes take the implicit path
    const long long key = (static_cast<long long>(B) << 40) ^ (static_cast<long long>(h) << 20) ^ w ^
                          (static_cast<long long>(implicit_ok(128, 128, 64)) << 62);
    if (key == ws_key_) return;
    const size_t as = eng_.mode() == kModeBf16 ? 2 : 4;
    size_t x = 0, col = 0, qkv = 0, merged = 0, inv = 0, glu = 0, partial = 0;
    long long H = h, W = w;
    const int n = d_.n_blocks;
    x = static_cast<size_t>(B) * H * W * d_.blocks[n - 1].channels;
    for (int i = n - 1; i >= 0; --i) {
        const VaeBlockDims& bd = d_.blocks[i];
        const size_t C = static_cast<size_t>(bd.channels);
        if (bd.has_upsample) {
            const int Cin = d_.blocks[i + 1].channels;
            if (!implicit_ok(static_cast<int>(H), static_cast<int>(W), Cin) || bd.channels % 8 != 0)
                col = std::max(col, static_cast<size_t>(B * H * W) * 4 * 9 * Cin);
            H *= 2;
            W *= 2;
        }
        const size_t P = static_cast<size_t>(B * H * W);
        x = std::max(x, P * C);
        if (bd.layers == 0) continue;
        if (bd.is_res_block) {
            if (!implicit_ok(static_cast<int>(H), static_cast<int>(W), static_cast<int>(C))) col = std::max(col, P * 9 * C);
        } else {
            qkv = std::max(qkv, P * 3 * C);
            merged = std::max(merged, P * 2 * C);
            inv = std::max(inv, P * 8 * C);
            glu = std::max(glu, P * 4 * C);
            const int heads = static_cast<int>(C) / d_.head_dim;
            partial = std::max(partial, static_cast<size_t>(B) * heads * (linattn_chunks(static_cast<int>(H * W)) + 1) *
                                            (d_.head_dim + 1) * d_.head_dim);
        }
    }
    x_.ensure(x * as);
    y_.ensure(x * as);
    g_.ensure(x * as);
    if (eng_.mode() == kModeBf16) par_.ensure(x * as);
    if (col) col_.ensure(col * as);
    if (qkv) {
        qkv_.ensure(qkv * as);
        ms_.ensure(qkv * as);
        merged_.ensure(merged * as);
        inv_.ensure(inv * as);
        glu_.ensure(glu * as);
        partial_.ensure(partial * 4);
    }
    ws_key_ = key;
}

void VaeDecoder::decode(const float* lat_d, int B, int h, int w, float* out_d) {
    if (!have_) throw std::runtime_error("vae weights not uploaded");
    if (B < 1 || h < 1 || w < 1) throw InvalidArg("vae decode latents must be rank 4");
    ensure_workspace(B, h, w);
    launches_ = 0;
    if (eng_.mode() == kModeBf16) decode_impl<bf16>(lat_d, B, h, w, out_d);
    else decode_impl<float>(lat_d, B, h, w, out_d);
}

void VaeDecoder::decode_host(const float* lat, int B, int h, int w, float* out) {
    if (!have_) throw std::runtime_error("vae weights not uploaded");
    if (B < 1 || h < 1 || w < 1) throw InvalidArg("vae decode latents must be rank 4");
    const int up = 1 << (d_.n_blocks - 1);
    const size_t nin = static_cast<size_t>(B) * d_.latent_channels * h * w;
    const size_t nout = static_cast<size_t>(B) * d_.out_channels * (h * up) * (w * up);
    lat_in_.ensure(nin * 4);
    img_out_.ensure(nout * 4);
    const cudaStream_t st = eng_.stream();
    SANA_CUDA(cudaMemcpyAsync(lat_in_.get(), lat, nin * 4, cudaMemcpyHostToDevice, st));
    decode(lat_in_.as<float>(), B, h, w, img_out_.as<float>());
    SANA_CUDA(cudaMemcpyAsync(out, img_out_.get(), nout * 4, cudaMemcpyDeviceToHost, st));
    SANA_CUDA(cudaStreamSynchronize(st));
    eng_.check_device_error();
}

template <class T>
void VaeDecoder::gemm_rows(const T* A, long long M, int K, const DevBuf& w, const float* bias, int N, int act, T* out) {
    GemmProblem p;
    p.A = A;
    p.lda = K;
    p.B = w.get();
    p.ldb = K;
    p.M = static_cast<int>(M);
    p.N = N;
    p.K = K;
    p.a_bf16 = p.b_bf16 = sizeof(T) == 2 ? 1 : 0;
    p.ep.bias = bias;
    p.ep.act = act;
    p.ep.out = out;
    p.ep.out_bf16 = sizeof(T) == 2 ? 1 : 0;
    p.ep.ldo = N;
    p.require_tc = 1;
    gemm(p, eng_.err(), eng_.stream(), eng_.num_sms());
    ++launches_;
}

bool VaeDecoder::implicit_ok(int H, int W, int Cin) const {
    if (eng_.mode() != kModeBf16) return false;
    // SANA_VAE_CONV=im2col selects the patch-gather path for every shape (a cross-check)
    const char* v = std::getenv("SANA_VAE_CONV");
    if (v && std::string(v) == "im2col") return false;
    GemmProblem p;
    p.conv.H = H;
    p.conv.W = W;
    p.conv.C = Cin;
    p.M = H * W;
    p.N = 16;
    p.K = 9 * Cin;
    p.ldb = p.K;
    p.A = p.B = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
    return gemm_conv_supported(p);
}

bool VaeDecoder::pair_ok(int H, int W, int Cin, int Cout) const {
    if (!implicit_ok(H, W, Cin) || Cout > 128 || Cout % 8 != 0 || W % 2 != 0) return false;
    // SANA_VAE_PAIR=0 keeps one pixel per product row everywhere (a cross-check)
    const char* v = std::getenv("SANA_VAE_PAIR");
    if (v && std::string(v) == "0") return false;
    GemmProblem p;
    p.conv.H = H;
    p.conv.W = W / 2;
    p.conv.C = 2 * Cin;
    p.conv.kw = 4;
    p.conv.pair = 1;
    p.M = H * W / 2;
    p.N = 2 * Cout;
    p.K = 12 * Cin;
    p.ldb = p.K;
    p.A = p.B = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
    return gemm_conv_supported(p);
}

template <class T>
void VaeDecoder::conv_gemm(const T* in, int B, int H, int W, int Cin, int kh, int kw, int oy, int ox, const void* w,
                           const float* bias, int Cout, int act, T* out, bool pair) {
    GemmProblem p;
    p.A = in;
    p.lda = Cin;
    p.B = w;
    p.ldb = static_cast<long long>(kh) * kw * Cin;
    p.M = B * H * W / (pair ? 2 : 1);
    p.N = Cout * (pair ? 2 : 1);
    p.K = kh * kw * Cin;
    p.a_bf16 = p.b_bf16 = 1;
    p.conv.H = H;
    p.conv.W = pair ? W / 2 : W;
    p.conv.C = pair ? 2 * Cin : Cin;
    p.conv.pair = pair ? 1 : 0;
    p.conv.kh = kh;
    p.conv.kw = kw;
    p.conv.oy = oy;
    p.conv.ox = ox;
    p.ep.bias = bias;
    p.ep.act = act;
    p.ep.out = out;
    p.ep.out_bf16 = 1;
    p.ep.ldo = p.N;
    gemm(p, eng_.err(), eng_.stream(), eng_.num_sms());
    ++launches_;
}

template <class T>
void VaeDecoder::upsample_conv(const T* in, int B, int H, int W, int Cin, const Block& blk, int Cout, T* out) {
    const cudaStream_t st = eng_.stream();
    if constexpr (sizeof(T) == 2) {
        if (implicit_ok(H, W, Cin) && Cout % 8 == 0) {
            // four 2x2 convolutions on the low-resolution image, one per output parity
            T* par = par_.as<T>();
            const long long plane = static_cast<long long>(B) * H * W * Cout;
            const bool pair = pair_ok(H, W, Cin, Cout) && blk.upw4p.get();
            for (int ij = 0; ij < 4; ++ij) {
                if (pair)  // pixel pairs: 2x3 tap columns, 2 Cout outputs per row
                    conv_gemm<T>(in, B, H, W, Cin, 2, 3, (ij >> 1) - 1, (ij & 1) - 1,
                                 blk.upw4p.as<T>() + static_cast<long long>(ij) * 2 * Cout * 6 * Cin,
                                 blk.upb2.as<float>(), Cout, kActNone, par + ij * plane, true);
                else
                    conv_gemm<T>(in, B, H, W, Cin, 2, 2, (ij >> 1) - 1, (ij & 1) - 1,
                                 blk.upw4.as<T>() + static_cast<long long>(ij) * Cout * 4 * Cin, blk.upb.as<float>(),
                                 Cout, kActNone, par + ij * plane);
            }
            const dim3 grid(blocks_for(4LL * H * W * (Cout / 8)), B);
            shuffle_shortcut_kernel<<<grid, 256, 0, st>>>(par, in, B, H, W, Cin, Cout, out);
            SANA_CUDA(cudaGetLastError());
            ++launches_;
            return;
        }
    }
    {
        conv3x3<T>(in, B, H, W, Cin, true, blk.upw, blk.upb.as<float>(), Cout, kActNone, out);
        const long long nout = static_cast<long long>(B) * (2 * H) * (2 * W) * Cout;
        up_shortcut_kernel<T><<<blocks_for(nout), 256, 0, st>>>(out, in, B, H, W, Cin, Cout);
    }
    SANA_CUDA(cudaGetLastError());
    ++launches_;
}

template <class T>
void VaeDecoder::conv3x3(const T* in, int B, int H, int W, int Cin, bool upsample, const DevBuf& w, const float* bias,
                         int Cout, int act, T* out) {
    if (!upsample && sizeof(T) == 2 && implicit_ok(H, W, Cin)) {
        conv_gemm<T>(in, B, H, W, Cin, 3, 3, -1, -1, w.get(), bias, Cout, act, out);
        return;
    }
    const int up = upsample ? 1 : 0;
    T* col = col_.as<T>();
    const size_t need = static_cast<size_t>(B) * (H << up) * (W << up) * 9 * Cin * sizeof(T);
    if (col_.bytes() < need) throw std::runtime_error("vae patch buffer smaller than the convolution needs");
    launch_im2col<T>(in, B, H, W, Cin, up, col, eng_.stream());
    ++launches_;
    const long long P = static_cast<long long>(B) * (H << up) * (W << up);
    gemm_rows<T>(col, P, 9 * Cin, w, bias, Cout, act, out);
}

template <class T>
void VaeDecoder::decode_impl(const float* lat_d, int B, int h, int w, float* out_d) {
    const VaeDims& d = d_;
    const cudaStream_t st = eng_.stream();
    const int n = d.n_blocks;
    int C = d.blocks[n - 1].channels, H = h, W = w;
    T* x = x_.as<T>();
    T* y = y_.as<T>();
    T* g = g_.as<T>();
    auto rms = [&](const T* src, long long rows, int Cc, const DevBuf& nw, const DevBuf& nb, const T* resid, int relu,
                   T* dst) {
        const int grid = blocks_for(rows * 32, 256);
        const float* wn = nw.as<float>();
        const float* bn = nb.as<float>();
        // rows per warp: enough loads in flight per warp for the narrow rows
        auto vgrid = [&](int rpw) { return blocks_for(rows, 8 * rpw); };
        if constexpr (sizeof(T) == 2) {
            if (Cc == 128) {
                rms_rows_vec_kernel<4, 1, 4><<<vgrid(4), 256, 0, st>>>(src, rows, Cc, wn, bn, 1e-5f, resid, relu, dst);
            } else if (Cc == 256) {
                rms_rows_vec_kernel<8, 1, 4><<<vgrid(4), 256, 0, st>>>(src, rows, Cc, wn, bn, 1e-5f, resid, relu, dst);
            } else if (Cc == 512) {
                rms_rows_vec_kernel<8, 2, 2><<<vgrid(2), 256, 0, st>>>(src, rows, Cc, wn, bn, 1e-5f, resid, relu, dst);
            } else if (Cc == 1024) {
                rms_rows_vec_kernel<8, 4, 1><<<vgrid(1), 256, 0, st>>>(src, rows, Cc, wn, bn, 1e-5f, resid, relu, dst);
            } else {
                rms_rows_kernel<T><<<grid, 256, 0, st>>>(src, rows, Cc, wn, bn, 1e-5f, resid, relu, dst);
            }
        } else {
            rms_rows_kernel<T><<<grid, 256, 0, st>>>(src, rows, Cc, wn, bn, 1e-5f, resid, relu, dst);
        }
        SANA_CUDA(cudaGetLastError());
        ++launches_;
    };
    {
        const long long pix = static_cast<long long>(B) * H * W;
        vae_conv_in_kernel<T><<<blocks_for(pix, kCinPix), 256, 0, st>>>(lat_d, B, d.latent_channels, H, W,
                                                                       cin_w_.as<float>(), cin_b_.as<float>(),
                                                                       1.0f / d.scaling_factor, C, x);
        SANA_CUDA(cudaGetLastError());
        ++launches_;
    }
    for (int i = n - 1; i >= 0; --i) {
        const VaeBlockDims& bd = d.blocks[i];
        Block& blk = blocks_[i];
        if (bd.has_upsample) {
            const int Cin = C;
            C = bd.channels;
            upsample_conv<T>(x, B, H, W, Cin, blk, C, y);
            H *= 2;
            W *= 2;
            std::swap(x, y);
        }
        const long long P = static_cast<long long>(B) * H * W;
        for (Layer& L : blk.layers) {
            if (bd.is_res_block) {
                if (sizeof(T) == 2 && L.c1w2.get() && pair_ok(H, W, C, C)) {
                    // 128-channel levels: pixel-pair rows make the product 256 wide
                    conv_gemm<T>(x, B, H, W, C, 3, 4, -1, -1, L.c1w2.get(), L.c1b2.as<float>(), C, kActSilu, g, true);
                    conv_gemm<T>(g, B, H, W, C, 3, 4, -1, -1, L.c2w2.get(), nullptr, C, kActNone, y, true);
                } else {
                    conv3x3<T>(x, B, H, W, C, false, L.c1w, L.c1b.as<float>(), C, kActSilu, g);
                    conv3x3<T>(g, B, H, W, C, false, L.c2w, nullptr, C, kActNone, y);
                }
                rms(y, P, C, L.n1w, L.n1b, x, 0, g);
                std::swap(x, g);
            } else {
                const int heads = C / d.head_dim;
                T* qkv = qkv_.as<T>();
                T* ms = ms_.as<T>();
                T* merged = merged_.as<T>();
                gemm_rows<T>(x, P, C, L.wqkv, nullptr, 3 * C, kActNone, qkv);
                const dim3 grid(ceil_div(W, kMsTileX) * ceil_div(H, kMsTileY), 3 * heads, B);
                if (d.ms_kernel == 5)
                    ms_branch_kernel<T, 5><<<grid, 256, 0, st>>>(qkv, B, H, W, 3 * C, L.msdw.as<float>(),
                                                                L.msgw.as<float>(), ms);
                else
                    ms_branch_kernel<T, 3><<<grid, 256, 0, st>>>(qkv, B, H, W, 3 * C, L.msdw.as<float>(),
                                                                L.msgw.as<float>(), ms);
                SANA_CUDA(cudaGetLastError());
                ++launches_;
                const int T_ = H * W;
                linear_attention<T>(qkv, 3 * C, 0, qkv, 3 * C, C, 2 * C, B, T_, T_, heads, d.head_dim,
                                    partial_.as<float>(), merged, 2 * C, st);
                linear_attention<T>(ms, 3 * C, 0, ms, 3 * C, C, 2 * C, B, T_, T_, heads, d.head_dim,
                                    partial_.as<float>(), merged + C, 2 * C, st);
                launches_ += 4;
                gemm_rows<T>(merged, P, 2 * C, L.wout, nullptr, C, kActNone, y);
                rms(y, P, C, L.n1w, L.n1b, x, 0, g);
                std::swap(x, g);
                // GLUMBConv
                T* inv = inv_.as<T>();
                T* glu = glu_.as<T>();
                gemm_rows<T>(x, P, C, L.winv, L.binv.as<float>(), 8 * C, kActSilu, inv);
                depthwise_glu<T>(inv, 8 * C, B, H, W, 8 * C, L.wdw.as<float>(), L.bdw.as<float>(), glu, 4 * C,
                                 eng_.err(), st);
                ++launches_;
                gemm_rows<T>(glu, P, 4 * C, L.wpt, nullptr, C, kActNone, y);
                rms(y, P, C, L.n2w, L.n2b, x, 0, g);
                std::swap(x, g);
            }
        }
    }
    const long long P = static_cast<long long>(B) * H * W;
    rms(x, P, C, nout_w_, nout_b_, nullptr, 1, y);
    if constexpr (sizeof(T) == 2) {
        static PerDeviceOnce attr;
        if (attr.pending()) {  // weights of up to 256 channels: 36 KB dynamic + the 20 KB halo
            const int smem_max = 9 * 256 * static_cast<int>(sizeof(float4));
            SANA_CUDA(cudaFuncSetAttribute(vae_conv_out_bf16_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           smem_max));
            SANA_CUDA(cudaFuncSetAttribute(vae_conv_out_bf16_kernel<false>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
            attr.mark();
        }
        const dim3 grid(ceil_div(W, kCoTileX), ceil_div(H, kCoTileY), B);
        const size_t smem = static_cast<size_t>(9) * C * sizeof(float4);
        if (d.out_channels == 4)
            vae_conv_out_bf16_kernel<true><<<grid, 256, smem, st>>>(y, H, W, C, cout_w_.as<float>(), cout_b_.as<float>(),
                                                                    d.out_channels, out_d);
        else
            vae_conv_out_bf16_kernel<false><<<grid, 256, smem, st>>>(y, H, W, C, cout_w_.as<float>(),
                                                                     cout_b_.as<float>(), d.out_channels, out_d);
    } else {
        const dim3 grid(blocks_for(static_cast<long long>(H) * W, 8 * kConvOutPix), B);
        auto go = [&](auto kern, int cpl) {
            const size_t smem = static_cast<size_t>(9) * 4 * cpl * 32 * sizeof(float);
            kern<<<grid, 256, smem, st>>>(y, B, H, W, C, cout_w_.as<float>(), cout_b_.as<float>(), d.out_channels,
                                          out_d);
        };
        // channels per lane: C / 32 rounded up to 1, 2, 4 or 8 (C is a multiple of 8, so a
        // lane's chunk is either wholly below C or wholly past it)
        if (C <= 32) go(vae_conv_out_kernel<T, 1>, 1);
        else if (C <= 64) go(vae_conv_out_kernel<T, 2>, 2);
        else if (C <= 128) go(vae_conv_out_kernel<T, 4>, 4);
        else go(vae_conv_out_kernel<T, 8>, 8);
    }
    SANA_CUDA(cudaGetLastError());
    ++launches_;
    // x/y/g rotate through three buffers; keep the members pointing at distinct storage
}

}  // namespace sana
