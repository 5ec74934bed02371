// Mix-FFN middle: depthwise 3x3 conv with zero padding and bias over all E channels of the
// NHWC token grid, then the GLU gate out[c] = dw[c] * silu(dw[c + E/2])
// (depthwise_conv2d_3x3, common_ops.cpp:484-505, per-plane taps summed ky-major then kx,
// bias last; glumb_conv's split and gate, common_ops.cpp:745-758).
//
// The input is the SiLU-ed output of the inverted 1x1 conv, already token-major, so the
// reference's NCHW round trips (tokens_to_grid_4d / grid_to_tokens_3d) disappear. Each
// thread produces 8 consecutive output channels of one pixel with 128-bit loads of the 9
// taps of the data and gate halves; neighbouring pixels' re-reads are served by L1/L2,
// so DRAM traffic stays at one read of the input and one write of the output.
#include "kernels.h"

namespace sana {
namespace {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __bfloat1622float2(h[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}

// bf16, 8 channels per thread (half % 8 == 0, 16-byte aligned rows). A block owns a tile
// of kGroups x 8 channels of both halves; their 3x3 taps and biases are staged once in
// shared memory, tap-major, so every weight read is a conflict-free 16-byte load. Lane i of
// a warp handles channel group i of one pixel: input loads and output stores are 512-byte
// contiguous runs. Threads stride over pixels.
constexpr int kGroups = 32;  // channel groups (of 8) per block
constexpr int kPixLanes = 8; // pixels in flight per block (blockDim = kGroups * kPixLanes)

__global__ void __launch_bounds__(kGroups * kPixLanes) dwglu_vec8_kernel(const bf16* __restrict__ in, long long ldi,
                                                                         int S, int H, int W, int half,
                                                                         const float* __restrict__ w,
                                                                         const float* __restrict__ b,
                                                                         bf16* __restrict__ out, long long ldo) {
    __shared__ __align__(16) float ws[2][9][kGroups * 8];  // [half][tap][channel in tile]
    __shared__ __align__(16) float bs[2][kGroups * 8];
    const int groups = half / 8;
    const int g0 = blockIdx.y * kGroups;
    const int ng = min(kGroups, groups - g0);
    for (int i = threadIdx.x; i < 2 * 9 * kGroups * 8; i += blockDim.x) {
        const int hf = i / (9 * kGroups * 8);
        const int rem = i % (9 * kGroups * 8);
        const int c = rem / 9, tap = rem % 9;  // coalesced read of w[(ch)*9 + tap]
        const int ch = g0 * 8 + c;
        ws[hf][tap][c] = (c < ng * 8) ? w[(static_cast<long long>(hf) * half + ch) * 9 + tap] : 0.f;
    }
    for (int i = threadIdx.x; i < 2 * kGroups * 8; i += blockDim.x) {
        const int hf = i / (kGroups * 8), c = i % (kGroups * 8);
        bs[hf][c] = (c < ng * 8) ? b[static_cast<long long>(hf) * half + g0 * 8 + c] : 0.f;
    }
    __syncthreads();
    const int gl = threadIdx.x % kGroups;
    if (gl >= ng) return;
    const int c0 = (g0 + gl) * 8;
    const long long pixels = static_cast<long long>(S) * H * W;
    for (long long pix = blockIdx.x * static_cast<long long>(kPixLanes) + threadIdx.x / kGroups; pix < pixels;
         pix += static_cast<long long>(gridDim.x) * kPixLanes) {
        const int x = static_cast<int>(pix % W);
        const int y = static_cast<int>((pix / W) % H);
        const long long sH = pix / (static_cast<long long>(W) * H) * H;
        float dv[8], gv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            dv[j] = 0.f;
            gv[j] = 0.f;
        }
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
            const int iy = y + ky - 1;
            if (iy < 0 || iy >= H) continue;
#pragma unroll
            for (int kx = 0; kx < 3; ++kx) {
                const int ix = x + kx - 1;
                if (ix < 0 || ix >= W) continue;
                const bf16* src = in + ((sH + iy) * W + ix) * ldi;
                float fd[8], fg[8];
                unpack8(*reinterpret_cast<const uint4*>(src + c0), fd);
                unpack8(*reinterpret_cast<const uint4*>(src + half + c0), fg);
                const int tap = ky * 3 + kx;
                const float4 wd0 = *reinterpret_cast<const float4*>(&ws[0][tap][gl * 8]);
                const float4 wd1 = *reinterpret_cast<const float4*>(&ws[0][tap][gl * 8 + 4]);
                const float4 wg0 = *reinterpret_cast<const float4*>(&ws[1][tap][gl * 8]);
                const float4 wg1 = *reinterpret_cast<const float4*>(&ws[1][tap][gl * 8 + 4]);
                const float wdv[8] = {wd0.x, wd0.y, wd0.z, wd0.w, wd1.x, wd1.y, wd1.z, wd1.w};
                const float wgv[8] = {wg0.x, wg0.y, wg0.z, wg0.w, wg1.x, wg1.y, wg1.z, wg1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    dv[j] = fmaf(fd[j], wdv[j], dv[j]);
                    gv[j] = fmaf(fg[j], wgv[j], gv[j]);
                }
            }
        }
        uint4 pk;
        uint32_t* pw = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const float o0 = (dv[j] + bs[0][gl * 8 + j]) * silu(gv[j] + bs[1][gl * 8 + j]);
            const float o1 = (dv[j + 1] + bs[0][gl * 8 + j + 1]) * silu(gv[j + 1] + bs[1][gl * 8 + j + 1]);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(o0, o1);
            pw[j / 2] = *reinterpret_cast<uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(out + pix * ldo + c0) = pk;
    }
}

// Any type / channel count: one output channel per thread.
template <class T>
__global__ void dwglu_scalar_kernel(const T* __restrict__ in, long long ldi, int S, int H, int W, int half,
                                    const float* __restrict__ w, const float* __restrict__ b, T* __restrict__ out,
                                    long long ldo) {
    const long long total = static_cast<long long>(S) * H * W * half;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % half);
        const long long pix = i / half;
        const int x = static_cast<int>(pix % W);
        const int y = static_cast<int>((pix / W) % H);
        const long long s = pix / (static_cast<long long>(W) * H);
        float dv = 0.f, gv = 0.f;
        for (int ky = 0; ky < 3; ++ky) {
            const int iy = y + ky - 1;
            if (iy < 0 || iy >= H) continue;
            for (int kx = 0; kx < 3; ++kx) {
                const int ix = x + kx - 1;
                if (ix < 0 || ix >= W) continue;
                const T* src = in + ((s * H + iy) * W + ix) * ldi;
                dv = fmaf(to_f(src[c]), w[c * 9 + ky * 3 + kx], dv);
                gv = fmaf(to_f(src[half + c]), w[(half + c) * 9 + ky * 3 + kx], gv);
            }
        }
        dv += b[c];
        gv += b[half + c];
        out[pix * ldo + c] = from_f<T>(dv * silu(gv));
    }
}

__global__ void depthwise_plain_kernel(const float* __restrict__ in, int S, int H, int W, int C,
                                       const float* __restrict__ w, const float* __restrict__ b,
                                       float* __restrict__ out) {
    const long long total = static_cast<long long>(S) * H * W * C;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        const long long pix = i / C;
        const int x = static_cast<int>(pix % W);
        const int y = static_cast<int>((pix / W) % H);
        const long long s = pix / (static_cast<long long>(W) * H);
        float acc = 0.f;
        for (int ky = 0; ky < 3; ++ky) {
            const int iy = y + ky - 1;
            if (iy < 0 || iy >= H) continue;
            for (int kx = 0; kx < 3; ++kx) {
                const int ix = x + kx - 1;
                if (ix < 0 || ix >= W) continue;
                acc = fmaf(in[((s * H + iy) * W + ix) * C + c], w[c * 9 + ky * 3 + kx], acc);
            }
        }
        if (b) acc += b[c];
        out[i] = acc;
    }
}

int grid_for(long long n) {
    long long g = (n + 255) / 256;
    if (g > 148LL * 16) g = 148LL * 16;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

template <class T>
void depthwise_glu(const T* in, long long ldi, int S, int H, int W, int E, const float* w, const float* b, T* out,
                   long long ldo, cudaStream_t st) {
    SANA_REQUIRE(E % 2 == 0, "channel count must be even");
    const int half = E / 2;
    const long long pixels = static_cast<long long>(S) * H * W;
    if (pixels == 0 || half == 0) return;
    bool vec = sizeof(T) == 2 && half % 8 == 0 && ldi % 8 == 0 && ldo % 8 == 0 &&
               (reinterpret_cast<uintptr_t>(in) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    if (vec) {
        const int tiles = ceil_div(half / 8, kGroups);
        long long px_blocks = (pixels + kPixLanes - 1) / kPixLanes;
        const long long cap = (148LL * 8 + tiles - 1) / tiles * 4;  // ~32 resident blocks per SM in total
        if (px_blocks > cap) px_blocks = cap;
        dwglu_vec8_kernel<<<dim3(static_cast<unsigned>(px_blocks), tiles), kGroups * kPixLanes, 0, st>>>(
            reinterpret_cast<const bf16*>(in), ldi, S, H, W, half, w, b, reinterpret_cast<bf16*>(out), ldo);
    } else {
        dwglu_scalar_kernel<T><<<grid_for(pixels * half), 256, 0, st>>>(in, ldi, S, H, W, half, w, b, out, ldo);
    }
    SANA_CUDA(cudaGetLastError());
}

void depthwise3x3(const float* in, int S, int H, int W, int C, const float* w, const float* b, float* out,
                  cudaStream_t st) {
    const long long n = static_cast<long long>(S) * H * W * C;
    if (n == 0) return;
    depthwise_plain_kernel<<<grid_for(n), 256, 0, st>>>(in, S, H, W, C, w, b, out);
    SANA_CUDA(cudaGetLastError());
}

template void depthwise_glu<float>(const float*, long long, int, int, int, int, const float*, const float*, float*,
                                   long long, cudaStream_t);
template void depthwise_glu<bf16>(const bf16*, long long, int, int, int, int, const float*, const float*, bf16*,
                                  long long, cudaStream_t);

}  // namespace sana
