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

// bf16 tiled path (half % 8 == 0, 16-byte aligned rows, W <= kTileW). A block owns 64
// channels of both halves and kTileRows full image rows of one sequence. The tile's input
// rows plus a one-pixel halo are copied to shared memory with asynchronous 16-byte copies
// (cp.async, zero-filled outside the image = the conv's zero padding), all issued before
// the first wait, so the block streams its ~87 KB at full bandwidth. Thread (channel quad,
// column) keeps its 4 data + 4 gate channels' 3x3 weights in registers and reads the 9 taps
// of each output from shared memory as 8-byte loads.
constexpr int kTileCh = 64;     // channels per half in a tile
constexpr int kTileRows = 8;
constexpr int kTileW = 64;      // widest image row handled by the tiled path
constexpr int kQuads = kTileCh / 4;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void unpack4(const uint2& u, float (&f)[4]) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

template <int WMAX>
__global__ void __launch_bounds__(256) dwglu_tile_kernel(const bf16* __restrict__ in, long long ldi, int S, int H,
                                                         int W, int half, const float* __restrict__ w,
                                                         const float* __restrict__ b, bf16* __restrict__ out,
                                                         long long ldo) {
    constexpr int PW = WMAX + 2;  // staged pixels per row (with halo)
    extern __shared__ __align__(16) bf16 tile[];  // [kTileRows+2][PW][2][kTileCh]
    const int c0 = blockIdx.y * kTileCh;          // first channel of the tile in each half
    const int nch = min(kTileCh, half - c0);      // a multiple of 8
    const int row_tiles = (H + kTileRows - 1) / kTileRows;
    const int s = blockIdx.x / row_tiles;
    const int y0 = (blockIdx.x % row_tiles) * kTileRows;
    {
        constexpr int kChunks = kTileCh / 8;  // 16-byte chunks per half-pixel
        const int total = (kTileRows + 2) * PW * 2 * kChunks;
        const uint32_t base = smem_u32(tile);
        for (int i = threadIdx.x; i < total; i += blockDim.x) {
            const int ck = i % kChunks;
            const int hf = (i / kChunks) % 2;
            const int px = (i / (2 * kChunks)) % PW;
            const int r = i / (2 * kChunks * PW);
            const int iy = y0 + r - 1, ix = px - 1;
            const bool ok = iy >= 0 && iy < H && ix >= 0 && ix < W && ck * 8 < nch;
            const bf16* src = ok ? in + ((static_cast<long long>(s) * H + iy) * W + ix) * ldi + hf * half + c0 + ck * 8
                                 : in;
            cp_async16(base + static_cast<uint32_t>(i) * 16u, src, ok ? 16u : 0u);
        }
    }
    const int q = threadIdx.x % kQuads;  // channel quad within the tile
    const int ch = c0 + q * 4;
    const bool qok = q * 4 < nch;
    float wd[4][9], wg[4][9], bd[4], bg[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int t = 0; t < 9; ++t) {
            wd[j][t] = qok ? w[static_cast<long long>(ch + j) * 9 + t] : 0.f;
            wg[j][t] = qok ? w[static_cast<long long>(half + ch + j) * 9 + t] : 0.f;
        }
        bd[j] = qok ? b[ch + j] : 0.f;
        bg[j] = qok ? b[half + ch + j] : 0.f;
    }
    cp_async_wait_all();
    __syncthreads();
    if (!qok) return;
    const int rows = min(kTileRows, H - y0);
    for (int x = threadIdx.x / kQuads; x < W; x += blockDim.x / kQuads) {
        for (int ry = 0; ry < rows; ++ry) {
            float dv[4] = {0.f, 0.f, 0.f, 0.f}, gv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const bf16* t = tile + (((ry + ky) * PW + (x + kx)) * 2) * kTileCh + q * 4;
                    float fd[4], fg[4];
                    unpack4(*reinterpret_cast<const uint2*>(t), fd);
                    unpack4(*reinterpret_cast<const uint2*>(t + kTileCh), fg);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        dv[j] = fmaf(fd[j], wd[j][ky * 3 + kx], dv[j]);
                        gv[j] = fmaf(fg[j], wg[j][ky * 3 + kx], gv[j]);
                    }
                }
            }
            const float o0 = (dv[0] + bd[0]) * silu(gv[0] + bg[0]);
            const float o1 = (dv[1] + bd[1]) * silu(gv[1] + bg[1]);
            const float o2 = (dv[2] + bd[2]) * silu(gv[2] + bg[2]);
            const float o3 = (dv[3] + bd[3]) * silu(gv[3] + bg[3]);
            uint2 pk;
            __nv_bfloat162 h0 = __floats2bfloat162_rn(o0, o1), h1 = __floats2bfloat162_rn(o2, o3);
            pk.x = *reinterpret_cast<uint32_t*>(&h0);
            pk.y = *reinterpret_cast<uint32_t*>(&h1);
            const long long pix = (static_cast<long long>(s) * H + y0 + ry) * W + x;
            *reinterpret_cast<uint2*>(out + pix * ldo + ch) = pk;
        }
    }
}

template <int WMAX>
size_t dwglu_tile_smem() {
    return sizeof(bf16) * (kTileRows + 2) * (WMAX + 2) * 2 * kTileCh;
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
    if (vec && W <= kTileW) {
        const int tiles = ceil_div(half, kTileCh);
        const int row_tiles = ceil_div(H, kTileRows);
        const dim3 grid(static_cast<unsigned>(S * row_tiles), tiles);
        if (W <= 32) {
            static bool a32 = false;
            if (!a32) {
                SANA_CUDA(cudaFuncSetAttribute(dwglu_tile_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(dwglu_tile_smem<32>())));
                a32 = true;
            }
            dwglu_tile_kernel<32><<<grid, 256, dwglu_tile_smem<32>(), st>>>(
                reinterpret_cast<const bf16*>(in), ldi, S, H, W, half, w, b, reinterpret_cast<bf16*>(out), ldo);
        } else {
            static bool a64 = false;
            if (!a64) {
                SANA_CUDA(cudaFuncSetAttribute(dwglu_tile_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(dwglu_tile_smem<64>())));
                a64 = true;
            }
            dwglu_tile_kernel<64><<<grid, 256, dwglu_tile_smem<64>(), st>>>(
                reinterpret_cast<const bf16*>(in), ldi, S, H, W, half, w, b, reinterpret_cast<bf16*>(out), ldo);
        }
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
