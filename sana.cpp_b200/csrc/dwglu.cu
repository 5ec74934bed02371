// Mix-FFN middle: depthwise 3x3 conv with zero padding and bias over all E channels of the
// NHWC token grid, then the GLU gate out[c] = dw[c] * silu(dw[c + E/2])
// (depthwise_conv2d_3x3, common_ops.cpp:484-505, per-plane taps summed ky-major then kx,
// bias last; glumb_conv's split and gate, common_ops.cpp:745-758).
//
// The input is the SiLU-ed output of the inverted 1x1 conv, already token-major, so the
// reference's NCHW round trips (tokens_to_grid_4d / grid_to_tokens_3d) disappear.
#include "kernels.h"

namespace sana {
namespace {

// bf16 tiled path (half % 8 == 0, 16-byte aligned rows, W <= kTileW). A block owns 64
// channels of both halves and kTileRows full image rows of one sequence. The tile's input
// rows plus a one-pixel halo are copied to shared memory with asynchronous 16-byte copies
// (cp.async, zero-filled outside the image = the conv's zero padding), all issued before
// the first wait, so the block streams its ~87 KB at full bandwidth.
constexpr int kTileCh = 64;     // channels per half in a tile
constexpr int kTileRows = 8;
constexpr int kTileW = 64;      // widest image row handled by the tiled path

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Packed fp32 pair arithmetic (sm_100 f32x2): one instruction for two channels.
__device__ __forceinline__ uint64_t pk2(float2 v) {
    return (static_cast<uint64_t>(__float_as_uint(v.y)) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 upk2(uint64_t u) {
    return make_float2(__uint_as_float(static_cast<uint32_t>(u)), __uint_as_float(static_cast<uint32_t>(u >> 32)));
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)), "l"(pk2(c)));
    return upk2(d);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
    return upk2(d);
}
// bf16 pair -> fp32 pair (exact: bf16 is the top half of an fp32)
__device__ __forceinline__ float2 bf2(uint32_t u) { return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u)); }

// Thread = (channel pair p of the tile = lane, column pair): it keeps its pair's 3x3 taps of
// both halves in registers and walks the tile's input rows top to bottom, loading the four
// pixels x0-1 .. x0+2 of each row once (4-byte shared loads, conflict-free across the warp)
// and adding row iy's taps into the three output rows iy-1, iy, iy+1 held in a rolling set
// of accumulators. Each output therefore receives its taps in the reference's order (ky
// major, then kx, from zero; bias last) with fp32 fused multiply-adds issued two channels
// at a time.
template <int WMAX>
__global__ void __launch_bounds__(256, 2) dwglu_tile_kernel(const bf16* __restrict__ in, long long ldi, int S, int H,
                                                            int W, int half, const float* __restrict__ w,
                                                            const float* __restrict__ b, bf16* __restrict__ out,
                                                            long long ldo) {
    constexpr int PW = WMAX + 2;  // staged pixels per row (with halo)
    constexpr int kPairs = kTileCh / 2;
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
    const int p = threadIdx.x % 32;  // channel pair within the tile
    const int ch = c0 + 2 * p;
    const bool pok = 2 * p < nch;
    float2 wv[9], wg[9], bv = make_float2(0.f, 0.f), bg = make_float2(0.f, 0.f);
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        wv[t] = pok ? make_float2(w[static_cast<long long>(ch) * 9 + t], w[static_cast<long long>(ch + 1) * 9 + t])
                    : make_float2(0.f, 0.f);
        wg[t] = pok ? make_float2(w[static_cast<long long>(half + ch) * 9 + t],
                                  w[static_cast<long long>(half + ch + 1) * 9 + t])
                    : make_float2(0.f, 0.f);
    }
    if (pok) {
        bv = make_float2(b[ch], b[ch + 1]);
        bg = make_float2(b[half + ch], b[half + ch + 1]);
    }
    cp_async_wait_all();
    __syncthreads();
    if (!pok) return;
    const int rows = min(kTileRows, H - y0);
    const uint32_t* t32 = reinterpret_cast<const uint32_t*>(tile);
    for (int x0 = 2 * (threadIdx.x / 32); x0 < W; x0 += 2 * (blockDim.x / 32)) {
        float2 acc[3][2][2];  // [output row slot][column][value, gate]
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int c = 0; c < 2; ++c) acc[a][c][0] = acc[a][c][1] = make_float2(0.f, 0.f);
#pragma unroll
        for (int r = 0; r < kTileRows + 2; ++r) {
            if (r >= rows + 2) break;
            float2 fv[4], fg[4];
            const uint32_t* rp = t32 + ((r * PW + x0) * 2) * kPairs + p;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                fv[j] = bf2(rp[(2 * j) * kPairs]);
                fg[j] = bf2(rp[(2 * j + 1) * kPairs]);
            }
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
                const int o = r - ky;  // the output row this input row feeds through tap row ky
                if (o < 0 || o >= kTileRows) continue;
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int kx = 0; kx < 3; ++kx) {
                        acc[o % 3][c][0] = fma2(fv[c + kx], wv[ky * 3 + kx], acc[o % 3][c][0]);
                        acc[o % 3][c][1] = fma2(fg[c + kx], wg[ky * 3 + kx], acc[o % 3][c][1]);
                    }
            }
            if (r >= 2) {  // output row r - 2 has all nine taps
                const int o = r - 2;
                const long long pix = (static_cast<long long>(s) * H + y0 + o) * W + x0;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const float2 v = add2(acc[o % 3][c][0], bv), g = add2(acc[o % 3][c][1], bg);
                    acc[o % 3][c][0] = acc[o % 3][c][1] = make_float2(0.f, 0.f);
                    if (x0 + c < W) {
                        const __nv_bfloat162 h = __floats2bfloat162_rn(v.x * silu_fast(g.x), v.y * silu_fast(g.y));
                        *reinterpret_cast<__nv_bfloat162*>(out + (pix + c) * ldo + ch) = h;
                    }
                }
            }
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
