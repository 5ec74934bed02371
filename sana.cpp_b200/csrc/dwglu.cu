// Mix-FFN middle: depthwise 3x3 conv with zero padding and bias over all E channels of the
// NHWC token grid, then the GLU gate out[c] = dw[c] * silu(dw[c + E/2])
// (depthwise_conv2d_3x3, common_ops.cpp:484-505, per-plane taps summed ky-major then kx,
// bias last; glumb_conv's split and gate, common_ops.cpp:745-758).
//
// The input is the SiLU-ed output of the inverted 1x1 conv, already token-major, so the
// reference's NCHW round trips (tokens_to_grid_4d / grid_to_tokens_3d) disappear.
#include "kernels.h"
#include "tma.h"

namespace sana {
namespace {

// bf16 tiled path (half % 8 == 0, 16-byte aligned rows, W <= kTileW). A block owns 64
// channels of both halves and kTileRows full image rows of one sequence. One thread loads
// the tile's input rows plus a one-pixel halo with two TMA copies (a 4-D box of
// [1 sequence, kTileRows + 2 rows, W + 2 pixels, 64 channels] per half); TMA reads the
// halo outside the image as zeros, which is the conv's zero padding.
constexpr int kTileCh = 64;     // channels per half in a tile
constexpr int kTileRows = 8;
constexpr int kTileW = 64;      // widest image row handled by the tiled path

// Staged pixels per image row: the row plus its halo, plus one more for odd widths so the
// last column pair's four-pixel window stays inside the row.
__host__ __device__ __forceinline__ int tile_pixels(int W) { return W + 2 + (W & 1); }

// Thread = (channel pair p of the tile = lane, column pair): it keeps its pair's 3x3 taps of
// both halves in registers and walks the tile's input rows top to bottom, loading the four
// pixels x0-1 .. x0+2 of each row once (4-byte shared loads, conflict-free across the warp)
// and adding row iy's taps into the three output rows iy-1, iy, iy+1 held in a rolling set
// of accumulators. Each output therefore receives its taps in the reference's order (ky
// major, then kx, from zero; bias last) with fp32 fused multiply-adds issued two channels
// at a time.
__global__ void __launch_bounds__(256, 2) dwglu_tile_kernel(const __grid_constant__ CUtensorMap map, int S, int H,
                                                            int W, int half, const float* __restrict__ w,
                                                            const float* __restrict__ b, bf16* __restrict__ out,
                                                            long long ldo, int* err) {
    constexpr int kPairs = kTileCh / 2;
    extern __shared__ __align__(16) unsigned char dyn[];
    __shared__ __align__(8) uint64_t bar_storage;
    // two boxes [kTileRows + 2][W + 2][kTileCh] (value half, gate half), 128-byte aligned
    bf16* tile = reinterpret_cast<bf16*>((reinterpret_cast<uintptr_t>(dyn) + 127) & ~uintptr_t(127));
    const int PW = tile_pixels(W);
    const int box = (kTileRows + 2) * PW * kTileCh;  // elements per half
    const int c0 = blockIdx.y * kTileCh;          // first channel of the tile in each half
    const int nch = min(kTileCh, half - c0);      // a multiple of 8
    const int row_tiles = (H + kTileRows - 1) / kTileRows;
    const int s = blockIdx.x / row_tiles;
    const int y0 = (blockIdx.x % row_tiles) * kTileRows;
    const uint32_t bar = smem_u32(&bar_storage);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * box * 2));
        tma_load_4d(&map, smem_u32(tile), bar, c0, -1, y0 - 1, s);
        tma_load_4d(&map, smem_u32(tile + box), bar, half + c0, -1, y0 - 1, s);
    }
    const int p = threadIdx.x % 32;  // channel pair within the tile
    const int ch = c0 + 2 * p;
    const bool pok = 2 * p < nch;
    uint64_t wv[9], wg[9], bv = 0, bg = 0;
#pragma unroll
    for (int t = 0; t < 9; ++t) {
        wv[t] = pok ? f2_make(w[static_cast<long long>(ch) * 9 + t], w[static_cast<long long>(ch + 1) * 9 + t]) : 0;
        wg[t] = pok ? f2_make(w[static_cast<long long>(half + ch) * 9 + t], w[static_cast<long long>(half + ch + 1) * 9 + t])
                    : 0;
    }
    if (pok) {
        bv = f2_make(b[ch], b[ch + 1]);
        bg = f2_make(b[half + ch], b[half + ch + 1]);
    }
    __syncthreads();  // the barrier is initialised before anyone waits on it
    if (!mbar_wait(bar, 0, err, kTimeout)) {
        if (threadIdx.x == 0) mbar_wait_quiet(bar, 0);  // let the copies land before the block exits
        return;
    }
    if (!pok) return;
    const int rows = min(kTileRows, H - y0);
    const uint32_t* t32 = reinterpret_cast<const uint32_t*>(tile);
    for (int x0 = 2 * (threadIdx.x / 32); x0 < W; x0 += 2 * (blockDim.x / 32)) {
        uint64_t acc[3][2][2];  // [output row slot][column][value, gate]; +0.0 pairs
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int c = 0; c < 2; ++c) acc[a][c][0] = acc[a][c][1] = 0;
#pragma unroll
        for (int r = 0; r < kTileRows + 2; ++r) {
            if (r >= rows + 2) break;
            uint64_t fv[4], fg[4];
            const uint32_t* rp = t32 + (r * PW + x0) * kPairs + p;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                fv[j] = f2_from_bf2(rp[j * kPairs]);
                fg[j] = f2_from_bf2(rp[box / 2 + j * kPairs]);
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
                    const uint64_t v = add2(acc[o % 3][c][0], bv);
                    const uint64_t g = add2(acc[o % 3][c][1], bg);
                    acc[o % 3][c][0] = acc[o % 3][c][1] = 0;
                    if (x0 + c < W) {
                        const float2 y = f2_split(mul2(v, silu2(g)));
                        *reinterpret_cast<__nv_bfloat162*>(out + (pix + c) * ldo + ch) = __floats2bfloat162_rn(y.x, y.y);
                    }
                }
            }
        }
    }
}

size_t dwglu_tile_smem(int W) {
    return sizeof(bf16) * (kTileRows + 2) * tile_pixels(W) * 2 * kTileCh + 128;
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
                   long long ldo, int* err, cudaStream_t st) {
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
        static bool attr = false;
        if (!attr) {
            SANA_CUDA(cudaFuncSetAttribute(dwglu_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(dwglu_tile_smem(kTileW))));
            attr = true;
        }
        // [S, H, W, channels] with the channel rows ldi apart; box = 64 channels x tile pixels
        // x (kTileRows + 2) rows x 1 sequence
        CUtensorMap map;
        const cuuint64_t dims[4] = {static_cast<cuuint64_t>(2 * half), static_cast<cuuint64_t>(W),
                                    static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(S)};
        const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ldi) * 2, static_cast<cuuint64_t>(ldi) * 2 * W,
                                       static_cast<cuuint64_t>(ldi) * 2 * W * H};
        const cuuint32_t box[4] = {static_cast<cuuint32_t>(kTileCh), static_cast<cuuint32_t>(tile_pixels(W)),
                                   static_cast<cuuint32_t>(kTileRows + 2), 1};
        tma_encode_tiled(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, in, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
        dwglu_tile_kernel<<<grid, 256, dwglu_tile_smem(W), st>>>(map, S, H, W, half, w, b,
                                                                  reinterpret_cast<bf16*>(out), ldo, err);
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
                                   long long, int*, cudaStream_t);
template void depthwise_glu<bf16>(const bf16*, long long, int, int, int, int, const float*, const float*, bf16*,
                                  long long, int*, cudaStream_t);

}  // namespace sana
