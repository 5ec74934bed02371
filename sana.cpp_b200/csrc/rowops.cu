// Row-wise and elementwise kernels of the denoiser step (see kernels.h for contracts).
#include "kernels.h"

namespace sana {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per row. Three passes over the row (it stays in L1): mean, centred variance,
// write — the order of tensor.cpp:243-265 (mean first, then sum of squared deviations).
template <class TO>
__global__ void ln_modulate_kernel(const float* __restrict__ x, long long rows, int C, int rows_per_seq,
                                   const float* __restrict__ gamma, const float* __restrict__ beta,
                                   const float* __restrict__ mod, long long mod_ld, int shift_idx, int scale_idx,
                                   float eps, TO* __restrict__ out) {
    const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * C;
    const bool vec = (C % 128 == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0);
    float s = 0.f;
    if (vec) {
        for (int c = lane * 4; c < C; c += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + c);
            s += (v.x + v.y) + (v.z + v.w);
        }
    } else {
        for (int c = lane; c < C; c += 32) s += xr[c];
    }
    const float mean = warp_sum(s) / static_cast<float>(C);
    float q = 0.f;
    if (vec) {
        for (int c = lane * 4; c < C; c += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + c);
            const float a = v.x - mean, b = v.y - mean, d = v.z - mean, e = v.w - mean;
            q += (a * a + b * b) + (d * d + e * e);
        }
    } else {
        for (int c = lane; c < C; c += 32) {
            const float d = xr[c] - mean;
            q += d * d;
        }
    }
    const float var = warp_sum(q) / static_cast<float>(C);
    const float inv_std = 1.0f / sqrtf(var + eps);
    const long long seq = row / rows_per_seq;
    const float* shift = mod ? mod + seq * mod_ld + static_cast<long long>(shift_idx) * C : nullptr;
    const float* scale = mod ? mod + seq * mod_ld + static_cast<long long>(scale_idx) * C : nullptr;
    TO* o = out + row * C;
    for (int c = lane; c < C; c += 32) {
        float v = (xr[c] - mean) * inv_std;
        if (gamma) v *= gamma[c];
        if (beta) v += beta[c];
        if (mod) v = v * (1.0f + scale[c]) + shift[c];
        o[c] = from_f<TO>(v);
    }
}

// Rows in registers (C = 128 * NV): a block of 8 warps takes 8 * RW consecutive rows, each
// warp RW of them (w, w + 8, ...; two when a row is at most 1024 wide, else one, so that the
// rows fit the registers), and every lane holds NV float4 of each row; the
// mean, then the centred variance come from the registers (the order of tensor.cpp:243-265),
// and the normalised, modulated rows are written with 8-byte (bf16) or 16-byte (fp32)
// stores. All of the block's row loads are in flight before anything else; meanwhile the
// block stages the shift and scale vectors of its first row's sequence in shared memory
// once, instead of every warp fetching them after its reductions.
constexpr int kLnWarps = 8;
template <int NV> constexpr int ln_rows_per_warp() { return NV <= 8 ? 2 : 1; }

template <class TO, int NV, int RW = ln_rows_per_warp<NV>()>
__global__ void __launch_bounds__(32 * kLnWarps, RW == 1 ? 4 : 2)
    ln_modulate_reg_kernel(const float* __restrict__ x, long long rows, int rows_per_seq,
                           const float* __restrict__ gamma, const float* __restrict__ beta,
                           const float* __restrict__ mod, long long mod_ld, int shift_idx, int scale_idx, float eps,
                           TO* __restrict__ out) {
    constexpr int C = 128 * NV;
    __shared__ float4 s_shift[32 * NV], s_scale[32 * NV];
    const long long row0 = static_cast<long long>(blockIdx.x) * (kLnWarps * RW);
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    float4 v[RW][NV];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const long long row = row0 + warp + r * kLnWarps;
        if (row < rows) {
            const float4* xr = reinterpret_cast<const float4*>(x + row * C);
#pragma unroll
            for (int i = 0; i < NV; ++i) v[r][i] = xr[lane + 32 * i];
        }
    }
    const long long seq0 = row0 / rows_per_seq;
    if (mod) {
        const float4* sh = reinterpret_cast<const float4*>(mod + seq0 * mod_ld + static_cast<long long>(shift_idx) * C);
        const float4* sc = reinterpret_cast<const float4*>(mod + seq0 * mod_ld + static_cast<long long>(scale_idx) * C);
        for (int i = threadIdx.x; i < 32 * NV; i += blockDim.x) {
            s_shift[i] = sh[i];
            s_scale[i] = sc[i];
        }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const long long row = row0 + warp + r * kLnWarps;
        if (row >= rows) break;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) s += (v[r][i].x + v[r][i].y) + (v[r][i].z + v[r][i].w);
        const float mean = warp_sum(s) / static_cast<float>(C);
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float a = v[r][i].x - mean, b = v[r][i].y - mean, c = v[r][i].z - mean, d = v[r][i].w - mean;
            q += (a * a + b * b) + (c * c + d * d);
        }
        const float var = warp_sum(q) / static_cast<float>(C);
        const float inv_std = 1.0f / sqrtf(var + eps);
        const long long seq = row / rows_per_seq;
        const bool staged = seq == seq0;
        const float* shift = mod ? mod + seq * mod_ld + static_cast<long long>(shift_idx) * C : nullptr;
        const float* scale = mod ? mod + seq * mod_ld + static_cast<long long>(scale_idx) * C : nullptr;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c = 4 * (lane + 32 * i);
            float o[4] = {(v[r][i].x - mean) * inv_std, (v[r][i].y - mean) * inv_std, (v[r][i].z - mean) * inv_std,
                          (v[r][i].w - mean) * inv_std};
            if (gamma) {
                const float4 g = *reinterpret_cast<const float4*>(gamma + c);
                o[0] *= g.x; o[1] *= g.y; o[2] *= g.z; o[3] *= g.w;
            }
            if (beta) {
                const float4 bb = *reinterpret_cast<const float4*>(beta + c);
                o[0] += bb.x; o[1] += bb.y; o[2] += bb.z; o[3] += bb.w;
            }
            if (mod) {
                const float4 sc = staged ? s_scale[lane + 32 * i] : *reinterpret_cast<const float4*>(scale + c);
                const float4 sh = staged ? s_shift[lane + 32 * i] : *reinterpret_cast<const float4*>(shift + c);
                o[0] = o[0] * (1.0f + sc.x) + sh.x;
                o[1] = o[1] * (1.0f + sc.y) + sh.y;
                o[2] = o[2] * (1.0f + sc.z) + sh.z;
                o[3] = o[3] * (1.0f + sc.w) + sh.w;
            }
            if constexpr (sizeof(TO) == 2) {
                __nv_bfloat162 h0 = __floats2bfloat162_rn(o[0], o[1]), h1 = __floats2bfloat162_rn(o[2], o[3]);
                uint2 pk;
                pk.x = *reinterpret_cast<uint32_t*>(&h0);
                pk.y = *reinterpret_cast<uint32_t*>(&h1);
                *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(out) + row * C + c) = pk;
            } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row * C + c) =
                    make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

template <class TO>
__global__ void rms_norm_kernel(const float* __restrict__ x, long long rows, int C, float eps,
                                const float* __restrict__ w, TO* __restrict__ out) {
    const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * C;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) s += xr[c] * xr[c];
    const float ms = warp_sum(s) / static_cast<float>(C);
    const float inv = 1.0f / sqrtf(ms + eps);
    TO* o = out + row * C;
    for (int c = lane; c < C; c += 32) {
        float v = xr[c] * inv;
        if (w) v *= w[c];
        o[c] = from_f<TO>(v);
    }
}

// In-place RMSNorm of rows of width C (row stride ld), fp32 math: one warp per row.
template <class T>
__global__ void rms_norm_rows_kernel(T* __restrict__ x, long long rows, int C, long long ld, float eps,
                                     const float* __restrict__ w) {
    const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    T* xr = x + row * ld;
    float s = 0.f;
    for (int c = lane; c < C; c += 32) {
        const float v = to_f(xr[c]);
        s += v * v;
    }
    const float inv = 1.0f / sqrtf(warp_sum(s) / static_cast<float>(C) + eps);
    for (int c = lane; c < C; c += 32) {
        float v = to_f(xr[c]) * inv;
        if (w) v *= w[c];
        xr[c] = from_f<T>(v);
    }
}

__global__ void block_modulation_kernel(const float* __restrict__ tmod, int S, int width,
                                        const float* __restrict__ tables, int n_blocks, float* __restrict__ mod) {
    const long long total = static_cast<long long>(n_blocks) * S * width;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int k = static_cast<int>(i % width);
        const long long bs = i / width;
        const int s = static_cast<int>(bs % S);
        const int b = static_cast<int>(bs / S);
        mod[i] = tmod[static_cast<long long>(s) * width + k] + tables[static_cast<long long>(b) * width + k];
    }
}

__global__ void final_modulation_kernel(const float* __restrict__ emb, int S, int C, const float* __restrict__ table,
                                        float* __restrict__ fmod) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S * C) return;
    const int s = i / C, c = i % C;
    fmod[static_cast<long long>(s) * 2 * C + c] = emb[i] + table[c];
    fmod[static_cast<long long>(s) * 2 * C + C + c] = emb[i] + table[C + c];
}

template <class TO>
__global__ void patch_tokens_kernel(const float* __restrict__ lat, int images, int seqs, int Cl, int HW,
                                    TO* __restrict__ out) {
    const long long total = static_cast<long long>(seqs) * HW * Cl;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % Cl);
        const long long r = i / Cl;
        const int t = static_cast<int>(r % HW);
        const int s = static_cast<int>(r / HW);
        const int img = s % images;
        out[i] = from_f<TO>(lat[(static_cast<long long>(img) * Cl + c) * HW + t]);
    }
}

template <class TO>
__global__ void broadcast_rows_kernel(const float* __restrict__ row, int S, int width, TO* __restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < S * width) out[i] = from_f<TO>(row[i % width]);
}

__global__ void kv_len_kernel(const float* __restrict__ bias, int S, int L, int* __restrict__ kv_len) {
    const int s = blockIdx.x;
    int last = -1;
    for (int j = threadIdx.x; j < L; j += blockDim.x) {
        if (bias[static_cast<long long>(s) * L + j] > -1000.0f) last = max(last, j);
    }
    __shared__ int red[32];
    for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = last;
    __syncthreads();
    if (threadIdx.x == 0) {
        int m = -1;
        for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) m = max(m, red[w]);
        kv_len[s] = (m < 0) ? L : m + 1;
    }
}

__global__ void cfg_scheduler_kernel(const float* __restrict__ noise, int images, int Cl, int HW,
                                     float* __restrict__ lat, float* __restrict__ hist_cur,
                                     const float* __restrict__ hist_prev, SchedCoef k) {
    const long long n = static_cast<long long>(images) * Cl * HW;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i % HW);
        const long long bc = i / HW;
        const int c = static_cast<int>(bc % Cl);
        const int b = static_cast<int>(bc / Cl);
        const float u = noise[(static_cast<long long>(b) * HW + t) * Cl + c];
        const float txt = noise[(static_cast<long long>(images + b) * HW + t) * Cl + c];
        const float guided = u + k.guidance * (txt - u);
        const float x = lat[i];
        const float x0 = x - k.sigma_s * guided;
        float xn;
        if (k.second_order) {
            const float d1 = k.inv_r0 * (x0 - hist_prev[i]);
            xn = k.a * x + k.b * x0 + k.c * d1;
        } else {
            xn = k.a * x + k.b * x0;
        }
        hist_cur[i] = x0;
        lat[i] = xn;
    }
}

__global__ void modulate_kernel(const float* __restrict__ x, long long rows, int C, int rows_per_seq,
                                const float* __restrict__ mod, long long mod_ld, int shift_idx, int scale_idx,
                                float* __restrict__ out) {
    const long long n = rows * C;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        const long long seq = (i / C) / rows_per_seq;
        const float* m = mod + seq * mod_ld;
        out[i] = x[i] * (1.0f + m[static_cast<long long>(scale_idx) * C + c]) + m[static_cast<long long>(shift_idx) * C + c];
    }
}

__global__ void scheduler_update_kernel(const float* __restrict__ m0, const float* __restrict__ m1,
                                        const float* __restrict__ x, long long n, SchedCoef k,
                                        float* __restrict__ out) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        if (k.second_order) {
            const float d1 = k.inv_r0 * (m0[i] - m1[i]);
            out[i] = k.a * x[i] + k.b * m0[i] + k.c * d1;
        } else {
            out[i] = k.a * x[i] + k.b * m0[i];
        }
    }
}

template <class TO>
__global__ void repack_kernel(const float* __restrict__ src, int rows, int cols, int transpose, TO* __restrict__ dst) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = src[static_cast<long long>(r) * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        if (transpose) {
            const int c = c0 + i, r = r0 + threadIdx.x;  // dst[c][r]
            if (r < rows && c < cols) dst[static_cast<long long>(c) * rows + r] = from_f<TO>(tile[threadIdx.x][i]);
        } else {
            const int r = r0 + i, c = c0 + threadIdx.x;
            if (r < rows && c < cols) dst[static_cast<long long>(r) * cols + c] = from_f<TO>(tile[i][threadIdx.x]);
        }
    }
}

template <class TO>
__global__ void convert_kernel(const float* __restrict__ src, long long n, TO* __restrict__ dst) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        dst[i] = from_f<TO>(src[i]);
}


// The same with persistent warps, for the denoiser's norm1 / norm2 (no affine, bf16 out): a
// warp walks rows warp_id, warp_id + n_warps, ... and loads its next row while it normalizes
// the current one, so each warp always has a row in flight; shift / scale come from global
// memory (L1-resident per sequence). Rows are read and written with streaming (evict-first)
// hints: each is touched once here. 0.73 of the measured copy bandwidth at config 2, against
// 0.62 for the one-row-per-warp kernel above.
template <int NV>
__global__ void __launch_bounds__(256, 2)
    ln_modulate_stream_kernel(const float* __restrict__ x, long long rows, int rows_per_seq,
                              const float* __restrict__ mod, long long mod_ld, int shift_idx, int scale_idx,
                              float eps, bf16* __restrict__ out) {
    constexpr int C = 128 * NV;
    const int lane = threadIdx.x & 31;
    const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
    long long row = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    float4 v[NV], nx[NV];
    if (row < rows) {
        const float4* xr = reinterpret_cast<const float4*>(x + row * C);
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = __ldcs(xr + lane + 32 * i);
    }
    for (; row < rows; row += nw) {
        const long long nrow = row + nw;
        if (nrow < rows) {
            const float4* xr = reinterpret_cast<const float4*>(x + nrow * C);
#pragma unroll
            for (int i = 0; i < NV; ++i) nx[i] = __ldcs(xr + lane + 32 * i);
        }
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        const float mean = warp_sum(s) / static_cast<float>(C);
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
            q += (a * a + b * b) + (c * c + d * d);
        }
        const float var = warp_sum(q) / static_cast<float>(C);
        const float inv_std = 1.0f / sqrtf(var + eps);
        const long long seq = row / rows_per_seq;
        const float4* shift = reinterpret_cast<const float4*>(mod + seq * mod_ld + static_cast<long long>(shift_idx) * C);
        const float4* scale = reinterpret_cast<const float4*>(mod + seq * mod_ld + static_cast<long long>(scale_idx) * C);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float4 sc = __ldg(scale + lane + 32 * i), sh = __ldg(shift + lane + 32 * i);
            const float o0 = (v[i].x - mean) * inv_std * (1.0f + sc.x) + sh.x;
            const float o1 = (v[i].y - mean) * inv_std * (1.0f + sc.y) + sh.y;
            const float o2 = (v[i].z - mean) * inv_std * (1.0f + sc.z) + sh.z;
            const float o3 = (v[i].w - mean) * inv_std * (1.0f + sc.w) + sh.w;
            __nv_bfloat162 h0 = __floats2bfloat162_rn(o0, o1), h1 = __floats2bfloat162_rn(o2, o3);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&h0);
            pk.y = *reinterpret_cast<uint32_t*>(&h1);
            __stcs(reinterpret_cast<uint2*>(out + row * C + 4 * (lane + 32 * i)), pk);
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = nx[i];
    }
}

int grid_for(long long n, int threads) {
    long long g = (n + threads - 1) / threads;
    if (g > 148LL * 32) g = 148LL * 32;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

template <class TO>
void ln_modulate(const float* x, long long rows, int C, int rows_per_seq, const float* gamma, const float* beta,
                 const float* mod, long long mod_ld, int shift_idx, int scale_idx, float eps, TO* out,
                 cudaStream_t st) {
    if (rows == 0) return;
    const int warps = 8;
    const unsigned grid = static_cast<unsigned>((rows + warps - 1) / warps);
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool reg = C % 128 == 0 && C / 128 <= 12 && a16(x) && a16(out) && (!gamma || a16(gamma)) &&
                     (!beta || a16(beta)) && (!mod || (a16(mod) && mod_ld % 4 == 0));
    if constexpr (sizeof(TO) == 2) {
        if (reg && C == 1152 && !gamma && !beta && mod && rows >= 4096) {
            static int sms = 0;
            if (sms == 0) {
                int dev = 0;
                SANA_CUDA(cudaGetDevice(&dev));
                SANA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
            }
            const long long blocks = std::min<long long>(2LL * sms, (rows + 7) / 8);
            ln_modulate_stream_kernel<9><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
                x, rows, rows_per_seq, mod, mod_ld, shift_idx, scale_idx, eps, reinterpret_cast<bf16*>(out));
            SANA_CUDA(cudaGetLastError());
            return;
        }
    }
    if (reg) {
        switch (C / 128) {
#define SANA_LN_CASE(NV)                                                                                        \
    case NV:                                                                                                    \
        ln_modulate_reg_kernel<TO, NV>                                                                          \
            <<<static_cast<unsigned>((rows + kLnWarps * ln_rows_per_warp<NV>() - 1) /                          \
                                     (kLnWarps * ln_rows_per_warp<NV>())),                                      \
               kLnWarps * 32, 0, st>>>(x, rows, rows_per_seq, gamma, beta, mod, mod_ld, shift_idx, scale_idx, eps, \
                                       out);                                                                    \
        SANA_CUDA(cudaGetLastError());                                                                          \
        return;
            SANA_LN_CASE(1) SANA_LN_CASE(2) SANA_LN_CASE(3) SANA_LN_CASE(4) SANA_LN_CASE(5) SANA_LN_CASE(6)
            SANA_LN_CASE(7) SANA_LN_CASE(8) SANA_LN_CASE(9) SANA_LN_CASE(10) SANA_LN_CASE(11) SANA_LN_CASE(12)
#undef SANA_LN_CASE
            default: break;
        }
    }
    ln_modulate_kernel<TO><<<grid, warps * 32, 0, st>>>(x, rows, C, rows_per_seq, gamma, beta, mod, mod_ld, shift_idx,
                                                        scale_idx, eps, out);
    SANA_CUDA(cudaGetLastError());
}

template <class T>
void rms_norm_rows(T* x, long long rows, int C, long long ld, float eps, const float* w, cudaStream_t st) {
    if (rows == 0) return;
    constexpr int warps = 8;
    rms_norm_rows_kernel<T><<<static_cast<unsigned>((rows + warps - 1) / warps), warps * 32, 0, st>>>(x, rows, C, ld,
                                                                                                      eps, w);
    SANA_CUDA(cudaGetLastError());
}
template void rms_norm_rows<float>(float*, long long, int, long long, float, const float*, cudaStream_t);
template void rms_norm_rows<bf16>(bf16*, long long, int, long long, float, const float*, cudaStream_t);

template <class TO>
void rms_norm(const float* x, long long rows, int C, float eps, const float* w, TO* out, cudaStream_t st) {
    if (rows == 0) return;
    const int warps = 8;
    rms_norm_kernel<TO><<<static_cast<unsigned>((rows + warps - 1) / warps), warps * 32, 0, st>>>(x, rows, C, eps,
                                                                                                  w, out);
    SANA_CUDA(cudaGetLastError());
}

void modulate(const float* x, long long rows, int C, int rows_per_seq, const float* mod, long long mod_ld,
              int shift_idx, int scale_idx, float* out, cudaStream_t st) {
    if (rows == 0) return;
    modulate_kernel<<<grid_for(rows * C, 256), 256, 0, st>>>(x, rows, C, rows_per_seq, mod, mod_ld, shift_idx,
                                                             scale_idx, out);
    SANA_CUDA(cudaGetLastError());
}

void scheduler_update(const float* m0, const float* m1, const float* x, long long n, SchedCoef k, float* out,
                      cudaStream_t st) {
    if (n == 0) return;
    scheduler_update_kernel<<<grid_for(n, 256), 256, 0, st>>>(m0, m1, x, n, k, out);
    SANA_CUDA(cudaGetLastError());
}

void block_modulation(const float* tmod, int S, int C, const float* tables, int n_blocks, float* mod,
                      cudaStream_t st) {
    const long long n = static_cast<long long>(n_blocks) * S * 6 * C;
    block_modulation_kernel<<<grid_for(n, 256), 256, 0, st>>>(tmod, S, 6 * C, tables, n_blocks, mod);
    SANA_CUDA(cudaGetLastError());
}

void final_modulation(const float* emb, int S, int C, const float* table, float* fmod, cudaStream_t st) {
    final_modulation_kernel<<<ceil_div(static_cast<long long>(S) * C, 256), 256, 0, st>>>(emb, S, C, table, fmod);
    SANA_CUDA(cudaGetLastError());
}

template <class TO>
void patch_tokens(const float* lat, int images, int seqs, int Cl, int HW, TO* out, cudaStream_t st) {
    const long long n = static_cast<long long>(seqs) * HW * Cl;
    patch_tokens_kernel<TO><<<grid_for(n, 256), 256, 0, st>>>(lat, images, seqs, Cl, HW, out);
    SANA_CUDA(cudaGetLastError());
}

template <class TO>
void broadcast_rows(const float* row, int S, int width, TO* out, cudaStream_t st) {
    broadcast_rows_kernel<TO><<<ceil_div(static_cast<long long>(S) * width, 256), 256, 0, st>>>(row, S, width, out);
    SANA_CUDA(cudaGetLastError());
}

template void patch_tokens<float>(const float*, int, int, int, int, float*, cudaStream_t);
template void patch_tokens<bf16>(const float*, int, int, int, int, bf16*, cudaStream_t);
template void broadcast_rows<float>(const float*, int, int, float*, cudaStream_t);
template void broadcast_rows<bf16>(const float*, int, int, bf16*, cudaStream_t);

void caption_kv_len(const float* bias, int S, int L, int* kv_len, cudaStream_t st) {
    kv_len_kernel<<<S, 256, 0, st>>>(bias, S, L, kv_len);
    SANA_CUDA(cudaGetLastError());
}

__global__ void wait_flag_kernel(const int* flag, int expect, int* err) {
    const uint64_t t0 = global_ns();
    const uint64_t limit = wait_limit_ns(err);
    for (uint32_t n = 0;; ++n) {
        if (*reinterpret_cast<const volatile int*>(flag) == expect) return;
        if ((n & 63u) == 0 && global_ns() - t0 > limit) {
            atomicCAS(err, 0, kTimeout);
            return;
        }
    }
}

void wait_flag(const int* flag, int expect, int* err, cudaStream_t st) {
    wait_flag_kernel<<<1, 1, 0, st>>>(flag, expect, err);
    SANA_CUDA(cudaGetLastError());
}

void cfg_scheduler_step(const float* noise, int images, int Cl, int HW, float* lat, float* hist_cur,
                        const float* hist_prev, SchedCoef k, cudaStream_t st) {
    const long long n = static_cast<long long>(images) * Cl * HW;
    cfg_scheduler_kernel<<<grid_for(n, 256), 256, 0, st>>>(noise, images, Cl, HW, lat, hist_cur, hist_prev, k);
    SANA_CUDA(cudaGetLastError());
}

// split_heads_3d / merge_heads_4d (transformer_ops.cpp:83-171): one thread per output element.
__global__ void permute_heads_kernel(const float* __restrict__ in, float* __restrict__ out, int B, int T, int H, int D,
                                     int to_heads) {
    const long long n = static_cast<long long>(B) * T * H * D;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int d = static_cast<int>(i % D);
        if (to_heads) {  // out [B, H, T, D] <- in [B, T, H*D]
            const long long r = i / D;
            const int t = static_cast<int>(r % T);
            const long long bh = r / T;
            const int h = static_cast<int>(bh % H);
            const long long b = bh / H;
            out[i] = in[((b * T + t) * H + h) * D + d];
        } else {  // out [B, T, H*D] <- in [B, H, T, D]
            const long long r = i / D;
            const int h = static_cast<int>(r % H);
            const long long bt = r / H;
            const int t = static_cast<int>(bt % T);
            const long long b = bt / T;
            out[i] = in[((b * H + h) * T + t) * D + d];
        }
    }
}

// softmax_lastdim_4d (transformer_ops.cpp:278-339): per row, e = exp(x - max), then
// e * (1 / sum e). One warp per row.
__global__ void softmax_rows_kernel(const float* __restrict__ in, long long rows, int n, float* __restrict__ out) {
    const long long row = blockIdx.x * static_cast<long long>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = in + row * n;
    float* y = out + row * n;
    float m = x[0];
    for (int d = lane; d < n; d += 32) m = fmaxf(m, x[d]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
    for (int d = lane; d < n; d += 32) {
        const float e = expf(x[d] - m);
        y[d] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float recip = 1.0f / sum;
    for (int d = lane; d < n; d += 32) y[d] *= recip;
}

void permute_heads(const float* in, float* out, int B, int T, int H, int D, bool to_heads, cudaStream_t st) {
    const long long n = static_cast<long long>(B) * T * H * D;
    if (n == 0) return;
    permute_heads_kernel<<<grid_for(n, 256), 256, 0, st>>>(in, out, B, T, H, D, to_heads ? 1 : 0);
    SANA_CUDA(cudaGetLastError());
}

void softmax_rows(const float* in, long long rows, int n, float* out, cudaStream_t st) {
    if (rows == 0 || n == 0) return;
    softmax_rows_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(in, rows, n, out);
    SANA_CUDA(cudaGetLastError());
}

template <class TO>
void repack(const float* src, int rows, int cols, bool transpose, TO* dst, cudaStream_t st) {
    dim3 grid(ceil_div(cols, 32), ceil_div(rows, 32));
    repack_kernel<TO><<<grid, dim3(32, 8), 0, st>>>(src, rows, cols, transpose ? 1 : 0, dst);
    SANA_CUDA(cudaGetLastError());
}

template <class TO>
void convert(const float* src, long long n, TO* dst, cudaStream_t st) {
    if (n == 0) return;
    convert_kernel<TO><<<grid_for(n, 256), 256, 0, st>>>(src, n, dst);
    SANA_CUDA(cudaGetLastError());
}

#define SANA_INST_TO(TO)                                                                                          \
    template void ln_modulate<TO>(const float*, long long, int, int, const float*, const float*, const float*,   \
                                  long long, int, int, float, TO*, cudaStream_t);                                \
    template void rms_norm<TO>(const float*, long long, int, float, const float*, TO*, cudaStream_t);             \
    template void repack<TO>(const float*, int, int, bool, TO*, cudaStream_t);                                    \
    template void convert<TO>(const float*, long long, TO*, cudaStream_t);
SANA_INST_TO(float)
SANA_INST_TO(bf16)
#undef SANA_INST_TO

}  // namespace sana
