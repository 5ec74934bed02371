// Masked softmax cross-attention to the caption on the fifth-generation tensor cores
// (attention_4d, transformer_ops.cpp:348-392, with the additive bias of :357-388), bf16 q / k / v
// in the token-major layouts of the fused projections, heads of D = 32, 64 or 72 channels.
//
// A persistent CTA walks work units (sequence, head, up to four 128-query tiles). For a unit
// its four softmax warps stage the head's keys K [keys, D] and the transposed values V^T
// [D, keys] of the sequence's live keys in shared memory (zero past the valid length, so the
// skipped keys contribute exactly nothing, as their -10000 bias makes them in fp32), together
// with the bias row. Then, per query tile:
//   warp 0   TMA producer: the 128 x D query tile, as D / 8 boxes [8 channels, 128 rows] that
//            land in the canonical K-major core-matrix layout (no swizzle)
//   warp 1   TMEM allocator + MMA issuer: S = Q K^T (M = 128, N = keys of a 128-key chunk,
//            K = D padded to 16) into one of two TMEM score buffers; once the softmax has
//            written P, O = P V (N = D padded to 16, K = the chunk's keys) into TMEM
//   warps 2-5 one query row per thread: the row's scores come out of TMEM, are scaled and
//            biased as the reference rounds them (scale, then bias), P = exp(s - max) goes to
//            shared memory as bf16 in the A-operand layout, and the row of O is read back,
//            rescaled across key chunks (online softmax, captions longer than 128 keys),
//            divided by the row sum and stored.
// The score MMA of the next tile overlaps the softmax of the current one (two score buffers);
// query tiles stream through a two-stage TMA ring. Every wait is bounded.
#include <algorithm>

#include "kernels.h"
#include "tcgen05.cuh"
#include "tma.h"

namespace sana {
namespace {

using namespace tc;

constexpr int kXQ = 128;            // queries per tile (MMA M)
constexpr int kXKeyChunk = 128;     // keys per score tile (MMA N)
constexpr int kXMaxKeys = 304;      // caption keys a unit can hold (19 x 16)
constexpr int kXTilesPerUnit = 4;   // query tiles per work unit
constexpr int kXThreads = 32 * 6;   // producer, MMA, four softmax warps

template <int D>
struct XtcCfg {
    static constexpr int DC = D / 8;                        // 16-byte slices of a head row
    static constexpr int DP = (D + 15) / 16 * 16;           // head dim padded to the MMA K step
    static constexpr int KCH = DP / 8;                      // slices including the padding
    static constexpr int kQBytes = KCH * kXQ * 16;          // [KCH][128 rows][8 ch]
    static constexpr int kQLoadBytes = DC * kXQ * 16;       // what TMA writes of it
    static constexpr int kKBytes = KCH * kXMaxKeys * 16;    // [KCH][keys][8 ch]
    static constexpr int kVBytes = (kXMaxKeys / 8) * DP * 16;  // [keys / 8][DP rows][8 keys]
    static constexpr int kPBytes = (kXKeyChunk / 8) * kXQ * 16;  // [keys / 8][128 rows][8 keys]
    static constexpr int kQOff = 0;
    static constexpr int kKOff = kQOff + 2 * kQBytes;
    static constexpr int kVOff = kKOff + kKBytes;
    static constexpr int kPOff = kVOff + kVBytes;
    static constexpr int kBiasOff = kPOff + kPBytes;
    static constexpr int kBarOff = kBiasOff + kXMaxKeys * 4;
    static constexpr int kBars = 12;
    static constexpr int kSmem = kBarOff + kBars * 8 + 16 + 128;
    static constexpr int kTmemS = 0;                        // two score buffers of 128 columns
    static constexpr int kTmemO = 2 * kXKeyChunk;           // the output accumulator, DP columns
    static constexpr int kTmemCols = 512;
    static_assert(D % 8 == 0 && DP <= 256 && kSmem <= 227 * 1024, "cross-attention tile configuration");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

struct XUnit {
    int s, h, tile0, ntiles;
};

__device__ __forceinline__ XUnit x_unit(int u, int heads, int groups, int qtiles) {
    XUnit x;
    const int g = u % groups;
    u /= groups;
    x.h = u % heads;
    x.s = u / heads;
    x.tile0 = g * kXTilesPerUnit;
    x.ntiles = min(kXTilesPerUnit, qtiles - x.tile0);
    return x;
}

template <int D>
__global__ void __launch_bounds__(kXThreads, 1)
    xattn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const bf16* __restrict__ kv, long long ldkv, int k_off,
                    int v_off, const float* __restrict__ bias, const int* __restrict__ kv_len, int S, int Tq, int L,
                    int heads, float scale, bf16* __restrict__ out, long long ldo, int* err) {
    using X = XtcCfg<D>;
    extern __shared__ uint8_t xs_raw[];
    const uint32_t raw = smem_u32(xs_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    uint8_t* gb = xs_raw + (base - raw);
    const uint32_t q_s = base + X::kQOff, k_s = base + X::kKOff, v_s = base + X::kVOff, p_s = base + X::kPOff;
    float* bsh = reinterpret_cast<float*>(gb + X::kBiasOff);
    const uint32_t bars = base + X::kBarOff;
    auto q_full = [&](int i) { return bars + 8u * i; };           // 2
    auto q_empty = [&](int i) { return bars + 8u * (2 + i); };    // 2
    const uint32_t kv_full = bars + 8u * 4, kv_empty = bars + 8u * 5;
    auto s_full = [&](int i) { return bars + 8u * (6 + i); };     // 2
    auto s_empty = [&](int i) { return bars + 8u * (8 + i); };    // 2
    const uint32_t p_full = bars + 8u * 10, o_full = bars + 8u * 11;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gb + X::kBarOff + X::kBars * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qtiles = (Tq + kXQ - 1) / kXQ;
    const int groups = (qtiles + kXTilesPerUnit - 1) / kXTilesPerUnit;
    const int units = S * heads * groups;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(q_full(i), 1);
            mbar_init(q_empty(i), 1);
            mbar_init(s_full(i), 1);
            mbar_init(s_empty(i), 4);
        }
        mbar_init(kv_full, 128);
        mbar_init(kv_empty, 1);
        mbar_init(p_full, 4);
        mbar_init(o_full, 1);
        fence_barrier_init();
    }
    // the query stages' padding slices (head channels D .. DP - 1) stay zero: TMA writes only
    // the first DC slices of a stage
    if constexpr (X::KCH > X::DC) {
        for (int i = threadIdx.x; i < 2 * (X::KCH - X::DC) * kXQ; i += blockDim.x) {
            const int st = i / ((X::KCH - X::DC) * kXQ), rem = i % ((X::KCH - X::DC) * kXQ);
            *reinterpret_cast<uint4*>(gb + X::kQOff + st * X::kQBytes + X::DC * kXQ * 16 + rem * 16) =
                make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), X::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer: query tiles ----------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
            int n = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
                const XUnit x = x_unit(u, heads, groups, qtiles);
                for (int t = 0; t < x.ntiles; ++t, ++n) {
                    const int st = n & 1;
                    if (!mbar_wait(q_empty(st), ((n >> 1) & 1) ^ 1, err, kTimeout)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(q_full(st), X::kQLoadBytes);
                    // one box [8 channels, 128 rows] per 16-byte slice of the head: each lands
                    // as 128 rows x 16 bytes, the K-major core-matrix column the MMA reads
                    const int row0 = x.s * Tq + (x.tile0 + t) * kXQ;
#pragma unroll
                    for (int c = 0; c < X::DC; ++c)
                        tma_load_2d(&tmQ, q_s + st * X::kQBytes + c * (kXQ * 16), q_full(st), x.h * D + 8 * c, row0);
                }
            }
            if (!ok) {  // the copies in flight land before the block exits
                for (int k = n > 2 ? n - 2 : 0; k < n; ++k) mbar_wait_quiet(q_full(k & 1), (k >> 1) & 1);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int n0 = 0;      // query tiles consumed before this unit
            int it0 = 0;     // (tile, key chunk) iterations before this unit
            int uc = 0;      // units processed
            bool ok = true;
            constexpr uint32_t kLboQ = kXQ * 16, kLboK = kXMaxKeys * 16, kLboV = X::DP * 16, kLboP = kXQ * 16;
            for (int u = blockIdx.x; ok && u < units; u += gridDim.x, ++uc) {
                const XUnit x = x_unit(u, heads, groups, qtiles);
                const int nkv = kv_len ? min(max(kv_len[x.s], 1), L) : L;
                const int npad = (nkv + 15) / 16 * 16;
                const int nch = (npad + kXKeyChunk - 1) / kXKeyChunk;
                const int iters = x.ntiles * nch;
                if (!mbar_wait(kv_full, uc & 1, err, kTimeout)) break;
                tc_fence_after();
                // S = Q K^T of iteration i (tile i / nch, key chunk i % nch) into score buffer i & 1
                auto issue_s = [&](int i) -> bool {
                    const int t = i / nch, c = i % nch, g = it0 + i, n = n0 + t, st = n & 1, sb = g & 1;
                    const int nk = min(kXKeyChunk, npad - c * kXKeyChunk);
                    if (c == 0) {
                        if (!mbar_wait(q_full(st), (n >> 1) & 1, err, kTimeout)) return false;
                    }
                    if (!mbar_wait(s_empty(sb), ((g >> 1) & 1) ^ 1, err, kTimeout)) return false;
                    tc_fence_after();
                    const uint32_t idesc_s = idesc_bf16_f32(kXQ, nk);
#pragma unroll
                    for (int kk = 0; kk < X::DP / 16; ++kk) {  // K steps of 16 = two 8-channel slices
                        const uint64_t a = kmajor_nosw_desc(q_s + st * X::kQBytes + 2 * kk * kLboQ, kLboQ, 128);
                        const uint64_t b = kmajor_nosw_desc(k_s + 2 * kk * kLboK + c * kXKeyChunk * 16, kLboK, 128);
                        umma_bf16(tmem + X::kTmemS + sb * kXKeyChunk, a, b, idesc_s, kk != 0 ? 1u : 0u);
                    }
                    umma_commit(s_full(sb));
                    if (c == nch - 1) umma_commit(q_empty(st));  // the tile's last read of its stage
                    return true;
                };
                ok = iters > 0 && issue_s(0);
                for (int i = 0; ok && i < iters; ++i) {
                    // the next score tile overlaps this iteration's softmax
                    if (i + 1 < iters && !issue_s(i + 1)) {
                        ok = false;
                        break;
                    }
                    // O = P V once the softmax has written this iteration's P (it has read the
                    // previous iteration's O by then)
                    const int c = i % nch, g = it0 + i;
                    const int nk = min(kXKeyChunk, npad - c * kXKeyChunk);
                    if (!mbar_wait(p_full, g & 1, err, kTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t idesc_o = idesc_bf16_f32(kXQ, X::DP);
                    for (int kk = 0; kk < nk / 16; ++kk) {
                        const uint64_t a = kmajor_nosw_desc(p_s + 2 * kk * kLboP, kLboP, 128);
                        const uint64_t b = kmajor_nosw_desc(v_s + (c * kXKeyChunk / 8 + 2 * kk) * kLboV, kLboV, 128);
                        umma_bf16(tmem + X::kTmemO, a, b, idesc_o, kk != 0 ? 1u : 0u);
                    }
                    umma_commit(o_full);
                }
                if (!ok) break;
                umma_commit(kv_empty);  // the unit's K / V / bias may be replaced
                n0 += x.ntiles;
                it0 += iters;
            }
            // every MMA this thread issued has completed before TMEM is released
            umma_commit(kv_empty);
            mbar_wait_quiet(kv_empty, uc & 1);
        }
    } else {
        // ---------------- softmax / epilogue: one query row per thread ----------------
        const int q4 = warp & 3;               // TMEM lane quarter of this warp
        const int row = q4 * 32 + lane;        // query row within the tile
        const int tid = threadIdx.x - 64;      // 0..127
        const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
        int n = 0, it = 0, uc = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++uc) {
            const XUnit x = x_unit(u, heads, groups, qtiles);
            const int nkv = kv_len ? min(max(kv_len[x.s], 1), L) : L;
            const int npad = (nkv + 15) / 16 * 16;
            const int nch = (npad + kXKeyChunk - 1) / kXKeyChunk;
            // the previous unit's MMAs are done with K / V (bounded wait; the first unit passes)
            if (!__all_sync(0xffffffffu, mbar_wait(kv_empty, (uc & 1) ^ 1, err, kTimeout))) break;
            // stage K [slice][key][8], V^T [key / 8][channel][8 keys] and the bias row
            const bf16* kvs = kv + static_cast<long long>(x.s) * L * ldkv;
            for (int i = tid; i < npad * X::KCH; i += 128) {
                const int j = i / X::KCH, c = i % X::KCH;
                uint4 kw = make_uint4(0u, 0u, 0u, 0u), vw = make_uint4(0u, 0u, 0u, 0u);
                if (j < nkv && c < X::DC) {
                    kw = *reinterpret_cast<const uint4*>(kvs + j * ldkv + k_off + x.h * D + c * 8);
                    vw = *reinterpret_cast<const uint4*>(kvs + j * ldkv + v_off + x.h * D + c * 8);
                }
                *reinterpret_cast<uint4*>(gb + X::kKOff + c * (kXMaxKeys * 16) + j * 16) = kw;
                const uint16_t* ve = reinterpret_cast<const uint16_t*>(&vw);
                uint8_t* vt = gb + X::kVOff + (j >> 3) * (X::DP * 16) + (j & 7) * 2;
#pragma unroll
                for (int e = 0; e < 8; ++e) *reinterpret_cast<uint16_t*>(vt + (c * 8 + e) * 16) = ve[e];
            }
            for (int j = tid; j < npad; j += 128)
                bsh[j] = (j < nkv && bias) ? bias[static_cast<long long>(x.s) * L + j] : 0.f;
            fence_proxy_async_smem();
            __syncwarp();
            mbar_arrive(kv_full);
            // all four warps' staging (the bias row included) is complete
            if (!__all_sync(0xffffffffu, mbar_wait(kv_full, uc & 1, err, kTimeout))) break;

            bool ok = true;
            for (int t = 0; ok && t < x.ntiles; ++t, ++n) {
                float o_acc[D];
#pragma unroll
                for (int d = 0; d < D; ++d) o_acc[d] = 0.f;
                float m_run = -INFINITY, l_run = 0.f;
                for (int c = 0; c < nch; ++c, ++it) {
                    const int sb = it & 1;
                    const int nk = min(kXKeyChunk, npad - c * kXKeyChunk);  // multiple of 16
                    const int nvalid = min(kXKeyChunk, nkv - c * kXKeyChunk);
                    if (!__all_sync(0xffffffffu, mbar_wait(s_full(sb), (it >> 1) & 1, err, kTimeout))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t s_addr = tmem + t_lane + X::kTmemS + sb * kXKeyChunk;
                    const float* bc = bsh + c * kXKeyChunk;
                    // pass 1: the chunk's maximum score
                    float mx = -INFINITY;
                    for (int j0 = 0; j0 < nk; j0 += 16) {
                        uint32_t r[16];
                        tmem_ld16(s_addr + j0, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (j0 + e < nvalid)
                                mx = fmaxf(mx, __fadd_rn(__fmul_rn(__uint_as_float(r[e]), scale), bc[j0 + e]));
                    }
                    const float m_new = fmaxf(m_run, mx);
                    const float corr = __expf(m_run - m_new);  // 0 on the first chunk (m_run = -inf)
                    // pass 2: P = exp(s - max) as bf16 into the A-operand layout, row sum in fp32
                    float sum = 0.f;
                    for (int j0 = 0; j0 < nk; j0 += 16) {
                        uint32_t r[16];
                        tmem_ld16(s_addr + j0, r);
                        tmem_wait_ld();
                        float p[16];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            p[e] = (j0 + e < nvalid)
                                       ? __expf(__fadd_rn(__fmul_rn(__uint_as_float(r[e]), scale), bc[j0 + e]) - m_new)
                                       : 0.f;
                            sum += p[e];
                        }
#pragma unroll
                        for (int h8 = 0; h8 < 2; ++h8) {
                            const uint4 w = make_uint4(pack_bf16x2(p[8 * h8], p[8 * h8 + 1]),
                                                       pack_bf16x2(p[8 * h8 + 2], p[8 * h8 + 3]),
                                                       pack_bf16x2(p[8 * h8 + 4], p[8 * h8 + 5]),
                                                       pack_bf16x2(p[8 * h8 + 6], p[8 * h8 + 7]));
                            *reinterpret_cast<uint4*>(gb + X::kPOff + ((j0 >> 3) + h8) * (kXQ * 16) + row * 16) = w;
                        }
                    }
                    // the score buffer is free; P is visible to the tensor cores
                    tc_fence_before();
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(s_empty(sb));
                        mbar_arrive(p_full);
                    }
                    // O of this chunk, folded into the running output with the rescale
                    if (!__all_sync(0xffffffffu, mbar_wait(o_full, it & 1, err, kTimeout))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t o_addr = tmem + t_lane + X::kTmemO;
#pragma unroll
                    for (int d0 = 0; d0 < X::DP; d0 += 16) {
                        uint32_t r[16];
                        tmem_ld16(o_addr + d0, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (d0 + e < D) o_acc[d0 + e] = fmaf(o_acc[d0 + e], corr, __uint_as_float(r[e]));
                    }
                    tc_fence_before();
                    l_run = fmaf(l_run, corr, sum);
                    m_run = m_new;
                }
                if (!ok) break;
                // the finished row: O / sum -> bf16, 16-byte stores
                const int tq = (x.tile0 + t) * kXQ + row;
                if (tq < Tq) {
                    const float inv = 1.0f / l_run;
                    bf16* o = out + (static_cast<long long>(x.s) * Tq + tq) * ldo + x.h * D;
#pragma unroll
                    for (int c = 0; c < X::DC; ++c)
                        *reinterpret_cast<uint4*>(o + c * 8) =
                            make_uint4(pack_bf16x2(o_acc[8 * c] * inv, o_acc[8 * c + 1] * inv),
                                       pack_bf16x2(o_acc[8 * c + 2] * inv, o_acc[8 * c + 3] * inv),
                                       pack_bf16x2(o_acc[8 * c + 4] * inv, o_acc[8 * c + 5] * inv),
                                       pack_bf16x2(o_acc[8 * c + 6] * inv, o_acc[8 * c + 7] * inv));
                }
            }
            if (!ok) break;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, X::kTmemCols);
    }
}

// The query rows [rows, cols] (row stride ldq elements) for TMA, box = 8 channels x 128 rows
// without swizzle: a box lands as 128 rows x 16 bytes, one K-major core-matrix column of the
// MMA's A operand. Its x coordinate (a head's channel offset + 8 c) is always 16-byte aligned.
CUtensorMap query_map(const bf16* q, long long ldq, long long rows, int cols) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldq) * 2};
    const cuuint32_t box[2] = {8, static_cast<cuuint32_t>(kXQ)};
    tma_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    return m;
}

template <int D>
void launch_tc(const bf16* q, long long ldq, const bf16* kv, long long ldkv, int k_off, int v_off, const float* bias,
               const int* kv_len, int S, int Tq, int L, int heads, float scale, bf16* out, long long ldo, int* err,
               cudaStream_t st) {
    using X = XtcCfg<D>;
    static PerDeviceOnce attr;
    static int sms[64] = {};
    int dev = 0;
    SANA_CUDA(cudaGetDevice(&dev));
    if (attr.pending()) {
        SANA_CUDA(cudaFuncSetAttribute(xattn_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, X::kSmem));
        attr.mark();
    }
    int& n_sm = sms[dev & 63];
    if (n_sm == 0) SANA_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    const CUtensorMap mq = query_map(q, ldq, static_cast<long long>(S) * Tq, heads * D);
    const int qtiles = (Tq + kXQ - 1) / kXQ;
    const long long units = static_cast<long long>(S) * heads * ((qtiles + kXTilesPerUnit - 1) / kXTilesPerUnit);
    SANA_REQUIRE(units < (1LL << 31), "cross attention: too many work units");
    const int grid = static_cast<int>(std::min<long long>(units, n_sm));
    xattn_tc_kernel<D><<<grid, kXThreads, X::kSmem, st>>>(mq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads,
                                                          scale, out, ldo, err);
    SANA_CUDA(cudaGetLastError());
}

}  // namespace

bool cross_attention_tc(const bf16* q, long long ldq, const bf16* kv, long long ldkv, int k_off, int v_off,
                        const float* bias, const int* kv_len, int S, int Tq, int L, int heads, int D, float scale,
                        bf16* out, long long ldo, int* err, cudaStream_t st) {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    // 16-byte rows and head offsets (TMA box and vector loads), the query tensor's width a whole
    // number of heads, and a caption that fits the unit's key buffer
    const bool ok = (D == 32 || D == 64 || D == 72) && L <= kXMaxKeys && L >= 1 && ldq % 8 == 0 &&
                    ldkv % 8 == 0 && ldo % 8 == 0 && k_off % 8 == 0 && v_off % 8 == 0 && a16(q) && a16(kv) &&
                    a16(out) && err != nullptr;
    if (!ok) return false;
    if (S == 0 || Tq == 0) return true;
    switch (D) {
        case 32: launch_tc<32>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, err, st); break;
        case 64: launch_tc<64>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, err, st); break;
        default: launch_tc<72>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, err, st); break;
    }
    return true;
}

}  // namespace sana
