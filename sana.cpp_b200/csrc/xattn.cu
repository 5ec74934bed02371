// Masked softmax cross-attention to the caption (attention_4d, transformer_ops.cpp:348-392,
// with the additive bias of :357-388). One thread per query token and head; the head's
// keys and values for the sequence's live key range sit in shared memory. Two passes per
// query: the maximum of the scaled, biased scores, then exp(s - max) weighted sums,
// divided once by their total (the softmax of :318-334 followed by probs @ v).
//
// bf16 mode runs the tensor-core variant below (xattn_mma_kernel) for head dims 32/64/72/128.
//
// Keys at index >= kv_len[s] are skipped: their bias is <= -1000 (caption_kv_len), so
// exp(score - max) underflows to exactly 0 in fp32 and the reference's sum is unchanged.
#include "kernels.h"

namespace sana {
namespace {

constexpr int kQ = 128;  // queries per block

template <class T, int DMAX>
__global__ void __launch_bounds__(kQ) xattn_kernel(const T* __restrict__ q, long long ldq, const T* __restrict__ kv,
                                                   long long ldkv, int k_off, int v_off,
                                                   const float* __restrict__ bias, const int* __restrict__ kv_len,
                                                   int Tq, int L, int D, float scale, T* __restrict__ out,
                                                   long long ldo) {
    extern __shared__ unsigned char smraw[];
    const int s = blockIdx.z, h = blockIdx.y;
    const int n_kv = kv_len ? kv_len[s] : L;
    T* Ks = reinterpret_cast<T*>(smraw);   // [n_kv][D]
    T* Vs = Ks + n_kv * D;                  // [n_kv][D]
    float* bs = reinterpret_cast<float*>(Vs + n_kv * D);  // 2 * n_kv * D * sizeof(T) bytes in: 4-aligned
    for (int i = threadIdx.x; i < n_kv * D; i += blockDim.x) {
        const int j = i / D, d = i % D;
        const long long row = static_cast<long long>(s) * L + j;
        Ks[i] = kv[row * ldkv + k_off + h * D + d];
        Vs[i] = kv[row * ldkv + v_off + h * D + d];
    }
    for (int j = threadIdx.x; j < n_kv; j += blockDim.x) bs[j] = bias ? bias[static_cast<long long>(s) * L + j] : 0.f;
    __syncthreads();

    const int t = blockIdx.x * kQ + threadIdx.x;
    if (t >= Tq) return;
    const T* qr = q + (static_cast<long long>(s) * Tq + t) * ldq + h * D;
    float qv[DMAX];
#pragma unroll
    for (int d = 0; d < DMAX; ++d) qv[d] = d < D ? to_f(qr[d]) : 0.f;

    float mx = -INFINITY;
    for (int j = 0; j < n_kv; ++j) {
        const T* kr = Ks + j * D;
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < DMAX; ++d)
            if (d < D) dot = fmaf(qv[d], to_f(kr[d]), dot);
        // scores * scale, then + bias, each rounded (transformer_ops.cpp:355, :381-383); with
        // a -10000 mask a fused multiply-add would round the sum differently
        const float sc = __fadd_rn(__fmul_rn(dot, scale), bs[j]);
        mx = fmaxf(mx, sc);
    }
    float acc[DMAX];
#pragma unroll
    for (int d = 0; d < DMAX; ++d) acc[d] = 0.f;
    float den = 0.f;
    for (int j = 0; j < n_kv; ++j) {
        const T* kr = Ks + j * D;
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < DMAX; ++d)
            if (d < D) dot = fmaf(qv[d], to_f(kr[d]), dot);
        const float p = expf(__fadd_rn(__fmul_rn(dot, scale), bs[j]) - mx);
        den += p;
        const T* vr = Vs + j * D;
#pragma unroll
        for (int d = 0; d < DMAX; ++d)
            if (d < D) acc[d] = fmaf(p, to_f(vr[d]), acc[d]);
    }
    const float inv = 1.0f / den;
    T* o = out + (static_cast<long long>(s) * Tq + t) * ldo + h * D;
#pragma unroll
    for (int d = 0; d < DMAX; ++d)
        if (d < D) o[d] = from_f<T>(acc[d] * inv);
}

template <class T, int DMAX>
void launch(const T* q, long long ldq, const T* kv, long long ldkv, int k_off, int v_off, const float* bias,
            const int* kv_len, int S, int Tq, int L, int heads, int D, float scale, T* out, long long ldo,
            cudaStream_t st) {
    const size_t smem = 2 * static_cast<size_t>(L) * D * sizeof(T) + static_cast<size_t>(L) * 4 + 8;
    static PerDeviceOnce attr;
    if (attr.pending()) {
        SANA_CUDA(cudaFuncSetAttribute(xattn_kernel<T, DMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       227 * 1024));
        attr.mark();
    }
    xattn_kernel<T, DMAX><<<dim3(ceil_div(Tq, kQ), heads, S), kQ, smem, st>>>(q, ldq, kv, ldkv, k_off, v_off, bias,
                                                                             kv_len, Tq, L, D, scale, out, ldo);
    SANA_CUDA(cudaGetLastError());
}


// ---------------------------------------------------------------------------------------
// bf16 path on tensor cores (mma.sync m16n8k16, fp32 accumulation), flash-style: a block
// takes 128 queries of one head; each warp owns 16 query rows. The query tile arrives with
// 16-byte async copies and is read into fragments with ldmatrix; keys and values stream
// through shared memory in chunks of 64 with an online softmax (running max / sum per row,
// rescaled accumulators), and only the 8-key column tiles holding live keys are multiplied.
// Scores are rounded as the reference rounds them (scale, then bias); P is rounded to bf16
// for the P.V product, so the exponentials use the hardware's fast path. The normalised
// output goes back through the warp's rows of the query tile and leaves as 16-byte stores.
// Shared tiles are padded to conflict-free row strides.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16_1688(float (&c)[4], const uint32_t (&a)[2], uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(b0));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

constexpr int kMmaWarps = 8;   // 16 query rows per warp, 128 per query tile
constexpr int kChunkKeys = 64;

// SMs of the current device (cached per device).
int xattn_sms() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
    }
    return cached[dev];
}
static_assert(kChunkKeys == 64, "a chunk is two groups of four 8-key column tiles");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x1(uint32_t addr, uint32_t& r0) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x1.shared.b16 {%0}, [%1];" : "=r"(r0) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Row strides (elements) whose 4-byte-word stride is 4 mod 8: every 8-row fragment load
// then touches 32 distinct banks.
__host__ __device__ constexpr int conflict_free_stride(int min_elems) {
    return ((min_elems / 2) % 8 == 4) ? min_elems : ((min_elems + 7) / 8 * 8 + ((((min_elems + 7) / 8 * 8) / 2) % 8 == 4 ? 0 : 8));
}

template <int D, int kXTiles>
struct XattnTiles {
    static constexpr int KS = D / 16;                      // k-steps of 16 over the head dim
    static constexpr bool KT = D % 16 != 0;                // and one of 8 (D = 72)
    static constexpr int KSTR = conflict_free_stride(D);   // Q and K tile row stride
    static constexpr int VSTR = conflict_free_stride(D);   // V tile row stride
    static constexpr int kQRows = 16 * kMmaWarps;
    // the query tile, then two buffers of one key / value / bias chunk each
    static constexpr size_t kChunkBytes = static_cast<size_t>(kChunkKeys) * (KSTR + VSTR) * 2 + kChunkKeys * 4;
    static constexpr size_t kBytes = static_cast<size_t>(kXTiles) * kQRows * KSTR * 2 + 2 * kChunkBytes;
};

// kXTiles query tiles of 128 per block (one or two, chosen by the launch).
template <int D, int kXTiles>
__global__ void __launch_bounds__(32 * kMmaWarps) xattn_mma_kernel(const bf16* __restrict__ q, long long ldq,
                                                                   const bf16* __restrict__ kv, long long ldkv,
                                                                   int k_off, int v_off,
                                                                   const float* __restrict__ bias,
                                                                   const int* __restrict__ kv_len, int Tq, int L,
                                                                   float scale, bf16* __restrict__ out,
                                                                   long long ldo) {
    using X = XattnTiles<D, kXTiles>;
    constexpr int KS = X::KS, KSTR = X::KSTR, VSTR = X::VSTR;
    constexpr bool KT = X::KT;
    static_assert(D % 8 == 0, "head dim in 8-column fragments");
    constexpr int NT = D / 8;  // 8-wide output tiles
    constexpr int RC = D / 8;  // 16-byte pieces of a row
    static_assert((KSTR / 2) % 8 == 4 && (VSTR / 2) % 8 == 4 && KSTR % 8 == 0 && VSTR % 8 == 0, "strides");
    extern __shared__ __align__(16) unsigned char xsm[];
    bf16* Qs = reinterpret_cast<bf16*>(xsm);  // kXTiles x [128][KSTR], later the output rows
    unsigned char* chunk0 = xsm + kXTiles * X::kQRows * KSTR * 2;  // two buffers of [K 64][KSTR], [V 64][VSTR], bias [64]
    auto Kbuf = [&](int b) { return reinterpret_cast<bf16*>(chunk0 + b * X::kChunkBytes); };
    auto Vbuf = [&](int b) { return Kbuf(b) + kChunkKeys * KSTR; };
    auto Bbuf = [&](int b) { return reinterpret_cast<float*>(Vbuf(b) + kChunkKeys * VSTR); };

    const int s = blockIdx.z, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tig = lane & 3;
    const int n_kv = kv_len ? kv_len[s] : L;
    const int nchunks = (n_kv + kChunkKeys - 1) / kChunkKeys;
    // Both query tiles of the block share the key / value chunks: with at most two chunks (the
    // captions' live keys fit in 128) they stay resident and load once; longer captions stream
    // them again for the second tile.
    const bool resident = nchunks <= 2;
    const int ntiles = min(kXTiles, (Tq - static_cast<int>(blockIdx.x) * kXTiles * X::kQRows + X::kQRows - 1) / X::kQRows);

    auto Qtile = [&](int t) { return Qs + t * X::kQRows * KSTR; };
    // query tile t (rows past Tq read as zeros); the caller commits the copies
    auto load_q = [&](int t) {
        const int qb = (blockIdx.x * kXTiles + t) * X::kQRows;
        bf16* Qt = Qtile(t);
        const uint32_t qt_s = smem_u32(Qt);
        for (int i = threadIdx.x; i < X::kQRows * RC; i += blockDim.x) {
            const int r = i / RC, ck = i % RC;
            if (qb + r < Tq)
                cp_async16(qt_s + static_cast<uint32_t>(r * KSTR + ck * 8) * 2u,
                           q + (static_cast<long long>(s) * Tq + qb + r) * ldq + h * D + ck * 8);
            else
                *reinterpret_cast<uint4*>(Qt + r * KSTR + ck * 8) = make_uint4(0u, 0u, 0u, 0u);
        }
    };
    // keys and values of chunk c into buffer b; keys past the chunk end are zeros (their scores
    // are masked to -inf)
    auto load_chunk = [&](int c, int b) {
        const int c0 = c * kChunkKeys, nk = min(kChunkKeys, n_kv - c0);
        bf16* Kb = Kbuf(b);
        bf16* Vb = Vbuf(b);
        const uint32_t kb = smem_u32(Kb), vb = smem_u32(Vb);
        for (int i = threadIdx.x; i < kChunkKeys * RC * 2; i += blockDim.x) {
            const int which = i / (kChunkKeys * RC), rem = i % (kChunkKeys * RC);
            const int j = rem / RC, ck = rem % RC;
            if (j < nk) {
                const bf16* src = kv + (static_cast<long long>(s) * L + c0 + j) * ldkv + (which ? v_off : k_off) + h * D +
                                  ck * 8;
                cp_async16(which ? vb + static_cast<uint32_t>(j * VSTR + ck * 8) * 2u
                                 : kb + static_cast<uint32_t>(j * KSTR + ck * 8) * 2u,
                           src);
            } else {
                bf16* dst = which ? Vb + j * VSTR + ck * 8 : Kb + j * KSTR + ck * 8;
                *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        float* bb = Bbuf(b);
        for (int j = threadIdx.x; j < kChunkKeys; j += blockDim.x)
            bb[j] = (j < nk && bias) ? bias[static_cast<long long>(s) * L + c0 + j] : 0.f;
    };
    auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };

    // the first query tile with the first chunk (and, when resident, the second chunk); the
    // second query tile after them, landing while the first computes
    load_q(0);
    load_chunk(0, 0);
    if (resident && nchunks == 2) load_chunk(1, 1);
    commit();
    if (resident && ntiles > 1) {
        load_q(1);
        commit();
    }

    for (int t = 0; t < ntiles; ++t) {
        const int q0 = (blockIdx.x * kXTiles + t) * X::kQRows + warp * 16;
        const bool active = q0 < Tq;
        const uint32_t qbase = smem_u32(Qtile(t));
        uint32_t qa[KS][4], qt[2];
        float o[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

        if (!resident && t > 0) {  // chunk buffers are free: the last chunk loop ended with a barrier
            load_q(t);
            load_chunk(0, 0);
            commit();
        }
        for (int c = 0; c < nchunks; ++c) {
            const int buf = c & 1;
            if (resident) {
                if (c == 0) {
                    if (t == 0 && ntiles > 1) asm volatile("cp.async.wait_group 1;" ::: "memory");
                    else asm volatile("cp.async.wait_group 0;" ::: "memory");
                    __syncthreads();
                }
            } else {
                if (c + 1 < nchunks) {
                    load_chunk(c + 1, buf ^ 1);
                    commit();
                    asm volatile("cp.async.wait_group 1;" ::: "memory");
                } else {
                    asm volatile("cp.async.wait_group 0;" ::: "memory");
                }
                __syncthreads();
            }
            const int c0 = c * kChunkKeys;
            const int nk = min(kChunkKeys, n_kv - c0);
            const uint32_t kbase = smem_u32(Kbuf(buf)), vbase = smem_u32(Vbuf(buf));
            const float* bsh = Bbuf(buf);
            if (active) {
                if (c == 0) {
#pragma unroll
                    for (int kk = 0; kk < KS; ++kk)
                        ldmatrix_x4(qbase + static_cast<uint32_t>((warp * 16 + (lane & 15)) * KSTR + kk * 16 + (lane >> 4) * 8) *
                                                2u,
                                    qa[kk]);
                    if constexpr (KT)
                        ldmatrix_x2(qbase + static_cast<uint32_t>((warp * 16 + (lane & 15)) * KSTR + KS * 16) * 2u, qt[0], qt[1]);
                }
                const int ntmax = (nk + 7) / 8;  // 8-key column tiles holding live keys
                float sc[kChunkKeys / 8][4];
#pragma unroll
                for (int nt = 0; nt < kChunkKeys / 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = -INFINITY;
                // Four 8-key column tiles at a time, k-steps outermost: four independent accumulator
                // chains per k-step instead of one. The second group runs only when it holds live
                // keys; tiles past the live ones read zero rows and stay masked.
#pragma unroll
                for (int grp = 0; grp < 2; ++grp) {
                    if (grp == 1 && ntmax <= 4) break;
                    float acc[4][4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
                    // K fragments by ldmatrix: 8 key rows x (two k-steps of 16) per x4 load
                    const uint32_t krow = kbase + static_cast<uint32_t>((grp * 32 + (lane & 7)) * KSTR + (lane >> 3) * 8) * 2u;
#pragma unroll
                    for (int kk = 0; kk + 1 < KS; kk += 2) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t b[4];
                            ldmatrix_x4(krow + static_cast<uint32_t>(j * 8 * KSTR + kk * 16) * 2u, b);
                            mma_bf16_16816(acc[j], qa[kk], b[0], b[1]);
                            mma_bf16_16816(acc[j], qa[kk + 1], b[2], b[3]);
                        }
                    }
                    if constexpr (KS % 2 == 1) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t b0, b1;
                            ldmatrix_x2(krow + static_cast<uint32_t>(j * 8 * KSTR + (KS - 1) * 16) * 2u, b0, b1);
                            mma_bf16_16816(acc[j], qa[KS - 1], b0, b1);
                        }
                    }
                    if constexpr (KT) {  // the last 8 head-dim columns: one m16n8k8 per tile
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t b0;
                            ldmatrix_x1(krow + static_cast<uint32_t>(j * 8 * KSTR + KS * 16) * 2u, b0);
                            mma_bf16_1688(acc[j], qt, b0);
                        }
                    }
                    // scores: scale, then bias, each rounded, two keys per packed operation
                    const uint64_t scale2 = f2_make(scale, scale);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int nt = grp * 4 + j;
                        const int key = nt * 8 + tig * 2;
                        const uint64_t b2 = *reinterpret_cast<const uint64_t*>(bsh + key);
                        const float2 r0 = f2_split(add2(mul2(f2_make(acc[j][0], acc[j][1]), scale2), b2));
                        const float2 r1 = f2_split(add2(mul2(f2_make(acc[j][2], acc[j][3]), scale2), b2));
                        if (key < nk) {
                            sc[nt][0] = r0.x;
                            sc[nt][2] = r1.x;
                        }
                        if (key + 1 < nk) {
                            sc[nt][1] = r0.y;
                            sc[nt][3] = r1.y;
                        }
                    }
                }
                float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                for (int nt = 0; nt < kChunkKeys / 8; ++nt) {
                    mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
                    mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
                }
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float mp0 = m0, mp1 = m1;
                m0 = mn0;
                m1 = mn1;
                float sum0 = 0.f, sum1 = 0.f;
                constexpr float kLog2e = 1.4426950408889634f;  // log2(e)
                const uint64_t l2e = f2_make(kLog2e, kLog2e);
                const uint64_t nb0 = f2_make(-mn0 * kLog2e, -mn0 * kLog2e), nb1 = f2_make(-mn1 * kLog2e, -mn1 * kLog2e);
#pragma unroll
                for (int nt = 0; nt < kChunkKeys / 8; ++nt) {
                    if (nt < ntmax) {
                        // exp(s - max) = 2^(s log2 e - max log2 e): one packed FMA per two keys and the
                        // hardware base-2 exponential (a few ulp; P is rounded to bf16 below)
                        const float2 e0 = f2_split(fma2(f2_make(sc[nt][0], sc[nt][1]), l2e, nb0));
                        const float2 e1 = f2_split(fma2(f2_make(sc[nt][2], sc[nt][3]), l2e, nb1));
                        sc[nt][0] = ex2_approx(e0.x);
                        sc[nt][1] = ex2_approx(e0.y);
                        sc[nt][2] = ex2_approx(e1.x);
                        sc[nt][3] = ex2_approx(e1.y);
                        sum0 += sc[nt][0] + sc[nt][1];
                        sum1 += sc[nt][2] + sc[nt][3];
                    } else {
                        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
                    }
                }
                if (c == 0) {  // nothing accumulated yet (the rescale would multiply zeros by exp(-inf) = 0)
                    l0 = sum0;
                    l1 = sum1;
                } else {
                    const float corr0 = __expf(mp0 - mn0), corr1 = __expf(mp1 - mn1);
                    l0 = l0 * corr0 + sum0;
                    l1 = l1 * corr1 + sum1;
                    const uint64_t c0 = f2_make(corr0, corr0), c1 = f2_make(corr1, corr1);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const float2 a = f2_split(mul2(f2_make(o[nt][0], o[nt][1]), c0));
                        const float2 b = f2_split(mul2(f2_make(o[nt][2], o[nt][3]), c1));
                        o[nt][0] = a.x;
                        o[nt][1] = a.y;
                        o[nt][2] = b.x;
                        o[nt][3] = b.y;
                    }
                }
                const int kmax = (nk + 15) / 16;  // k-steps holding live keys
#pragma unroll
                for (int kk = 0; kk < kChunkKeys / 16; ++kk) {
                    if (kk >= kmax) break;
                    const uint32_t pa[4] = {pack_bf16(sc[2 * kk][0], sc[2 * kk][1]), pack_bf16(sc[2 * kk][2], sc[2 * kk][3]),
                                            pack_bf16(sc[2 * kk + 1][0], sc[2 * kk + 1][1]),
                                            pack_bf16(sc[2 * kk + 1][2], sc[2 * kk + 1][3])};
                    const uint32_t vrow = vbase + static_cast<uint32_t>((kk * 16 + (lane & 15)) * VSTR) * 2u;
                    // V fragments of two 8-column output tiles per x4 load (lanes 16-31 address the second)
                    const uint32_t vrow4 = vrow + static_cast<uint32_t>((lane >> 4) * 8) * 2u;
#pragma unroll
                    for (int nt = 0; nt + 1 < NT; nt += 2) {
                        uint32_t b[4];
                        ldmatrix_x4_trans(vrow4 + static_cast<uint32_t>(nt * 16), b);
                        mma_bf16_16816(o[nt], pa, b[0], b[1]);
                        mma_bf16_16816(o[nt + 1], pa, b[2], b[3]);
                    }
                    if constexpr (NT % 2 == 1) {
                        uint32_t b0, b1;
                        ldmatrix_x2_trans(vrow + static_cast<uint32_t>((NT - 1) * 16), b0, b1);
                        mma_bf16_16816(o[NT - 1], pa, b0, b1);
                    }
                }
            }
            if (!resident) __syncthreads();  // buffer `buf` is free for chunk c + 2
        }
        if (active) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
            l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
            l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
            l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
            const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
            // the warp's 16 output rows through its own rows of the query tile, then 16-byte stores
            bf16* orows = Qtile(t) + warp * 16 * KSTR;
            const uint64_t i0 = f2_make(inv0, inv0), i1 = f2_make(inv1, inv1);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float2 a = f2_split(mul2(f2_make(o[nt][0], o[nt][1]), i0));
                const float2 b = f2_split(mul2(f2_make(o[nt][2], o[nt][3]), i1));
                *reinterpret_cast<uint32_t*>(orows + g * KSTR + nt * 8 + tig * 2) = pack_bf16(a.x, a.y);
                *reinterpret_cast<uint32_t*>(orows + (g + 8) * KSTR + nt * 8 + tig * 2) = pack_bf16(b.x, b.y);
            }
            __syncwarp();
            for (int i = lane; i < 16 * RC; i += 32) {
                const int r = i / RC, ck = i % RC;
                if (q0 + r < Tq)
                    *reinterpret_cast<uint4*>(out + (static_cast<long long>(s) * Tq + q0 + r) * ldo + h * D + ck * 8) =
                        *reinterpret_cast<const uint4*>(orows + r * KSTR + ck * 8);
            }
        }
    }
}

template <int D, int kXTiles>
void launch_mma_tiles(const bf16* q, long long ldq, const bf16* kv, long long ldkv, int k_off, int v_off,
                      const float* bias, const int* kv_len, int S, int Tq, int L, int heads, float scale, bf16* out,
                      long long ldo, cudaStream_t st) {
    constexpr size_t smem = XattnTiles<D, kXTiles>::kBytes;
    static PerDeviceOnce attr;
    if (attr.pending()) {
        SANA_CUDA(cudaFuncSetAttribute(xattn_mma_kernel<D, kXTiles>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
        attr.mark();
    }
    xattn_mma_kernel<D, kXTiles><<<dim3(ceil_div(Tq, kXTiles * 16 * kMmaWarps), heads, S), 32 * kMmaWarps, smem, st>>>(
        q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, Tq, L, scale, out, ldo);
    SANA_CUDA(cudaGetLastError());
}

// Two query tiles per block share one load of the keys and values: measured 6 % faster at
// config 2 (32 sequences of 1024 queries) and 1-5 % faster in the loop at 4-16 sequences, but
// 12 % slower on 4096-query sequences with 300 live keys (the keys stream again for each tile).
// So: two tiles for grids of at least four waves (two blocks per SM), and for sequences of up to
// 2048 queries whenever the two-tile grid still gives every SM a block; one tile otherwise.
template <int D>
bool launch_mma(const bf16* q, long long ldq, const bf16* kv, long long ldkv, int k_off, int v_off, const float* bias,
                const int* kv_len, int S, int Tq, int L, int heads, float scale, bf16* out, long long ldo,
                cudaStream_t st) {
    const long long blocks2 = static_cast<long long>(ceil_div(Tq, 2 * 16 * kMmaWarps)) * heads * S;
    if (blocks2 >= 4LL * 2 * xattn_sms() || (Tq <= 2048 && blocks2 >= xattn_sms()))
        launch_mma_tiles<D, 2>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, st);
    else
        launch_mma_tiles<D, 1>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, st);
    return true;
}

// Tensor-core path when the operands allow 32-bit fragment loads.
template <class T>
bool try_mma(const T*, long long, const T*, long long, int, int, const float*, const int*, int, int, int, int, int,
             float, T*, long long, cudaStream_t) {
    return false;
}
template <>
bool try_mma<bf16>(const bf16* q, long long ldq, const bf16* kv, long long ldkv, int k_off, int v_off,
                   const float* bias, const int* kv_len, int S, int Tq, int L, int heads, int D, float scale, bf16* out,
                   long long ldo, cudaStream_t st) {
    // 16-byte copies of Q / K / V / O rows: row starts, offsets and the head stride 8-element aligned
    const bool aligned = ldq % 8 == 0 && ldkv % 8 == 0 && ldo % 8 == 0 && k_off % 8 == 0 && v_off % 8 == 0 &&
                         D % 8 == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(kv) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    if (!aligned) return false;
    switch (D) {
        case 32: return launch_mma<32>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, st);
        case 64: return launch_mma<64>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, st);
        case 72: return launch_mma<72>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, st);
        case 128: return launch_mma<128>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, scale, out, ldo, st);
        default: return false;
    }
}

}  // namespace

template <class T>
void cross_attention(const T* q, long long ldq, const T* kv, long long ldkv, int k_off, int v_off,
                     const float* bias, const int* kv_len, int S, int Tq, int L, int heads, int D, float scale,
                     T* out, long long ldo, int* err, cudaStream_t st) {
    SANA_REQUIRE(D >= 1 && D <= 128, "cross attention supports head_dim 1..128");
    SANA_REQUIRE(L >= 1, "cross attention needs at least one key");
    const size_t smem = 2 * static_cast<size_t>(L) * D * sizeof(T) + static_cast<size_t>(L) * 4 + 8;
    SANA_REQUIRE(smem <= 227 * 1024, "caption too long for the shared-memory key/value tile");
    if (S == 0 || Tq == 0) return;
    (void)err;
    if (try_mma<T>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st)) return;
    if (D <= 8) launch<T, 8>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
    else if (D <= 32) launch<T, 32>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
    else if (D <= 72) launch<T, 72>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
    else launch<T, 128>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
}

template void cross_attention<float>(const float*, long long, const float*, long long, int, int, const float*,
                                     const int*, int, int, int, int, int, float, float*, long long, int*,
                                     cudaStream_t);
template void cross_attention<bf16>(const bf16*, long long, const bf16*, long long, int, int, const float*,
                                    const int*, int, int, int, int, int, float, bf16*, long long, int*, cudaStream_t);

}  // namespace sana
