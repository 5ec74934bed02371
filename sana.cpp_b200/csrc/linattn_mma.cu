// ReLU linear attention (linear_attention_4d, transformer_ops.cpp:402-543) on bf16 tensor
// cores: both of its contractions are GEMMs, so they run as mma.sync m16n8k16 (bf16 operands,
// fp32 accumulation) and the op becomes bound by HBM instead of by CUDA-core FMAs.
//
//   state:  S'[d][n] = sum_t relu(k_t)[d] * [v_t | 1][n]      (n < D: relu(K)^T V; n = D: z)
//   apply:  o_t[n]   = (relu(q_t) . S'[:, n]) / (relu(q_t) . S'[:, D] + 1e-15)
//
// The ones column appended to V makes z = sum_t relu(k_t) the last column of the same
// product, and relu(q_t) . z the last column of the apply product. relu(k) and v are bf16
// (the activations' own precision), so the state's products are exact and only the fp32
// accumulation order differs from the reference's sequential loop. The state is split into
// bf16 hi + lo parts for the apply product (two MMAs), which keeps it to ~2^-16 relative.
//
// Kernel 1 (state): one CTA per (token split, head, sequence); K and V chunks of 128 (head
// dim 32) or 64 tokens stream through a 3-stage cp.async ring; warp (m-tile, token slice)
// accumulates a 16-row slab of S' over its slice of each chunk; slices are summed through
// shared memory and the split's D x (D+1) partial state is written to global memory.
// Kernel 2 (apply): one CTA per (token split, head, sequence) sums the partial states,
// converts them to hi/lo bf16 in shared memory, then streams Q chunks of 64 tokens; each
// warp computes 16 tokens' outputs, scales them by the reciprocal of the last column and
// writes bf16 rows.
#include "common.cuh"
#include "kernels.h"

namespace sana {
namespace {

constexpr int kChunk = 64;   // tokens per pipeline stage
constexpr int kStages = 3;

__host__ __device__ constexpr int dpad(int D) { return (D + 15) / 16 * 16; }
__host__ __device__ constexpr int npad(int D) { return D + 8; }
// Row stride (elements): a multiple of 8 (16-byte rows) that is 8 mod 16, so the eight
// 16-byte rows of an ldmatrix fragment fall in distinct bank groups.
__host__ __device__ constexpr int row_stride(int w) {
    return ((w + 7) / 8 * 8) % 16 == 8 ? (w + 7) / 8 * 8 : (w + 7) / 8 * 8 + 8;
}

__device__ __forceinline__ void cp_async16z(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16u : 0u)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t relu2(uint32_t x) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&x);
    v = __hmax2(v, __nv_bfloat162(__float2bfloat16_rn(0.f), __float2bfloat16_rn(0.f)));
    return *reinterpret_cast<uint32_t*>(&v);
}

// Copies a [CH, D] bf16 tile (rows t0.., columns from `src` of a row-major matrix with row
// stride ld) into shared memory rows of `stride` elements; rows at or past t_end are zero.
template <int D, int CH, int NT>
__device__ __forceinline__ void load_tile(uint32_t dst, const bf16* src, long long ld, int row0, int t0, int t_end,
                                          int stride) {
    constexpr int cpr = D / 8;
#pragma unroll
    for (int k = 0; k < (CH * cpr + NT - 1) / NT; ++k) {
        const int i = threadIdx.x + k * NT;
        if (CH * cpr % NT == 0 || i < CH * cpr) {
            const int r = i / cpr, c = i % cpr;
            const bool ok = t0 + r < t_end;
            const bf16* p = src + static_cast<long long>(row0 + (ok ? t0 + r : t_end - 1)) * ld + c * 8;
            cp_async16z(dst + static_cast<uint32_t>(r * stride + c * 8) * 2u, p, ok);
        }
    }
}

template <int D, int TS, int CH>
__global__ void __launch_bounds__(32 * (dpad(D) / 16) * TS)
    la_state_kernel(const bf16* __restrict__ kv, long long ld, int k_off, int v_off, int Tk, int heads, int splits,
                    int per_split, float* __restrict__ partial) {
    constexpr int DP = dpad(D), NP = npad(D), MT = DP / 16, NT = NP / 8, KS = row_stride(DP);
    constexpr int kTile = CH * KS;  // elements per stage per matrix
    constexpr int kThreads = 32 * MT * TS;
    extern __shared__ __align__(16) unsigned char smem[];
    bf16* Ks = reinterpret_cast<bf16*>(smem);
    bf16* Vs = Ks + kStages * kTile;
    const int split = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int t_begin = split * per_split, t_end = min(Tk, t_begin + per_split);
    const int nchunks = t_end > t_begin ? (t_end - t_begin + CH - 1) / CH : 0;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int mt = warp % MT, ts = warp / MT;
    if (DP > D) {  // pad columns of every stage stay zero
        for (int i = threadIdx.x; i < 2 * kStages * CH; i += blockDim.x)
            for (int c = D; c < DP; ++c) Ks[i * KS + c] = __float2bfloat16_rn(0.f);
    }
    const bf16* kbase = kv + k_off + h * D;
    const bf16* vbase = kv + v_off + h * D;
    const uint32_t ks0 = smem_u32(Ks), vs0 = smem_u32(Vs);
    auto issue = [&](int c) {
        if (c < nchunks) {
            const int stg = c % kStages;
            const int t0 = t_begin + c * CH;
            load_tile<D, CH, kThreads>(ks0 + static_cast<uint32_t>(stg * kTile) * 2u, kbase, ld, s * Tk, t0, t_end, KS);
            load_tile<D, CH, kThreads>(vs0 + static_cast<uint32_t>(stg * kTile) * 2u, vbase, ld, s * Tk, t0, t_end, KS);
        }
        cp_async_commit();
    };
    // the ones column of [V | 1]: B[k][n] = (n == 0) for the z n-tile
    const uint32_t ones = (lane / 4 == 0) ? 0x3F803F80u : 0u;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    __syncthreads();
    for (int c = 0; c < kStages - 1; ++c) issue(c);
    constexpr int kSlice = CH / TS;
    for (int c = 0; c < nchunks; ++c) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        issue(c + kStages - 1);
        const uint32_t kc = ks0 + static_cast<uint32_t>((c % kStages) * kTile) * 2u;
        const uint32_t vc = vs0 + static_cast<uint32_t>((c % kStages) * kTile) * 2u;
#pragma unroll
        for (int k0 = 0; k0 < kSlice; k0 += 16) {
            const int t = ts * kSlice + k0;
            uint32_t a[4];
            {
                const int i = lane % 8, j = lane / 8;
                ldsm_x4_t(kc + static_cast<uint32_t>((t + i + 8 * (j >> 1)) * KS + mt * 16 + 8 * (j & 1)) * 2u, a);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) a[r] = relu2(a[r]);
            const uint32_t vrow = vc + static_cast<uint32_t>((t + lane % 8 + 8 * ((lane / 8) & 1)) * KS) * 2u;
#pragma unroll
            for (int n = 0; n < NT - 1; ++n) {
                uint32_t b0, b1;
                ldsm_x2_t(vrow + static_cast<uint32_t>(n * 8) * 2u, b0, b1);
                mma16816(acc[n], a, b0, b1);
            }
            mma16816(acc[NT - 1], a, ones, ones);
        }
    }
    cp_async_wait<0>();
    __syncthreads();
    // sum the token slices through shared memory (the stage buffers are free now)
    float* red = reinterpret_cast<float*>(smem);  // [TS][DP][NP]
    {
        const int g = lane / 4, q2 = (lane % 4) * 2;
        float* r0 = red + (ts * DP + mt * 16 + g) * NP;
        float* r1 = r0 + 8 * NP;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            r0[n * 8 + q2] = acc[n][0];
            r0[n * 8 + q2 + 1] = acc[n][1];
            r1[n * 8 + q2] = acc[n][2];
            r1[n * 8 + q2 + 1] = acc[n][3];
        }
    }
    __syncthreads();
    float* out = partial + ((static_cast<long long>(s) * heads + h) * splits + split) * (D * (D + 1));
    for (int e = threadIdx.x; e < D * (D + 1); e += blockDim.x) {
        const int d = e / (D + 1), n = e % (D + 1);
        float v = 0.f;
#pragma unroll
        for (int i = 0; i < TS; ++i) v += red[(i * DP + d) * NP + n];
        out[e] = v;
    }
}

template <int D>
__global__ void __launch_bounds__(128)
    la_apply_kernel(const bf16* __restrict__ q, long long ldq, int q_off, int Tq, int heads, int splits,
                    const float* __restrict__ partial, int per_cta, bf16* __restrict__ out, long long ldo) {
    constexpr int DP = dpad(D), NP = npad(D), NT = NP / 8, QS = row_stride(DP), BS = row_stride(NP);
    constexpr int kTile = kChunk * QS;
    extern __shared__ __align__(16) unsigned char smem[];
    bf16* Bhi = reinterpret_cast<bf16*>(smem);  // [DP][BS]
    bf16* Blo = Bhi + DP * BS;
    bf16* Qs = Blo + DP * BS;                   // [kStages][kChunk][QS]
    const int blk = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
    const int t_begin = blk * per_cta, t_end = min(Tq, t_begin + per_cta);
    const int nchunks = t_end > t_begin ? (t_end - t_begin + kChunk - 1) / kChunk : 0;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const bf16* qbase = q + q_off + h * D;
    const uint32_t qs0 = smem_u32(Qs);
    auto issue = [&](int c) {
        if (c < nchunks)
            load_tile<D, kChunk, 128>(qs0 + static_cast<uint32_t>((c % kStages) * kTile) * 2u, qbase, ldq, s * Tq,
                                      t_begin + c * kChunk, t_end, QS);
        cp_async_commit();
    };
    for (int c = 0; c < kStages - 1; ++c) issue(c);
    // the summed state as hi + lo bf16, rows d >= D and columns n > D zero
    const float* P = partial + (static_cast<long long>(s) * heads + h) * splits * (D * (D + 1));
    for (int e = threadIdx.x; e < DP * NP; e += blockDim.x) {
        const int d = e / NP, n = e % NP;
        float v = 0.f;
        if (d < D && n <= D)
            for (int sp = 0; sp < splits; ++sp) v += P[sp * (D * (D + 1)) + d * (D + 1) + n];
        const bf16 hi = __float2bfloat16_rn(v);
        Bhi[d * BS + n] = hi;
        Blo[d * BS + n] = __float2bfloat16_rn(v - __bfloat162float(hi));
    }
    if (DP > D) {
        for (int i = threadIdx.x; i < kStages * kChunk; i += blockDim.x)
            for (int c = D; c < DP; ++c) Qs[i * QS + c] = __float2bfloat16_rn(0.f);
    }
    const uint32_t bhi0 = smem_u32(Bhi), blo0 = smem_u32(Blo);
    const int g = lane / 4, q2 = (lane % 4) * 2;
    for (int c = 0; c < nchunks; ++c) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        issue(c + kStages - 1);
        const int stg = c % kStages;
        const uint32_t qc = qs0 + static_cast<uint32_t>(stg * kTile) * 2u;
        // hi and lo parts accumulate separately (independent MMA chains), summed at the end
        float acc[NT][4], acl[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[n][r] = acl[n][r] = 0.f;
#pragma unroll
        for (int k0 = 0; k0 < DP; k0 += 16) {
            uint32_t a[4];
            ldsm_x4(qc + static_cast<uint32_t>((warp * 16 + lane % 8 + 8 * ((lane / 8) & 1)) * QS + k0 +
                                               8 * (lane / 16)) * 2u, a);
#pragma unroll
            for (int r = 0; r < 4; ++r) a[r] = relu2(a[r]);
            const uint32_t brow = static_cast<uint32_t>((k0 + lane % 8 + 8 * ((lane / 8) & 1)) * BS) * 2u;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                uint32_t b0, b1;
                ldsm_x2_t(bhi0 + brow + static_cast<uint32_t>(n * 8) * 2u, b0, b1);
                mma16816(acc[n], a, b0, b1);
                ldsm_x2_t(blo0 + brow + static_cast<uint32_t>(n * 8) * 2u, b0, b1);
                mma16816(acl[n], a, b0, b1);
            }
        }
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[n][r] += acl[n][r];
        // denominators: column D (first column of the last n-tile) of rows g and g + 8; one
        // reciprocal per row (within an ulp of dividing each element)
        const float den0 = __frcp_rn(__shfl_sync(0xffffffffu, acc[NT - 1][0], lane & ~3) + 1e-15f);
        const float den1 = __frcp_rn(__shfl_sync(0xffffffffu, acc[NT - 1][2], lane & ~3) + 1e-15f);
        // stage this warp's 16 output rows in its own (consumed) Q rows, then store them
        __syncwarp();
        bf16* orow = Qs + stg * kTile + (warp * 16) * QS;
#pragma unroll
        for (int n = 0; n < NT - 1; ++n) {
            *reinterpret_cast<__nv_bfloat162*>(orow + g * QS + n * 8 + q2) =
                __floats2bfloat162_rn(acc[n][0] * den0, acc[n][1] * den0);
            *reinterpret_cast<__nv_bfloat162*>(orow + (g + 8) * QS + n * 8 + q2) =
                __floats2bfloat162_rn(acc[n][2] * den1, acc[n][3] * den1);
        }
        __syncwarp();
        const int t0 = t_begin + c * kChunk + warp * 16;
        constexpr int cpr = D / 8;
        for (int i = lane; i < 16 * cpr; i += 32) {
            const int r = i / cpr, cc = i % cpr;
            if (t0 + r < t_end)
                *reinterpret_cast<uint4*>(out + static_cast<long long>(s * Tq + t0 + r) * ldo + h * D + cc * 8) =
                    *reinterpret_cast<const uint4*>(orow + r * QS + cc * 8);
        }
    }
    cp_async_wait<0>();
}

template <int D, int TS, int CH>
size_t state_smem() {
    constexpr int DP = dpad(D), NP = npad(D);
    const size_t ring = static_cast<size_t>(2) * kStages * CH * row_stride(DP) * 2;
    const size_t red = static_cast<size_t>(TS) * DP * NP * 4;
    return ring > red ? ring : red;
}
template <int D>
size_t apply_smem() {
    constexpr int DP = dpad(D);
    return static_cast<size_t>(2) * DP * row_stride(npad(D)) * 2 + static_cast<size_t>(kStages) * kChunk *
                                                                        row_stride(DP) * 2;
}

int sm_count() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
    }
    return cached[dev];
}

// Splits of T tokens (multiples of kChunk, at least `min_tokens` each) so that
// units * splits reaches two CTAs per SM where the tokens allow.
int token_splits(int units, int T, int min_tokens, int* per) {
    const int target = 2 * sm_count();
    int splits = std::max(1, (target + units - 1) / units);
    splits = std::min(splits, std::max(1, (T + min_tokens - 1) / min_tokens));
    *per = (T + splits - 1) / splits;
    *per = (*per + kChunk - 1) / kChunk * kChunk;
    return (T + *per - 1) / *per;
}

template <int D, int TS, int CH>
void launch(const bf16* q, long long ldq, int q_off, const bf16* kv, long long ldkv, int k_off, int v_off, int S,
            int Tq, int Tk, int heads, float* partial, bf16* out, long long ldo, cudaStream_t st) {
    static PerDeviceOnce attr;
    const size_t sm1 = state_smem<D, TS, CH>(), sm2 = apply_smem<D>();
    if (attr.pending()) {
        SANA_CUDA(cudaFuncSetAttribute(la_state_kernel<D, TS, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(sm1)));
        SANA_CUDA(cudaFuncSetAttribute(la_apply_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(sm2)));
        attr.mark();
    }
    // at least 128 tokens per state split: the partial-state buffer holds ceil(Tk / 128)
    // states per (sequence, head)
    int per1 = 0, per2 = 0;
    const int splits = token_splits(S * heads, Tk, 128, &per1);
    const int blocks = token_splits(S * heads, Tq, kChunk, &per2);
    constexpr int kWarps = (dpad(D) / 16) * TS;
    la_state_kernel<D, TS, CH><<<dim3(splits, heads, S), 32 * kWarps, sm1, st>>>(kv, ldkv, k_off, v_off, Tk, heads,
                                                                             splits, per1, partial);
    SANA_CUDA(cudaGetLastError());
    la_apply_kernel<D><<<dim3(blocks, heads, S), 128, sm2, st>>>(q, ldq, q_off, Tq, heads, splits, partial, per2,
                                                                 out, ldo);
    SANA_CUDA(cudaGetLastError());
}

}  // namespace

bool linattn_mma(const bf16* q, long long ldq, int q_off, const bf16* kv, long long ldkv, int k_off, int v_off,
                 int S, int Tq, int Tk, int heads, int D, float* partial, bf16* out, long long ldo,
                 cudaStream_t st) {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if ((D != 32 && D != 64 && D != 72) || ldq % 8 || ldkv % 8 || ldo % 8 || q_off % 8 || k_off % 8 || v_off % 8 ||
        !a16(q) || !a16(kv) || !a16(out) || Tk <= 0 || Tq <= 0)
        return false;
    switch (D) {
        case 32: launch<32, 4, 128>(q, ldq, q_off, kv, ldkv, k_off, v_off, S, Tq, Tk, heads, partial, out, ldo, st); break;
        case 64: launch<64, 2, 64>(q, ldq, q_off, kv, ldkv, k_off, v_off, S, Tq, Tk, heads, partial, out, ldo, st); break;
        default: launch<72, 2, 64>(q, ldq, q_off, kv, ldkv, k_off, v_off, S, Tq, Tk, heads, partial, out, ldo, st); break;
    }
    return true;
}

}  // namespace sana
