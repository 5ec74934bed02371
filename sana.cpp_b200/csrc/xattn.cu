// Masked softmax cross-attention to the caption (attention_4d, transformer_ops.cpp:348-392,
// with the additive bias of :357-388). One thread per query token and head; the head's
// keys and values for the sequence's live key range sit in shared memory. Two passes per
// query: the maximum of the scaled, biased scores, then exp(s - max) weighted sums,
// divided once by their total (the softmax of :318-334 followed by probs @ v).
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
    static bool attr = false;
    if (!attr) {
        SANA_CUDA(cudaFuncSetAttribute(xattn_kernel<T, DMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       227 * 1024));
        attr = true;
    }
    xattn_kernel<T, DMAX><<<dim3(ceil_div(Tq, kQ), heads, S), kQ, smem, st>>>(q, ldq, kv, ldkv, k_off, v_off, bias,
                                                                             kv_len, Tq, L, D, scale, out, ldo);
    SANA_CUDA(cudaGetLastError());
}

}  // namespace

template <class T>
void cross_attention(const T* q, long long ldq, const T* kv, long long ldkv, int k_off, int v_off,
                     const float* bias, const int* kv_len, int S, int Tq, int L, int heads, int D, float scale,
                     T* out, long long ldo, cudaStream_t st) {
    SANA_REQUIRE(D >= 1 && D <= 128, "cross attention supports head_dim 1..128");
    SANA_REQUIRE(L >= 1, "cross attention needs at least one key");
    const size_t smem = 2 * static_cast<size_t>(L) * D * sizeof(T) + static_cast<size_t>(L) * 4 + 8;
    SANA_REQUIRE(smem <= 227 * 1024, "caption too long for the shared-memory key/value tile");
    if (S == 0 || Tq == 0) return;
    if (D <= 8) launch<T, 8>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
    else if (D <= 32) launch<T, 32>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
    else if (D <= 72) launch<T, 72>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
    else launch<T, 128>(q, ldq, kv, ldkv, k_off, v_off, bias, kv_len, S, Tq, L, heads, D, scale, out, ldo, st);
}

template void cross_attention<float>(const float*, long long, const float*, long long, int, int, const float*,
                                     const int*, int, int, int, int, int, float, float*, long long, cudaStream_t);
template void cross_attention<bf16>(const bf16*, long long, const bf16*, long long, int, int, const float*,
                                    const int*, int, int, int, int, int, float, bf16*, long long, cudaStream_t);

}  // namespace sana
