// Generic CUDA-core GEMM with the fused epilogue of gemm.h. Serves the fp32 check mode
// (fp32 operands, fp32 FMA accumulation in increasing k, like gemm_row_major's scalar
// loop, common_ops.cpp:49-63), the reference's tiny known-answer shapes, and any operand
// layout the tensor-core kernel does not take. 64 x 64 output tile per 256-thread block,
// 4 x 4 outputs per thread, k-steps of 16 staged through shared memory.
#include "gemm.h"

namespace sana {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

template <class TA, class TB>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TA* __restrict__ A, long long lda,
                                                        const TB* __restrict__ B, long long ldb, int M, int N,
                                                        int K, Epilogue ep) {
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    const int tx = threadIdx.x % 16;  // column group
    const int ty = threadIdx.x / 16;  // row group
    const int m0 = blockIdx.y * TM;
    const int n0 = blockIdx.x * TN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += TK) {
        for (int i = threadIdx.x; i < TM * TK; i += 256) {
            const int r = i / TK, k = i % TK;
            const int gr = m0 + r, gk = k0 + k;
            As[k][r] = (gr < M && gk < K) ? to_f(A[static_cast<long long>(gr) * lda + gk]) : 0.0f;
        }
        for (int i = threadIdx.x; i < TN * TK; i += 256) {
            const int c = i / TK, k = i % TK;
            const int gc = n0 + c, gk = k0 + k;
            Bs[k][c] = (gc < N && gk < K) ? to_f(B[static_cast<long long>(gc) * ldb + gk]) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < TK; ++k) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = m0 + ty * 4 + i;
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n >= N) continue;
            float x = acc[i][j];
            if (ep.bias) x += ep.bias[n];
            if (ep.act == kActSilu) x = silu(x);
            else if (ep.act == kActGelu) x = gelu_tanh(x);
            if (ep.resid) {
                const float g = ep.gate ? ep.gate[static_cast<long long>(r / ep.rows_per_gate) * ep.gate_ld + n] : 1.0f;
                x = ep.resid[static_cast<long long>(r) * ep.ldr + n] + g * x;
            }
            if (ep.out) {
                const long long idx = static_cast<long long>(r) * ep.ldo + n;
                if (ep.out_bf16) static_cast<bf16*>(ep.out)[idx] = __float2bfloat16_rn(x);
                else static_cast<float*>(ep.out)[idx] = x;
            }
            if (ep.out2) {
                const long long idx = static_cast<long long>(r) * ep.ldo2 + n;
                const float y = ep.act2 == kActSilu ? silu(x) : x;
                if (ep.out2_bf16) static_cast<bf16*>(ep.out2)[idx] = __float2bfloat16_rn(y);
                else static_cast<float*>(ep.out2)[idx] = y;
            }
        }
    }
}

template <class TA, class TB>
void launch(const GemmProblem& p, cudaStream_t stream) {
    dim3 grid(ceil_div(p.N, TN), ceil_div(p.M, TM));
    gemm_simt_kernel<TA, TB><<<grid, 256, 0, stream>>>(static_cast<const TA*>(p.A), p.lda,
                                                        static_cast<const TB*>(p.B), p.ldb, p.M, p.N, p.K, p.ep);
    SANA_CUDA(cudaGetLastError());
}

}  // namespace

void gemm_simt(const GemmProblem& p, cudaStream_t stream) {
    if (p.M == 0 || p.N == 0) return;
    if (p.a_bf16 && p.b_bf16) launch<bf16, bf16>(p, stream);
    else if (p.a_bf16) launch<bf16, float>(p, stream);
    else if (p.b_bf16) launch<float, bf16>(p, stream);
    else launch<float, float>(p, stream);
}

}  // namespace sana
