// The text-encoder output contract on the device: the padded, sliced, uncond-first
// conditioning and its additive mask that the denoiser reads, assembled from the encoder's
// raw hidden states of several prompt pairs in one launch (gemma_encoder.cpp:188-244 does
// it for one pair on the host).
//
// Output rows follow the denoiser's batch convention for n pairs: rows 0..n-1 are the
// negative (uncond) branches, rows n..2n-1 the positive ones. A positive branch keeps its
// row 0 (BOS) and its last L-1 rows (select_rows_first_and_last, gemma_encoder.cpp:51-77);
// a negative branch is already L rows. The mask row is (1 - m) * -10000 with m = 1 on real
// tokens (gemma_encoder.cpp:177-184), which is -0.0 there and -10000 after.
#include "kernels.h"

namespace sana {

namespace {

__global__ void prompt_pairs_kernel(const float* __restrict__ negative, const float* __restrict__ positive,
                                    int pairs, int positive_rows, int hidden, int L, PromptPairCounts counts,
                                    int vec, float* __restrict__ enc, float* __restrict__ bias) {
    const int row = blockIdx.x;  // output row in [0, 2 * pairs * L)
    const int seq = row / L, t = row - seq * L;
    const bool pos = seq >= pairs;
    const int pair = pos ? seq - pairs : seq;
    long long src_row;
    if (!pos) {
        src_row = static_cast<long long>(pair) * L + t;
    } else {
        const int kept = t == 0 ? 0 : positive_rows - (L - 1) + (t - 1);
        src_row = static_cast<long long>(pair) * positive_rows + kept;
    }
    const float* src = (pos ? positive : negative) + src_row * hidden;
    float* dst = enc + static_cast<long long>(row) * hidden;
    if (vec) {  // rows of 16-byte vectors (hidden % 4 == 0, 16-byte aligned buffers)
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = src[i];
    }
    if (threadIdx.x == 0) {
        const float mask = t < counts.real[seq] ? 1.0f : 0.0f;
        bias[row] = (1.0f - mask) * -10000.0f;
    }
}

}  // namespace

void prompt_pairs(const float* negative, const float* positive, int pairs, int positive_rows, int hidden, int L,
                  const PromptPairCounts& counts, float* enc, float* bias, cudaStream_t st) {
    const bool vec = (hidden & 3) == 0 && (reinterpret_cast<uintptr_t>(negative) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(positive) & 15) == 0 && (reinterpret_cast<uintptr_t>(enc) & 15) == 0;
    const int threads = hidden >= 512 ? 256 : 128;
    prompt_pairs_kernel<<<2 * pairs * L, threads, 0, st>>>(negative, positive, pairs, positive_rows, hidden, L, counts,
                                                           vec ? 1 : 0, enc, bias);
    SANA_CUDA(cudaGetLastError());
}

}  // namespace sana
