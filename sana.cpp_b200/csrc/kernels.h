// Launchers for the memory-bound kernels of the denoiser path. Activations are
// token-major [rows, channels]; T is the activation type of the precision mode (bf16 fast
// path or fp32 check mode). Citations name the reference code each kernel replaces.
#pragma once

#include "common.cuh"

namespace sana {

// --- rowops.cu ---------------------------------------------------------------------------

// LayerNorm over the last dim (eps, optional affine) followed by AdaLN modulation
// x*(1 + scale) + shift (tensor.cpp:188-271 then :323-376). Row r belongs to sequence
// r / rows_per_seq; its shift/scale are mod[seq * mod_ld + shift_idx * C + c] and
// mod[seq * mod_ld + scale_idx * C + c].
template <class TO>
void ln_modulate(const float* x, long long rows, int C, int rows_per_seq, const float* gamma, const float* beta,
                 const float* mod, long long mod_ld, int shift_idx, int scale_idx, float eps, TO* out,
                 cudaStream_t st);

// AdaLN modulation alone, x*(1 + scale) + shift (modulate_3d_lastdim, tensor.cpp:323-376),
// with the same shift/scale addressing as ln_modulate.
void modulate(const float* x, long long rows, int C, int rows_per_seq, const float* mod, long long mod_ld,
              int shift_idx, int scale_idx, float* out, cudaStream_t st);

// RMSNorm (tensor.cpp:276-316): out = x / sqrt(mean(x^2) + eps) * w.
template <class TO>
void rms_norm(const float* x, long long rows, int C, float eps, const float* w, TO* out, cudaStream_t st);
// In place on rows of width C with row stride ld (rms_norm_3d_lastdim's arithmetic): the optional
// cross-attention q / k normalisation.
template <class T>
void rms_norm_rows(T* x, long long rows, int C, long long ld, float eps, const float* w, cudaStream_t st);

// Block modulation of compute_sana_block_modulation (transformer.cpp:496-542) for a run
// of blocks: mod[b][s][i] = tmod[s][i] + tables[b][i], i < 6C.
void block_modulation(const float* tmod, int S, int C, const float* tables, int n_blocks, float* mod,
                      cudaStream_t st);

// Final-layer modulation (compute_final_modulation, transformer.cpp:126-163):
// fmod[s][0][c] = emb[s][c] + table[0][c] (shift), fmod[s][1][c] = emb[s][c] + table[1][c].
void final_modulation(const float* emb, int S, int C, const float* table, float* fmod, cudaStream_t st);

// NCHW latents [images, Cl, HW] -> token rows [seqs * HW, Cl]; sequence s reads image
// s % images (repeat_batch_4d_local, transformer.cpp:55-75, then the 1x1 conv's input
// order; grid_to_tokens_3d, tensor.cpp:427).
template <class TO>
void patch_tokens(const float* lat, int images, int seqs, int Cl, int HW, TO* out, cudaStream_t st);

// Sinusoidal timestep features for all sequences: out[s] = table row (precomputed on the
// host with the reference's arithmetic) broadcast; used only to fill [S, 256].
template <class TO>
void broadcast_rows(const float* row, int S, int width, TO* out, cudaStream_t st);

// split_heads_3d ([B, T, H*D] -> [B, H, T, D], to_heads) and merge_heads_4d (the inverse),
// transformer_ops.cpp:83-171; fp32.
void permute_heads(const float* in, float* out, int B, int T, int H, int D, bool to_heads, cudaStream_t st);
// softmax_lastdim_4d (transformer_ops.cpp:278-339) over `rows` rows of n values; fp32.
void softmax_rows(const float* in, long long rows, int n, float* out, cudaStream_t st);

// Effective key count per caption row: 1 + the last index whose additive bias exceeds
// -1000 (L when every key is masked, so the softmax runs over all of them as the
// reference does). Keys past it carry <= -1000 and contribute exactly 0 in fp32.
void caption_kv_len(const float* bias, int S, int L, int* kv_len, cudaStream_t st);

// Real-token count of each output sequence of prompt_pairs (negatives first).
constexpr int kMaxPromptPairs = 64;
struct PromptPairCounts {
    int real[2 * kMaxPromptPairs];
};
// Text-encoder output contract (conditioning.cu): negative [pairs, L, hidden] and positive
// [pairs, positive_rows, hidden] fp32 hidden states -> enc [2 * pairs, L, hidden] (negatives
// first, positives sliced to row 0 + last L-1 rows) and bias [2 * pairs, 1, L].
void prompt_pairs(const float* negative, const float* positive, int pairs, int positive_rows, int hidden, int L,
                  const PromptPairCounts& counts, float* enc, float* bias, cudaStream_t st);

// One fused classifier-free-guidance + DPM-Solver++ update (apply_classifier_free_guidance,
// transformer.cpp:570-602; step_sana_scheduler, scheduler.cpp:272-318) on NCHW latents:
//   guided = u + g (c - u) from token-major noise rows (uncond sequences first)
//   x0     = x - sigma_s * guided                        (convert, scheduler.cpp:155-173)
//   x'     = a x + b x0 [+ c (x0 - x0_prev) / r0]         (first / midpoint second order)
// x0 is stored to hist_cur; hist_prev holds the previous step's x0.
struct SchedCoef {
    float guidance;
    float sigma_s;
    float a, b, c;
    float inv_r0;
    int second_order;
};
// One thread waits (bounded by the handle's wait limit) for *flag == expect; on expiry the
// error word records kTimeout (the failure-detection self-test).
void wait_flag(const int* flag, int expect, int* err, cudaStream_t st);

void cfg_scheduler_step(const float* noise, int images, int Cl, int HW, float* lat, float* hist_cur,
                        const float* hist_prev, SchedCoef k, cudaStream_t st);

// --- cfgpair.cu: guidance across two GPUs ------------------------------------------------------

// One GPU's view of the exchange: its own receive buffers (2 x capacity floats, written by the
// peer), flags (incremented by the peer) and per-slot exchange counts, and the peer's receive
// buffers and flags mapped through CUDA IPC.
constexpr int kPairBlocks = 64;
struct PairLink {
    float* recv;
    float* peer_recv;
    int* flags;
    int* peer_flags;
    int* count;
    long long capacity;  // floats per receive buffer, a multiple of 4
};
// CFG + scheduler update of this GPU's branch (0 unconditional, 1 conditional) against the
// peer's: pushes own_noise (token-major [images * HW, Cl]) to the peer, waits for the peer's
// (bounded; kTimeout in err on expiry, the latents then left unchanged) and updates lat /
// hist_cur as cfg_scheduler_step does.
void cfg_pair_step(const float* own_noise, const PairLink& link, int images, int Cl, int HW, float* lat,
                   float* hist_cur, const float* hist_prev, SchedCoef k, int branch, int* err, cudaStream_t st);

// The update alone on already-converted outputs: out = a x + b m0 [+ c (m0 - m1) / r0]
// (sana_scheduler_first_order_update / _second_order_update, scheduler.cpp:175-270).
void scheduler_update(const float* m0, const float* m1, const float* x, long long n, SchedCoef k, float* out,
                      cudaStream_t st);

// Weight repacking: src fp32 [rows, cols] -> dst [cols, rows] (transpose) or [rows, cols]
// (copy), converted to T. Used to turn the reference's [in, out] linear weights into the
// K-major [out, in] operand.
template <class TO>
void repack(const float* src, int rows, int cols, bool transpose, TO* dst, cudaStream_t st);

// fp32 -> T elementwise conversion.
template <class TO>
void convert(const float* src, long long n, TO* dst, cudaStream_t st);

// --- linattn.cu ---------------------------------------------------------------------------

// ReLU linear attention (linear_attention_4d, transformer_ops.cpp:402-543) on token-major
// q/k/v columns of a fused projection: head h of sequence s uses columns
// [q_off + h*D, +D) etc. of rows s*T .. s*T+T-1 with row stride ld.
// Phase 1 writes per-chunk partial states [S, H, chunks, (D+1), D] (S = relu(K)^T V rows
// 0..D-1, row D = sum of relu(K)); phase 2 sums the chunks and applies
// out = relu(q) S / (relu(q) . z + 1e-15).
// q rows at column q_off + h*D of `q` (stride ldq); k and v rows of `kv` (stride ldkv).
// partial must hold S * heads * (linattn_chunks(Tk) + 1) * (D + 1) * D floats.
int linattn_chunks(int T);
// bf16 tensor-core path of linear_attention (head_dim 32, 64 or 72, 16-byte aligned rows);
// returns false, launching nothing, when the shape or alignment does not fit it.
bool linattn_mma(const bf16* q, long long ldq, int q_off, const bf16* kv, long long ldkv, int k_off, int v_off,
                 int S, int Tq, int Tk, int heads, int D, float* partial, bf16* out, long long ldo,
                 cudaStream_t st);
template <class T>
void linear_attention(const T* q, long long ldq, int q_off, const T* kv, long long ldkv, int k_off, int v_off,
                      int S, int Tq, int Tk, int heads, int D, float* partial, T* out, long long ldo,
                      cudaStream_t st);

// --- xattn.cu -----------------------------------------------------------------------------

// Masked softmax cross-attention (attention_4d, transformer_ops.cpp:348-392): per head,
// softmax(q k^T * scale + bias) v over the first kv_len[s] keys. q rows s*Tq.. at column
// h*D (stride ldq); k/v rows s*L.. at columns k_off + h*D / v_off + h*D (stride ldkv);
// bias fp32 [S, L] or null; out rows at column h*D (stride ldo). bf16 runs on tensor cores
// (mma.sync) for head dims 32 / 64 / 72 / 128 with 16-byte aligned rows, fp32 on CUDA cores.
// err: the handle's device error word.
template <class T>
void cross_attention(const T* q, long long ldq, const T* kv, long long ldkv, int k_off, int v_off,
                     const float* bias, const int* kv_len, int S, int Tq, int L, int heads, int D, float scale,
                     T* out, long long ldo, int* err, cudaStream_t st);

// --- dwglu.cu -----------------------------------------------------------------------------

// Depthwise 3x3 conv (zero padding, bias) over all E channels of the NHWC grid followed by
// the GLU gate data * silu(gate) (depthwise_conv2d_3x3, common_ops.cpp:510-572, then
// glumb_conv's split and gate, :745-758). in [S*H*W, E] (stride ldi), out [S*H*W, E/2].
template <class T>
// err: the device error word (a bounded wait records kTimeout there).
void depthwise_glu(const T* in, long long ldi, int S, int H, int W, int E, const float* w, const float* b, T* out,
                   long long ldo, int* err, cudaStream_t st);

// The depthwise 3x3 conv alone (depthwise_conv2d_3x3), all C channels, NHWC fp32.
void depthwise3x3(const float* in, int S, int H, int W, int C, const float* w, const float* b, float* out,
                  cudaStream_t st);

}  // namespace sana
