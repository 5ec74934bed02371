/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle for the Sana denoiser hot path (see sana_oracle.h).
 *
 * Restates the reference's fp32 Linux code path: the arithmetic and the order of every
 * floating-point accumulation follow the reference lines cited per function, so that the
 * oracle agrees with the compiled reference to a few ulps (tests/test_oracle_pin.py).
 * OpenMP parallelises over independent rows / heads / planes only; no reduction changes
 * order. Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU leg, never by the
 * product.
 */
#include "sana_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static _Thread_local char g_err[256];

static int fail(int code, const char *msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return code;
}

const char *orc_last_error(void) { return g_err; }

#define ORC_INVALID(msg) return fail(1, msg)

/* ------------------------------------------------------------------------------------
 * Random numbers: torch.randn on a CPU generator, as restated by torch_rng.cpp:9-68.
 * MT19937 (Matsumoto & Nishimura, 1998), 24-bit uniforms in [0,1), Box-Muller on
 * complete blocks of 16 (first 8 -> radius, last 8 -> angle), and a re-drawn final
 * block of 16 when the size is not a multiple of 16.
 * ---------------------------------------------------------------------------------- */
typedef struct {
    uint32_t s[624];
    int idx;
} mt_state;

static void mt_seed(mt_state *m, uint32_t seed) {
    m->s[0] = seed;
    for (int i = 1; i < 624; ++i) {
        m->s[i] = 1812433253u * (m->s[i - 1] ^ (m->s[i - 1] >> 30)) + (uint32_t)i;
    }
    m->idx = 624;
}

static uint32_t mt_next(mt_state *m) {
    if (m->idx >= 624) {
        for (int i = 0; i < 624; ++i) {
            uint32_t y = (m->s[i] & 0x80000000u) | (m->s[(i + 1) % 624] & 0x7fffffffu);
            uint32_t v = m->s[(i + 397) % 624] ^ (y >> 1);
            if (y & 1u) v ^= 0x9908b0dfu;
            m->s[i] = v;
        }
        m->idx = 0;
    }
    uint32_t y = m->s[m->idx++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

static float uniform24(mt_state *m) {
    return (float)(mt_next(m) & 0xffffffu) * (1.0f / 16777216.0f);
}

static void box_muller16(float *d) {
    const double pi = 3.14159265358979323846;
    for (int j = 0; j < 8; ++j) {
        const float u1 = 1.0f - d[j];
        const float u2 = d[j + 8];
        const float radius = sqrtf(-2.0f * logf(u1));
        const float theta = (float)(2.0 * pi * (double)u2);
        d[j] = radius * cosf(theta);
        d[j + 8] = radius * sinf(theta);
    }
}

int orc_randn(float *out, size_t n, uint64_t seed) {
    if (n < 16) ORC_INVALID("randn needs at least 16 elements");
    mt_state m;
    mt_seed(&m, (uint32_t)(seed & 0xffffffffu));
    for (size_t i = 0; i < n; ++i) out[i] = uniform24(&m);
    size_t i = 0;
    for (; i + 16 <= n; i += 16) box_muller16(out + i);
    if (n % 16 != 0) {
        float *tail = out + n - 16;
        for (int j = 0; j < 16; ++j) tail[j] = uniform24(&m);
        box_muller16(tail);
    }
    return 0;
}

/* ------------------------------------------------------------------------------------
 * Dense algebra.
 * gemm: C[M,N] = bias + A[M,K] B[K,N] (or B stored [N,K] when bt), each output summed
 * over k in increasing order starting from the bias, as gemm_row_major's scalar path
 * (common_ops.cpp:49-63). Rows are processed in blocks of 8 so that each row of B is
 * read once per block; the per-element order is unchanged.
 * ---------------------------------------------------------------------------------- */
static void gemm(const float *A, const float *Bm, const float *bias, float *C, size_t M, size_t K,
                 size_t N, int bt) {
    const long long Mb = (long long)((M + 7) / 8);
#pragma omp parallel for schedule(dynamic, 1) if (M * K * N > 65536)
    for (long long blk = 0; blk < Mb; ++blk) {
        const size_t m0 = (size_t)blk * 8;
        const size_t m1 = m0 + 8 < M ? m0 + 8 : M;
        for (size_t m = m0; m < m1; ++m) {
            float *c = C + m * N;
            for (size_t n = 0; n < N; ++n) c[n] = bias ? bias[n] : 0.0f;
        }
        if (!bt) {
            for (size_t k = 0; k < K; ++k) {
                const float *b = Bm + k * N;
                for (size_t m = m0; m < m1; ++m) {
                    const float a = A[m * K + k];
                    float *c = C + m * N;
                    for (size_t n = 0; n < N; ++n) c[n] += a * b[n];
                }
            }
        } else {
            for (size_t m = m0; m < m1; ++m) {
                float *c = C + m * N;
                for (size_t k = 0; k < K; ++k) {
                    const float a = A[m * K + k];
                    for (size_t n = 0; n < N; ++n) c[n] += a * Bm[n * K + k];
                }
            }
        }
    }
}

/* linear_3d_lastdim (common_ops.cpp:177-209): rows = B*T, weight [K, N]. */
int orc_linear_3d(const float *x, size_t B, size_t T, size_t K, const float *w, const float *bias,
                  size_t N, float *out) {
    gemm(x, w, bias, out, B * T, K, N, 0);
    return 0;
}

/* Tensor::transpose_2d (tensor.cpp:162-183) of a PyTorch [out, in] weight. */
static float *transpose_new(const float *src, size_t rows, size_t cols) {
    float *dst = (float *)malloc(rows * cols * sizeof(float));
    for (size_t i = 0; i < rows; ++i)
        for (size_t j = 0; j < cols; ++j) dst[j * rows + i] = src[i * cols + j];
    return dst;
}

/* ------------------------------------------------------------------------------------
 * Row operations.
 * ---------------------------------------------------------------------------------- */

/* layer_norm_3d_lastdim, scalar path (tensor.cpp:236-267). */
int orc_layer_norm(const float *x, size_t B, size_t T, size_t C, float eps, const float *gamma,
                   const float *beta, float *out) {
    const long long R = (long long)(B * T);
#pragma omp parallel for if (R * (long long)C > 65536)
    for (long long r = 0; r < R; ++r) {
        const float *row = x + (size_t)r * C;
        float *o = out + (size_t)r * C;
        float mean = 0.0f;
        for (size_t h = 0; h < C; ++h) mean += row[h];
        mean /= (float)C;
        float var = 0.0f;
        for (size_t h = 0; h < C; ++h) {
            const float d = row[h] - mean;
            var += d * d;
        }
        var /= (float)C;
        const float inv_std = 1.0f / sqrtf(var + eps);
        for (size_t h = 0; h < C; ++h) {
            float v = (row[h] - mean) * inv_std;
            if (gamma) v *= gamma[h];
            if (beta) v += beta[h];
            o[h] = v;
        }
    }
    return 0;
}

/* rms_norm_3d_lastdim (tensor.cpp:276-316). */
int orc_rms_norm(const float *x, size_t B, size_t T, size_t C, float eps, const float *weight,
                 float *out) {
    const long long R = (long long)(B * T);
#pragma omp parallel for if (R * (long long)C > 65536)
    for (long long r = 0; r < R; ++r) {
        const float *row = x + (size_t)r * C;
        float *o = out + (size_t)r * C;
        float ms = 0.0f;
        for (size_t h = 0; h < C; ++h) ms += row[h] * row[h];
        ms /= (float)C;
        const float inv = 1.0f / sqrtf(ms + eps);
        for (size_t h = 0; h < C; ++h) {
            float v = row[h] * inv;
            if (weight) v *= weight[h];
            o[h] = v;
        }
    }
    return 0;
}

/* modulate_3d_lastdim, scalar path (tensor.cpp:364-372); shift/scale [B, C]. */
int orc_modulate(const float *x, size_t B, size_t T, size_t C, const float *shift,
                 const float *scale, float *out) {
    for (size_t b = 0; b < B; ++b)
        for (size_t t = 0; t < T; ++t)
            for (size_t h = 0; h < C; ++h) {
                const size_t i = (b * T + t) * C + h;
                out[i] = x[i] * (1.0f + scale[b * C + h]) + shift[b * C + h];
            }
    return 0;
}

/* Tensor::silu_inplace scalar path (tensor.cpp:551-555). */
static void silu_inplace(float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* gelu_tanh (transformer_ops.cpp:15-18). */
static void gelu_tanh_inplace(float *x, size_t n) {
    const float alpha = sqrtf(2.0f / (float)3.14159265358979323846);
    for (size_t i = 0; i < n; ++i) {
        const float v = x[i];
        x[i] = 0.5f * v * (1.0f + tanhf(alpha * (v + 0.044715f * v * v * v)));
    }
}

/* ------------------------------------------------------------------------------------
 * Attention.
 * ---------------------------------------------------------------------------------- */

/* linear_attention_4d, scalar path (transformer_ops.cpp:496-538): per (b, h)
 *   S[row][d] = sum_t v[t,row] relu(k[t,d]),  z[d] = sum_t relu(k[t,d])   (t ascending)
 *   out[t,row] = (sum_d S[row][d] relu(q[t,d])) / (sum_d z[d] relu(q[t,d]) + 1e-15) */
int orc_linear_attention(const float *q, const float *k, const float *v, size_t B, size_t H,
                         size_t Tq, size_t Tk, size_t D, float *out) {
    const long long BH = (long long)(B * H);
#pragma omp parallel for schedule(dynamic, 1)
    for (long long bh = 0; bh < BH; ++bh) {
        float *S = (float *)calloc((D + 1) * D, sizeof(float));
        const float *kb = k + (size_t)bh * Tk * D;
        const float *vb = v + (size_t)bh * Tk * D;
        const float *qb = q + (size_t)bh * Tq * D;
        float *ob = out + (size_t)bh * Tq * D;
        for (size_t t = 0; t < Tk; ++t) {
            for (size_t d = 0; d < D; ++d) {
                const float kv = kb[t * D + d] > 0.0f ? kb[t * D + d] : 0.0f;
                for (size_t row = 0; row < D; ++row) S[row * D + d] += vb[t * D + row] * kv;
                S[D * D + d] += kv;
            }
        }
        for (size_t t = 0; t < Tq; ++t) {
            for (size_t row = 0; row < D; ++row) {
                float num = 0.0f;
                for (size_t d = 0; d < D; ++d) {
                    const float qv = qb[t * D + d] > 0.0f ? qb[t * D + d] : 0.0f;
                    num += S[row * D + d] * qv;
                }
                ob[t * D + row] = num;
            }
            float den = 0.0f;
            for (size_t d = 0; d < D; ++d) {
                const float qv = qb[t * D + d] > 0.0f ? qb[t * D + d] : 0.0f;
                den += S[D * D + d] * qv;
            }
            den += 1e-15f;
            for (size_t row = 0; row < D; ++row) ob[t * D + row] /= den;
        }
        free(S);
    }
    return 0;
}

/* attention_4d (transformer_ops.cpp:348-392): scores = q k^T (gemm with transposed B,
 * transformer_ops.cpp:214-221), times (float)(1/sqrt((double)D)) (:355), plus bias
 * [B,1,Tk] (:381-383), softmax_lastdim_4d scalar path (:318-334), then probs v
 * (attention_values_4d, :268). */
int orc_attention(const float *q, const float *k, const float *v, size_t B, size_t H, size_t Tq,
                  size_t Tk, size_t D, const float *bias, float *out) {
    const float scale = (float)(1.0 / sqrt((double)D));
    const long long BH = (long long)(B * H);
#pragma omp parallel for schedule(dynamic, 1)
    for (long long bh = 0; bh < BH; ++bh) {
        const size_t b = (size_t)bh / H;
        float *s = (float *)malloc(Tq * Tk * sizeof(float));
        gemm(q + (size_t)bh * Tq * D, k + (size_t)bh * Tk * D, NULL, s, Tq, D, Tk, 1);
        for (size_t i = 0; i < Tq * Tk; ++i) s[i] *= scale;
        if (bias) {
            for (size_t i = 0; i < Tq; ++i)
                for (size_t j = 0; j < Tk; ++j) s[i * Tk + j] += bias[b * Tk + j];
        }
        for (size_t i = 0; i < Tq; ++i) {
            float *row = s + i * Tk;
            float mx = row[0];
            for (size_t j = 0; j < Tk; ++j)
                if (row[j] > mx) mx = row[j];
            float den = 0.0f;
            for (size_t j = 0; j < Tk; ++j) {
                const float e = expf(row[j] - mx);
                row[j] = e;
                den += e;
            }
            const float r = 1.0f / den;
            for (size_t j = 0; j < Tk; ++j) row[j] *= r;
        }
        gemm(s, v + (size_t)bh * Tk * D, NULL, out + (size_t)bh * Tq * D, Tq, Tk, D, 0);
        free(s);
    }
    return 0;
}

/* split_heads_3d (transformer_ops.cpp:83-126): [B,T,h*d] -> [B,h,T,d]. */
static void split_heads(const float *x, size_t B, size_t T, size_t Hn, size_t D, float *out) {
    for (size_t b = 0; b < B; ++b)
        for (size_t h = 0; h < Hn; ++h)
            for (size_t t = 0; t < T; ++t)
                memcpy(out + ((b * Hn + h) * T + t) * D, x + (b * T + t) * Hn * D + h * D,
                       D * sizeof(float));
}

/* merge_heads_4d (transformer_ops.cpp:133-171). */
static void merge_heads(const float *x, size_t B, size_t Hn, size_t T, size_t D, float *out) {
    for (size_t b = 0; b < B; ++b)
        for (size_t h = 0; h < Hn; ++h)
            for (size_t t = 0; t < T; ++t)
                memcpy(out + (b * T + t) * Hn * D + h * D, x + ((b * Hn + h) * T + t) * D,
                       D * sizeof(float));
}

/* ------------------------------------------------------------------------------------
 * Convolutions (NCHW).
 * ---------------------------------------------------------------------------------- */

/* conv2d_1x1, scalar path (common_ops.cpp:260-309, 389-403): out[b,oc,s] = bias[oc] +
 * sum_ic w[oc,ic] x[b,ic,s], ic ascending. */
int orc_conv1x1(const float *x, size_t B, size_t Cin, size_t H, size_t W, const float *w,
                const float *bias, size_t Cout, float *out) {
    const size_t S = H * W;
    const long long BO = (long long)(B * Cout);
#pragma omp parallel for schedule(static) if (BO * (long long)(Cin * S) > 65536)
    for (long long bo = 0; bo < BO; ++bo) {
        const size_t b = (size_t)bo / Cout, oc = (size_t)bo % Cout;
        float *o = out + (b * Cout + oc) * S;
        for (size_t s = 0; s < S; ++s) o[s] = bias ? bias[oc] : 0.0f;
        for (size_t ic = 0; ic < Cin; ++ic) {
            const float wv = w[oc * Cin + ic];
            const float *xi = x + (b * Cin + ic) * S;
            for (size_t s = 0; s < S; ++s) o[s] += wv * xi[s];
        }
    }
    return 0;
}

/* depthwise_conv2d_3x3, scalar plane path (common_ops.cpp:484-505): zero padding, taps
 * summed ky-major then kx, bias added last. */
int orc_depthwise3x3(const float *x, size_t B, size_t C, size_t H, size_t W, const float *w,
                     const float *bias, float *out) {
    const long long P = (long long)(B * C);
#pragma omp parallel for schedule(static) if (P * (long long)(H * W) > 65536)
    for (long long p = 0; p < P; ++p) {
        const size_t c = (size_t)p % C;
        const float *xi = x + (size_t)p * H * W;
        float *o = out + (size_t)p * H * W;
        for (size_t y = 0; y < H; ++y) {
            for (size_t xx = 0; xx < W; ++xx) {
                float sum = 0.0f;
                for (int ky = 0; ky < 3; ++ky) {
                    for (int kx = 0; kx < 3; ++kx) {
                        const long iy = (long)y + ky - 1, ix = (long)xx + kx - 1;
                        if (iy >= 0 && iy < (long)H && ix >= 0 && ix < (long)W) {
                            sum += xi[(size_t)iy * W + (size_t)ix] * w[(c * 3 + (size_t)ky) * 3 + (size_t)kx];
                        }
                    }
                }
                if (bias) sum += bias[c];
                o[y * W + xx] = sum;
            }
        }
    }
    return 0;
}

/* glumb_conv (common_ops.cpp:733-761). */
int orc_glumb_conv(const float *x, size_t B, size_t Cin, size_t H, size_t W, const float *w_inv,
                   const float *b_inv, size_t E, const float *w_dw, const float *b_dw,
                   const float *w_pt, size_t Cout, float *out) {
    if (E % 2 != 0) ORC_INVALID("channel count must be even");
    const size_t S = H * W, half = E / 2;
    float *h = (float *)malloc(B * E * S * sizeof(float));
    float *d = (float *)malloc(B * E * S * sizeof(float));
    float *g = (float *)malloc(B * half * S * sizeof(float));
    orc_conv1x1(x, B, Cin, H, W, w_inv, b_inv, E, h);
    silu_inplace(h, B * E * S);
    orc_depthwise3x3(h, B, E, H, W, w_dw, b_dw, d);
    for (size_t b = 0; b < B; ++b) {
        const float *data = d + b * E * S;
        const float *gate = data + half * S;
        float *gb = g + b * half * S;
        for (size_t i = 0; i < half * S; ++i) {
            const float gv = gate[i] / (1.0f + expf(-gate[i]));
            gb[i] = data[i] * gv;
        }
    }
    orc_conv1x1(g, B, half, H, W, w_pt, NULL, Cout, out);
    free(h);
    free(d);
    free(g);
    return 0;
}

/* project_caption_context (transformer_ops.cpp:64-76): linear, GELU-tanh, linear,
 * RMSNorm(eps 1e-5, weight). Weights [in, out]. */
int orc_project_caption(const float *enc, size_t B, size_t L, size_t Din, const float *w1,
                        const float *b1, size_t C, const float *w2, const float *b2,
                        const float *norm_w, float *out) {
    float *h = (float *)malloc(B * L * C * sizeof(float));
    float *p = (float *)malloc(B * L * C * sizeof(float));
    gemm(enc, w1, b1, h, B * L, Din, C, 0);
    gelu_tanh_inplace(h, B * L * C);
    gemm(h, w2, b2, p, B * L, C, C, 0);
    orc_rms_norm(p, B, L, C, 1e-5f, norm_w, out);
    free(h);
    free(p);
    return 0;
}

/* apply_classifier_free_guidance (transformer.cpp:595-599). */
int orc_cfg(const float *noise, size_t B, size_t Cl, size_t H, size_t W, float g, float *out) {
    const size_t n = B * Cl * H * W;
    for (size_t i = 0; i < n; ++i) out[i] = noise[i] + g * (noise[n + i] - noise[i]);
    return 0;
}

/* ------------------------------------------------------------------------------------
 * Scheduler: DPM-Solver++ (2M) on flow sigmas (scheduler.cpp).
 * ---------------------------------------------------------------------------------- */

/* build_sana_scheduler_timesteps (scheduler.cpp:89-141), default config but flow_shift. */
int orc_scheduler_schedule(size_t n, float flow_shift, float *timesteps, float *sigmas) {
    if (n == 0) ORC_INVALID("num_inference_steps must be positive");
    const float denom = 1000.0f;
    float *shifted = (float *)malloc((n + 1) * sizeof(float));
    for (size_t i = 0; i <= n; ++i) {
        const float alpha = 1.0f + (1.0f / denom - 1.0f) * ((float)i / (float)n);
        const float sigma = 1.0f - alpha;
        shifted[i] = flow_shift * sigma / (1.0f + (flow_shift - 1.0f) * sigma);
    }
    for (size_t i = 0; i < n; ++i) {
        const float s = shifted[n - i];
        sigmas[i] = s;
        timesteps[i] = (float)(int)(s * denom);
    }
    sigmas[n] = 0.0f;
    free(shifted);
    return 0;
}

/* lambda = log(alpha) - log(sigma) with alpha = 1 - sigma (scheduler.cpp:71-81). */
static float lambda_of(float sigma) { return logf(1.0f - sigma) - logf(sigma); }

/* step_sana_scheduler (scheduler.cpp:272-318) applied n_steps times; the converted
 * outputs (:155-173) keep a history of two; first order (:175-205) at the first step
 * and the last, midpoint second order (:207-260) elsewhere. */
int orc_scheduler_run(size_t n_steps, float flow_shift, const float *model_outputs,
                      const float *sample, size_t numel, float *samples_out) {
    float *ts = (float *)malloc(n_steps * sizeof(float));
    float *sg = (float *)malloc((n_steps + 1) * sizeof(float));
    int rc = orc_scheduler_schedule(n_steps, flow_shift, ts, sg);
    if (rc) {
        free(ts);
        free(sg);
        return rc;
    }
    float *x = (float *)malloc(numel * sizeof(float));
    float *m0 = (float *)malloc(numel * sizeof(float));
    float *m1 = (float *)malloc(numel * sizeof(float));
    memcpy(x, sample, numel * sizeof(float));
    size_t hist = 0, lower = 0;
    for (size_t s = 0; s < n_steps; ++s) {
        const float *v = model_outputs + s * numel;
        const float sig = sg[s];
        /* history shift: m1 <- m0, m0 <- converted */
        float *tmp = m1;
        m1 = m0;
        m0 = tmp;
        for (size_t i = 0; i < numel; ++i) m0[i] = x[i] - sig * v[i];
        if (hist < 2) hist++;
        const int last = (s == n_steps - 1);
        const float sigma_t = 1.0f * sg[s + 1];
        const float alpha_t = 1.0f - sg[s + 1];
        if (lower < 1 || last) {
            const float sigma_s = sg[s];
            const float h = lambda_of(sigma_t) - lambda_of(sigma_s);
            const float a = sigma_t / sigma_s;
            const float bcoef = -alpha_t * (expf(-h) - 1.0f);
            for (size_t i = 0; i < numel; ++i) x[i] = a * x[i] + bcoef * m0[i];
        } else {
            const float sigma_s0 = sg[s], sigma_s1 = sg[s - 1];
            const float lt = lambda_of(sigma_t), l0 = lambda_of(sigma_s0), l1 = lambda_of(sigma_s1);
            const float h = lt - l0, h0 = l0 - l1;
            const float r0 = h0 / h;
            const float a = sigma_t / sigma_s0;
            const float bcoef = -alpha_t * (expf(-h) - 1.0f);
            const float ccoef = -0.5f * alpha_t * (expf(-h) - 1.0f);
            for (size_t i = 0; i < numel; ++i) {
                const float d1 = (1.0f / r0) * (m0[i] - m1[i]);
                x[i] = a * x[i] + bcoef * m0[i] + ccoef * d1;
            }
        }
        if (lower < 2) lower++;
        memcpy(samples_out + s * numel, x, numel * sizeof(float));
    }
    free(ts);
    free(sg);
    free(x);
    free(m0);
    free(m1);
    return 0;
}

/* ------------------------------------------------------------------------------------
 * Model.
 * ---------------------------------------------------------------------------------- */
typedef struct {
    float *table;                    /* [6, C] */
    float *attn_gamma, *attn_beta;   /* [C] */
    float *wq, *wk, *wv, *wo;        /* [C, C] (in, out) */
    float *bq, *bk, *bv, *bo;        /* [C] */
    float *cwq, *cwk, *cwv, *cwo;    /* [C, C] */
    float *cbq, *cbk, *cbv, *cbo;    /* [C] */
    float *mlp_gamma, *mlp_beta;     /* [C] */
    float *w_inv, *b_inv;            /* [E, C], [E] */
    float *w_dw, *b_dw;              /* [E, 9], [E] */
    float *w_pt;                     /* [C, E/2] */
    /* optional RMSNorm of the cross-attention q and k projections (not in the reference) */
    int cqk_norm;                    /* 0 = off (the reference) */
    float cqk_eps;
    float *cq_norm, *ck_norm;        /* [C] weights, NULL = ones */
} orc_block;

typedef struct {
    size_t n_blocks, C, Cl, Din, E, self_heads, cross_heads;
    float *cap_w1, *cap_b1, *cap_w2, *cap_b2; /* [Din, C], [C], [C, C], [C] */
    float *patch_w, *patch_b;                 /* [C, Cl], [C] */
    float *te_w1, *te_b1, *te_w2, *te_b2;     /* [256, C], [C], [C, C], [C] */
    float *tp_w, *tp_b;                       /* [C, 6C], [6C] */
    float *cap_norm;                          /* [C] */
    float *final_table;                       /* [2, C] */
    float *out_w, *out_b;                     /* [C, Cl], [Cl] */
    orc_block *blocks;
} orc_model;

static float *copy_new(const float *src, size_t n) {
    float *d = (float *)malloc(n * sizeof(float));
    memcpy(d, src, n * sizeof(float));
    return d;
}

static float *fill_new(size_t n, float v) {
    float *d = (float *)malloc(n * sizeof(float));
    for (size_t i = 0; i < n; ++i) d[i] = v;
    return d;
}

/* Mirrors load_block_weights / load_denoiser_weights (transformer.cpp:200-399, 453-488). */
void *orc_model_create(const float *const *t, size_t n_blocks, size_t C, size_t Cl, size_t Din,
                       size_t E, size_t self_heads, size_t cross_heads) {
    if (n_blocks == 0 || C == 0 || self_heads == 0 || cross_heads == 0 || C % self_heads ||
        C % cross_heads || E % 2) {
        fail(1, "invalid model dimensions");
        return NULL;
    }
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->n_blocks = n_blocks;
    m->C = C;
    m->Cl = Cl;
    m->Din = Din;
    m->E = E;
    m->self_heads = self_heads;
    m->cross_heads = cross_heads;
    m->cap_w1 = transpose_new(t[0], C, Din);
    m->cap_b1 = copy_new(t[1], C);
    m->cap_w2 = transpose_new(t[2], C, C);
    m->cap_b2 = copy_new(t[3], C);
    m->patch_w = copy_new(t[4], C * Cl);
    m->patch_b = copy_new(t[5], C);
    m->te_w1 = transpose_new(t[6], C, 256);
    m->te_b1 = copy_new(t[7], C);
    m->te_w2 = transpose_new(t[8], C, C);
    m->te_b2 = copy_new(t[9], C);
    m->tp_w = transpose_new(t[10], 6 * C, C);
    m->tp_b = copy_new(t[11], 6 * C);
    m->cap_norm = copy_new(t[12], C);
    m->final_table = copy_new(t[13], 2 * C);
    m->out_w = transpose_new(t[14], Cl, C);
    m->out_b = copy_new(t[15], Cl);
    m->blocks = (orc_block *)calloc(n_blocks, sizeof(orc_block));
    for (size_t i = 0; i < n_blocks; ++i) {
        const float *const *b = t + 16 + 19 * i;
        orc_block *k = &m->blocks[i];
        k->table = copy_new(b[0], 6 * C);
        k->attn_gamma = fill_new(C, 1.0f);
        k->attn_beta = fill_new(C, 0.0f);
        k->wq = transpose_new(b[1], C, C);
        k->wk = transpose_new(b[2], C, C);
        k->wv = transpose_new(b[3], C, C);
        k->wo = transpose_new(b[4], C, C);
        k->bq = fill_new(C, 0.0f);
        k->bk = fill_new(C, 0.0f);
        k->bv = fill_new(C, 0.0f);
        k->bo = copy_new(b[5], C);
        k->cwq = transpose_new(b[6], C, C);
        k->cbq = copy_new(b[7], C);
        k->cwk = transpose_new(b[8], C, C);
        k->cbk = copy_new(b[9], C);
        k->cwv = transpose_new(b[10], C, C);
        k->cbv = copy_new(b[11], C);
        k->cwo = transpose_new(b[12], C, C);
        k->cbo = copy_new(b[13], C);
        k->mlp_gamma = fill_new(C, 1.0f);
        k->mlp_beta = fill_new(C, 0.0f);
        k->w_inv = copy_new(b[14], E * C);
        k->b_inv = copy_new(b[15], E);
        k->w_dw = copy_new(b[16], E * 9);
        k->b_dw = copy_new(b[17], E);
        k->w_pt = copy_new(b[18], C * (E / 2));
    }
    return m;
}

void orc_model_destroy(void *mp) {
    orc_model *m = (orc_model *)mp;
    if (!m) return;
    float **fields[] = {&m->cap_w1, &m->cap_b1, &m->cap_w2, &m->cap_b2, &m->patch_w,
                        &m->patch_b, &m->te_w1, &m->te_b1, &m->te_w2, &m->te_b2,
                        &m->tp_w, &m->tp_b, &m->cap_norm, &m->final_table, &m->out_w,
                        &m->out_b};
    for (size_t i = 0; i < sizeof fields / sizeof fields[0]; ++i) free(*fields[i]);
    for (size_t i = 0; i < m->n_blocks; ++i) {
        orc_block *k = &m->blocks[i];
        float *bf[] = {k->table, k->attn_gamma, k->attn_beta, k->wq, k->wk, k->wv, k->wo,
                       k->bq, k->bk, k->bv, k->bo, k->cwq, k->cwk, k->cwv, k->cwo, k->cbq,
                       k->cbk, k->cbv, k->cbo, k->mlp_gamma, k->mlp_beta, k->w_inv, k->b_inv,
                       k->w_dw, k->b_dw, k->w_pt, k->cq_norm, k->ck_norm};
        for (size_t j = 0; j < sizeof bf / sizeof bf[0]; ++j) free(bf[j]);
    }
    free(m->blocks);
    free(m);
}

int orc_model_set_block_extras(void *mp, size_t block, const float *q_bias, const float *k_bias,
                               const float *v_bias, const float *attn_gamma,
                               const float *attn_beta, const float *mlp_gamma,
                               const float *mlp_beta) {
    orc_model *m = (orc_model *)mp;
    if (!m || block >= m->n_blocks) ORC_INVALID("block index out of range");
    orc_block *k = &m->blocks[block];
    const size_t C = m->C;
    if (q_bias) memcpy(k->bq, q_bias, C * sizeof(float));
    if (k_bias) memcpy(k->bk, k_bias, C * sizeof(float));
    if (v_bias) memcpy(k->bv, v_bias, C * sizeof(float));
    if (attn_gamma) memcpy(k->attn_gamma, attn_gamma, C * sizeof(float));
    if (attn_beta) memcpy(k->attn_beta, attn_beta, C * sizeof(float));
    if (mlp_gamma) memcpy(k->mlp_gamma, mlp_gamma, C * sizeof(float));
    if (mlp_beta) memcpy(k->mlp_beta, mlp_beta, C * sizeof(float));
    return 0;
}

/* Optional RMSNorm of the cross-attention query and key projections over all C channels of a
 * token (the form of rms_norm_3d_lastdim, tensor.cpp:276-316, with eps and weight given):
 * enable = 0 switches it off (the reference's block, the default). Weights NULL = ones. */
int orc_model_set_cross_qk_norm(void *mp, size_t block, int enable, const float *q_weight,
                                const float *k_weight, float eps) {
    orc_model *m = (orc_model *)mp;
    if (!m || block >= m->n_blocks) ORC_INVALID("block index out of range");
    orc_block *k = &m->blocks[block];
    const size_t C = m->C;
    free(k->cq_norm);
    free(k->ck_norm);
    k->cq_norm = k->ck_norm = NULL;
    k->cqk_norm = enable != 0;
    k->cqk_eps = eps;
    if (enable && q_weight) {
        k->cq_norm = (float *)malloc(C * sizeof(float));
        memcpy(k->cq_norm, q_weight, C * sizeof(float));
    }
    if (enable && k_weight) {
        k->ck_norm = (float *)malloc(C * sizeof(float));
        memcpy(k->ck_norm, k_weight, C * sizeof(float));
    }
    return 0;
}

/* tokens [S, T, C] -> grid [S, C, side, side] (tensor.cpp:382-421) and back (:427-456). */
static void tokens_to_grid(const float *x, size_t S, size_t T, size_t C, float *out) {
    for (size_t b = 0; b < S; ++b)
        for (size_t t = 0; t < T; ++t)
            for (size_t h = 0; h < C; ++h) out[(b * C + h) * T + t] = x[(b * T + t) * C + h];
}

static void grid_to_tokens(const float *x, size_t S, size_t C, size_t T, float *out) {
    for (size_t b = 0; b < S; ++b)
        for (size_t h = 0; h < C; ++h)
            for (size_t t = 0; t < T; ++t) out[(b * T + t) * C + h] = x[(b * C + h) * T + t];
}

static int infer_side(size_t T, size_t *side) {
    size_t s = (size_t)sqrt((double)T);
    if (s * s != T) return fail(1, "token count must form a square grid");
    *side = s;
    return 0;
}

/* block_forward (transformer.cpp:726-778) with compute_sana_block_modulation (:496-542). */
int orc_block_forward(void *mp, size_t block, const float *x, size_t S, size_t T, const float *ctx,
                      size_t L, const float *tmod, const float *bias, float *after_self,
                      float *after_cross, float *after_ff) {
    orc_model *m = (orc_model *)mp;
    if (!m || block >= m->n_blocks) ORC_INVALID("block index out of range");
    const orc_block *k = &m->blocks[block];
    const size_t C = m->C, E = m->E, half = E / 2, M = S * T;
    size_t side = 0;
    if (infer_side(T, &side)) return 1;
    const size_t Hs = m->self_heads, Ds = C / Hs, Hc = m->cross_heads, Dc = C / Hc;

    /* modulation: mod[b][part][h] = tmod[b, part*C + h] + table[part, h] */
    float *mod = (float *)malloc(S * 6 * C * sizeof(float));
    for (size_t b = 0; b < S; ++b)
        for (size_t i = 0; i < 6 * C; ++i) mod[b * 6 * C + i] = tmod[b * 6 * C + i] + k->table[i];
    float *shift_msa = (float *)malloc(S * C * sizeof(float)), *scale_msa = (float *)malloc(S * C * sizeof(float));
    float *shift_mlp = (float *)malloc(S * C * sizeof(float)), *scale_mlp = (float *)malloc(S * C * sizeof(float));
    for (size_t b = 0; b < S; ++b) {
        memcpy(shift_msa + b * C, mod + b * 6 * C + 0 * C, C * sizeof(float));
        memcpy(scale_msa + b * C, mod + b * 6 * C + 1 * C, C * sizeof(float));
        memcpy(shift_mlp + b * C, mod + b * 6 * C + 3 * C, C * sizeof(float));
        memcpy(scale_mlp + b * C, mod + b * 6 * C + 4 * C, C * sizeof(float));
    }

    float *a = (float *)malloc(M * C * sizeof(float));
    float *a2 = (float *)malloc(M * C * sizeof(float));
    float *qp = (float *)malloc(M * C * sizeof(float));
    float *kp = (float *)malloc(M * C * sizeof(float));
    float *vp = (float *)malloc(M * C * sizeof(float));
    float *qh = (float *)malloc(M * C * sizeof(float));
    float *kh = (float *)malloc(M * C * sizeof(float));
    float *vh = (float *)malloc(M * C * sizeof(float));
    float *res = (float *)malloc(M * C * sizeof(float));

    /* self attention (transformer.cpp:736-750; transformer_ops.cpp:545-570) */
    orc_layer_norm(x, S, T, C, 1e-6f, k->attn_gamma, k->attn_beta, a);
    orc_modulate(a, S, T, C, shift_msa, scale_msa, a2);
    gemm(a2, k->wq, k->bq, qp, M, C, C, 0);
    gemm(a2, k->wk, k->bk, kp, M, C, C, 0);
    gemm(a2, k->wv, k->bv, vp, M, C, C, 0);
    split_heads(qp, S, T, Hs, Ds, qh);
    split_heads(kp, S, T, Hs, Ds, kh);
    split_heads(vp, S, T, Hs, Ds, vh);
    orc_linear_attention(qh, kh, vh, S, Hs, T, T, Ds, qp);
    merge_heads(qp, S, Hs, T, Ds, kp);
    gemm(kp, k->wo, k->bo, vp, M, C, C, 0);
    for (size_t b = 0; b < S; ++b)
        for (size_t t = 0; t < T; ++t)
            for (size_t h = 0; h < C; ++h) {
                const size_t i = (b * T + t) * C + h;
                const float gated = vp[i] * mod[b * 6 * C + 2 * C + h];
                res[i] = x[i] + gated;
            }
    if (after_self) memcpy(after_self, res, M * C * sizeof(float));

    /* cross attention (transformer.cpp:751-762; transformer_ops.cpp:572-608) */
    {
        float *ck = (float *)malloc(S * L * C * sizeof(float));
        float *cv = (float *)malloc(S * L * C * sizeof(float));
        float *ckh = (float *)malloc(S * L * C * sizeof(float));
        float *cvh = (float *)malloc(S * L * C * sizeof(float));
        gemm(res, k->cwq, k->cbq, qp, M, C, C, 0);
        gemm(ctx, k->cwk, k->cbk, ck, S * L, C, C, 0);
        gemm(ctx, k->cwv, k->cbv, cv, S * L, C, C, 0);
        if (k->cqk_norm) {
            orc_rms_norm(qp, 1, M, C, k->cqk_eps, k->cq_norm, qp);
            orc_rms_norm(ck, 1, S * L, C, k->cqk_eps, k->ck_norm, ck);
        }
        split_heads(qp, S, T, Hc, Dc, qh);
        split_heads(ck, S, L, Hc, Dc, ckh);
        split_heads(cv, S, L, Hc, Dc, cvh);
        orc_attention(qh, ckh, cvh, S, Hc, T, L, Dc, bias, qp);
        merge_heads(qp, S, Hc, T, Dc, kp);
        gemm(kp, k->cwo, k->cbo, vp, M, C, C, 0);
        for (size_t i = 0; i < M * C; ++i) res[i] += vp[i];
        free(ck);
        free(cv);
        free(ckh);
        free(cvh);
    }
    if (after_cross) memcpy(after_cross, res, M * C * sizeof(float));

    /* mix-FFN (transformer.cpp:763-777) */
    {
        float *grid = (float *)malloc(M * C * sizeof(float));
        float *gout = (float *)malloc(M * C * sizeof(float));
        orc_layer_norm(res, S, T, C, 1e-6f, k->mlp_gamma, k->mlp_beta, a);
        orc_modulate(a, S, T, C, shift_mlp, scale_mlp, a2);
        tokens_to_grid(a2, S, T, C, grid);
        /* conv weights are [out, in]: glumb takes w_inv [E, C], w_pt [C, E/2] */
        orc_glumb_conv(grid, S, C, side, side, k->w_inv, k->b_inv, E, k->w_dw, k->b_dw, k->w_pt,
                       C, gout);
        grid_to_tokens(gout, S, C, T, a);
        for (size_t b = 0; b < S; ++b)
            for (size_t t = 0; t < T; ++t)
                for (size_t h = 0; h < C; ++h) {
                    const size_t i = (b * T + t) * C + h;
                    const float gated = a[i] * mod[b * 6 * C + 5 * C + h];
                    res[i] = res[i] + gated;
                }
        free(grid);
        free(gout);
    }
    (void)half;
    if (after_ff) memcpy(after_ff, res, M * C * sizeof(float));

    free(mod);
    free(shift_msa);
    free(scale_msa);
    free(shift_mlp);
    free(scale_mlp);
    free(a);
    free(a2);
    free(qp);
    free(kp);
    free(vp);
    free(qh);
    free(kh);
    free(vh);
    free(res);
    return 0;
}

/* run_model_blocks (transformer.cpp:544-568). */
int orc_run_model_blocks(void *mp, const float *x, size_t S, size_t T, const float *ctx, size_t L,
                         const float *tmod, const float *bias, size_t begin, size_t end,
                         float *out) {
    orc_model *m = (orc_model *)mp;
    if (!m || begin > end || end > m->n_blocks) ORC_INVALID("invalid model block range");
    const size_t n = S * T * m->C;
    float *cur = (float *)malloc(n * sizeof(float));
    float *nxt = (float *)malloc(n * sizeof(float));
    memcpy(cur, x, n * sizeof(float));
    for (size_t b = begin; b < end; ++b) {
        int rc = orc_block_forward(m, b, cur, S, T, ctx, L, tmod, bias, NULL, NULL, nxt);
        if (rc) {
            free(cur);
            free(nxt);
            return rc;
        }
        float *tmp = cur;
        cur = nxt;
        nxt = tmp;
    }
    memcpy(out, cur, n * sizeof(float));
    free(cur);
    free(nxt);
    return 0;
}

int orc_model_project_caption(void *mp, const float *enc, size_t S, size_t L, size_t Din,
                              float *out) {
    orc_model *m = (orc_model *)mp;
    if (Din != m->Din) ORC_INVALID("encoder width mismatch");
    return orc_project_caption(enc, S, L, Din, m->cap_w1, m->cap_b1, m->C, m->cap_w2, m->cap_b2,
                               m->cap_norm, out);
}

/* timestep_embedding_2d (transformer.cpp:77-122) and the t-embedding MLP and t_block
 * (transformer.cpp:638-656). */
int orc_time_embed(void *mp, const float *tvals, size_t S, float *emb_out, float *tmod_out) {
    orc_model *m = (orc_model *)mp;
    const size_t C = m->C, dim = 256, half = 128;
    float freq[128];
    const float log_scale = -logf(10000.0f) / (float)half;
    for (size_t i = 0; i < half; ++i) freq[i] = expf((float)i * log_scale);
    float *proj = (float *)malloc(S * dim * sizeof(float));
    for (size_t b = 0; b < S; ++b)
        for (size_t i = 0; i < half; ++i) {
            const float v = tvals[b] * freq[i];
            proj[b * dim + i] = cosf(v);
            proj[b * dim + half + i] = sinf(v);
        }
    float *h = (float *)malloc(S * C * sizeof(float));
    float *emb = (float *)malloc(S * C * sizeof(float));
    gemm(proj, m->te_w1, m->te_b1, h, S, dim, C, 0);
    silu_inplace(h, S * C);
    gemm(h, m->te_w2, m->te_b2, emb, S, C, C, 0);
    memcpy(h, emb, S * C * sizeof(float));
    silu_inplace(h, S * C);
    if (tmod_out) gemm(h, m->tp_w, m->tp_b, tmod_out, S, C, 6 * C, 0);
    if (emb_out) memcpy(emb_out, emb, S * C * sizeof(float));
    free(proj);
    free(h);
    free(emb);
    return 0;
}

/* Denoiser forward for S sequences at timestep t, no CFG (transformer.cpp:631-681). */
int orc_forward_nocfg(void *mp, const float *latents, size_t S, size_t H, size_t W, float t,
                      const float *ctx, size_t L, const float *bias, float *noise_pred) {
    orc_model *m = (orc_model *)mp;
    const size_t C = m->C, Cl = m->Cl, T = H * W;
    float *grid = (float *)malloc(S * C * T * sizeof(float));
    float *x = (float *)malloc(S * T * C * sizeof(float));
    float *y = (float *)malloc(S * T * C * sizeof(float));
    float *emb = (float *)malloc(S * C * sizeof(float));
    float *tmod = (float *)malloc(S * 6 * C * sizeof(float));
    float *tv = (float *)malloc(S * sizeof(float));
    for (size_t b = 0; b < S; ++b) tv[b] = t;
    orc_conv1x1(latents, S, Cl, H, W, m->patch_w, m->patch_b, C, grid);
    grid_to_tokens(grid, S, C, T, x);
    orc_time_embed(m, tv, S, emb, tmod);
    int rc = orc_run_model_blocks(m, x, S, T, ctx, L, tmod, bias, 0, m->n_blocks, y);
    if (rc == 0) {
        float *shift = (float *)malloc(S * C * sizeof(float));
        float *scale = (float *)malloc(S * C * sizeof(float));
        for (size_t b = 0; b < S; ++b)
            for (size_t h = 0; h < C; ++h) {
                shift[b * C + h] = emb[b * C + h] + m->final_table[h];
                scale[b * C + h] = emb[b * C + h] + m->final_table[C + h];
            }
        orc_layer_norm(y, S, T, C, 1e-6f, NULL, NULL, x);
        orc_modulate(x, S, T, C, shift, scale, y);
        float *proj = (float *)malloc(S * T * Cl * sizeof(float));
        gemm(y, m->out_w, m->out_b, proj, S * T, C, Cl, 0);
        tokens_to_grid(proj, S, T, Cl, noise_pred);
        free(proj);
        free(shift);
        free(scale);
    }
    free(grid);
    free(x);
    free(y);
    free(emb);
    free(tmod);
    free(tv);
    return rc;
}

/* run_full_denoising_loop_with_cfg (transformer.cpp:692-724) over
 * run_full_denoising_step_with_cfg (:604-690), stopping after run_steps. */
int orc_denoise(void *mp, const float *latents, size_t B, size_t H, size_t W, const float *enc,
                size_t L, size_t Din, const float *bias, float guidance, size_t num_steps,
                size_t run_steps, float *out, size_t *step_index_out) {
    orc_model *m = (orc_model *)mp;
    const size_t C = m->C, Cl = m->Cl, n = B * Cl * H * W;
    if (num_steps == 0) ORC_INVALID("num_inference_steps must be positive");
    if (run_steps > num_steps) run_steps = num_steps;
    float *ts = (float *)malloc(num_steps * sizeof(float));
    float *sg = (float *)malloc((num_steps + 1) * sizeof(float));
    orc_scheduler_schedule(num_steps, 3.0f, ts, sg);
    float *ctx = (float *)malloc(2 * B * L * C * sizeof(float));
    int rc = orc_model_project_caption(m, enc, 2 * B, L, Din, ctx);
    float *x = (float *)malloc(n * sizeof(float));
    float *pair = (float *)malloc(2 * n * sizeof(float));
    float *noise = (float *)malloc(2 * n * sizeof(float));
    float *guided = (float *)malloc(n * sizeof(float));
    memcpy(x, latents, n * sizeof(float));
    /* Scheduler history needs all guided outputs; run the scheduler step by step. */
    size_t lower = 0;
    float *m0 = (float *)malloc(n * sizeof(float));
    float *m1 = (float *)malloc(n * sizeof(float));
    for (size_t s = 0; rc == 0 && s < run_steps; ++s) {
        memcpy(pair, x, n * sizeof(float));
        memcpy(pair + n, x, n * sizeof(float));
        rc = orc_forward_nocfg(m, pair, 2 * B, H, W, ts[s], ctx, L, bias, noise);
        if (rc) break;
        orc_cfg(noise, B, Cl, H, W, guidance, guided);
        /* step_sana_scheduler (scheduler.cpp:272-318), as in orc_scheduler_run */
        float *tmp = m1;
        m1 = m0;
        m0 = tmp;
        for (size_t i = 0; i < n; ++i) m0[i] = x[i] - sg[s] * guided[i];
        const int last = (s == num_steps - 1);
        const float sigma_t = sg[s + 1], alpha_t = 1.0f - sg[s + 1];
        if (lower < 1 || last) {
            const float h = lambda_of(sigma_t) - lambda_of(sg[s]);
            const float a = sigma_t / sg[s], bc = -alpha_t * (expf(-h) - 1.0f);
            for (size_t i = 0; i < n; ++i) x[i] = a * x[i] + bc * m0[i];
        } else {
            const float lt = lambda_of(sigma_t), l0 = lambda_of(sg[s]), l1 = lambda_of(sg[s - 1]);
            const float h = lt - l0, h0 = l0 - l1, r0 = h0 / h;
            const float a = sigma_t / sg[s], bc = -alpha_t * (expf(-h) - 1.0f);
            const float cc = -0.5f * alpha_t * (expf(-h) - 1.0f);
            for (size_t i = 0; i < n; ++i) {
                const float d1 = (1.0f / r0) * (m0[i] - m1[i]);
                x[i] = a * x[i] + bc * m0[i] + cc * d1;
            }
        }
        if (lower < 2) lower++;
    }
    if (rc == 0) {
        memcpy(out, x, n * sizeof(float));
        if (step_index_out) *step_index_out = run_steps;
    }
    free(ts);
    free(sg);
    free(ctx);
    free(x);
    free(pair);
    free(noise);
    free(guided);
    free(m0);
    free(m1);
    return rc;
}

/* attention_block_3d (transformer_ops.cpp:545-570): q/k/v projections, head split,
 * linear attention, merge, output projection. Weights [in, out]; biases may be NULL. */
int orc_attention_block(const float *x, size_t B, size_t T, size_t C, const float *wq,
                        const float *bq, const float *wk, const float *bk, const float *wv,
                        const float *bv, const float *wo, const float *bo, size_t heads,
                        float *out) {
    if (heads == 0 || C % heads) ORC_INVALID("hidden size must be divisible by num_heads");
    const size_t M = B * T, D = C / heads;
    float *p[5];
    for (int i = 0; i < 5; ++i) p[i] = (float *)malloc(M * C * sizeof(float));
    float *qh = (float *)malloc(M * C * sizeof(float));
    gemm(x, wq, bq, p[0], M, C, C, 0);
    gemm(x, wk, bk, p[1], M, C, C, 0);
    gemm(x, wv, bv, p[2], M, C, C, 0);
    split_heads(p[0], B, T, heads, D, qh);
    split_heads(p[1], B, T, heads, D, p[3]);
    split_heads(p[2], B, T, heads, D, p[4]);
    orc_linear_attention(qh, p[3], p[4], B, heads, T, T, D, p[0]);
    merge_heads(p[0], B, heads, T, D, p[1]);
    gemm(p[1], wo, bo, out, M, C, C, 0);
    for (int i = 0; i < 5; ++i) free(p[i]);
    free(qh);
    return 0;
}

/* cross_attention_block_3d (transformer_ops.cpp:572-608): q from x, k/v from ctx,
 * masked softmax attention, output projection. */
int orc_cross_attention_block(const float *x, size_t B, size_t T, size_t C, const float *ctx,
                              size_t L, const float *bias, const float *wq, const float *bq,
                              const float *wk, const float *bk, const float *wv, const float *bv,
                              const float *wo, const float *bo, size_t heads, float *out) {
    if (heads == 0 || C % heads) ORC_INVALID("hidden size must be divisible by num_heads");
    const size_t M = B * T, D = C / heads;
    float *q = (float *)malloc(M * C * sizeof(float)), *qh = (float *)malloc(M * C * sizeof(float));
    float *k = (float *)malloc(B * L * C * sizeof(float)), *kh = (float *)malloc(B * L * C * sizeof(float));
    float *v = (float *)malloc(B * L * C * sizeof(float)), *vh = (float *)malloc(B * L * C * sizeof(float));
    gemm(x, wq, bq, q, M, C, C, 0);
    gemm(ctx, wk, bk, k, B * L, C, C, 0);
    gemm(ctx, wv, bv, v, B * L, C, C, 0);
    split_heads(q, B, T, heads, D, qh);
    split_heads(k, B, L, heads, D, kh);
    split_heads(v, B, L, heads, D, vh);
    orc_attention(qh, kh, vh, B, heads, T, L, D, bias, q);
    merge_heads(q, B, heads, T, D, qh);
    gemm(qh, wo, bo, out, M, C, C, 0);
    free(q); free(qh); free(k); free(kh); free(v); free(vh);
    return 0;
}

/* sigma_to_alpha_sigma_t (scheduler.cpp:71-77) and compute_lambda (:79-81). */
static void alpha_sigma_of(const orc_sched_config *c, float sigma, float *alpha, float *sig) {
    if (c->use_flow_sigmas) {
        *alpha = 1.0f - sigma;
        *sig = sigma;
    } else {
        *alpha = 1.0f / sqrtf(sigma * sigma + 1.0f);
        *sig = sigma * *alpha;
    }
}

/* init_sana_scheduler_state (scheduler.cpp:143-153, built by :89-141 with the config's
 * num_train_timesteps), then step_sana_scheduler (:272-318) n_steps times: convert (:155-173),
 * history push capped at solver_order, order 1 when solver_order is 1, before the first
 * completed step or at the final step with lower_order_final / zero final sigma, else the
 * second-order update (:207-270, midpoint or heun coefficient). */
int orc_scheduler_run_config(const orc_sched_config *c, size_t n_steps, const float *sigmas_in,
                             const float *model_outputs, const float *sample, size_t numel,
                             float *timesteps_out, float *sigmas_out, float *samples_out) {
    if (c->solver_order <= 0) ORC_INVALID("solver_order must be positive");
    if (c->solver_order > 2) ORC_INVALID("only solver_order <= 2 is supported");
    if (n_steps == 0) ORC_INVALID("num_inference_steps must be positive");
    float *sg = sigmas_out;
    if (sigmas_in) {
        memcpy(sg, sigmas_in, (n_steps + 1) * sizeof(float));
        for (size_t i = 0; i < n_steps; ++i) timesteps_out[i] = 0.0f;
    } else {
        if (!c->use_flow_sigmas) ORC_INVALID("only use_flow_sigmas=true is supported");
        if (!c->final_sigmas_zero) ORC_INVALID("only zero final_sigmas_type is supported");
        if (c->num_train_timesteps <= 0) ORC_INVALID("num_train_timesteps must be positive");
        const float denom = (float)c->num_train_timesteps;
        for (size_t i = 0; i <= n_steps; ++i) {
            const float alpha = 1.0f + (1.0f / denom - 1.0f) * ((float)i / (float)n_steps);
            const float sigma = 1.0f - alpha;
            const float shifted = c->flow_shift * sigma / (1.0f + (c->flow_shift - 1.0f) * sigma);
            if (i > 0) {
                sg[n_steps - i] = shifted;
                timesteps_out[n_steps - i] = (float)(int)(shifted * denom);
            }
        }
        sg[n_steps] = 0.0f;
    }
    float *x = (float *)malloc(numel * sizeof(float));
    float *m0 = (float *)malloc(numel * sizeof(float));
    float *m1 = (float *)malloc(numel * sizeof(float));
    memcpy(x, sample, numel * sizeof(float));
    size_t hist = 0, lower = 0;
    int rc = 0;
    for (size_t s = 0; s < n_steps; ++s) {
        const float *v = model_outputs + s * numel;
        float *tmp = m1;
        m1 = m0;
        m0 = tmp;
        for (size_t i = 0; i < numel; ++i) m0[i] = x[i] - sg[s] * v[i];
        hist = hist + 1 < (size_t)c->solver_order ? hist + 1 : (size_t)c->solver_order;
        const int lower_final = (s == n_steps - 1) && (c->lower_order_final || c->final_sigmas_zero);
        float at, st, a0, s0;
        alpha_sigma_of(c, sg[s + 1], &at, &st);
        alpha_sigma_of(c, sg[s], &a0, &s0);
        const float lt = logf(at) - logf(st), l0 = logf(a0) - logf(s0);
        const float h = lt - l0;
        const float a = st / s0;
        const float bcoef = -at * (expf(-h) - 1.0f);
        if (c->solver_order == 1 || lower < 1 || lower_final) {
            for (size_t i = 0; i < numel; ++i) x[i] = a * x[i] + bcoef * m0[i];
        } else {
            if (s == 0) {
                rc = fail(1, "second-order update requires at least one previous step");
                break;
            }
            if (hist < 2) {
                rc = fail(1, "second-order update requires two model outputs");
                break;
            }
            float a1, s1;
            alpha_sigma_of(c, sg[s - 1], &a1, &s1);
            const float h0 = l0 - (logf(a1) - logf(s1));
            const float r0 = h0 / h;
            const float ccoef = c->solver_heun ? at * ((expf(-h) - 1.0f) / h + 1.0f)
                                               : -0.5f * at * (expf(-h) - 1.0f);
            for (size_t i = 0; i < numel; ++i) {
                const float d1 = (1.0f / r0) * (m0[i] - m1[i]);
                x[i] = a * x[i] + bcoef * m0[i] + ccoef * d1;
            }
        }
        if (lower < (size_t)c->solver_order) lower++;
        memcpy(samples_out + s * numel, x, numel * sizeof(float));
    }
    free(x);
    free(m0);
    free(m1);
    return rc;
}

/* convert_sana_scheduler_model_output (scheduler.cpp:155-173): x0 = sample - sigma_s v. */
int orc_scheduler_convert(const float *sigmas, size_t n_sigmas, size_t step_index,
                          const float *model_output, const float *sample, size_t numel,
                          float *out) {
    if (n_sigmas < 2 || step_index >= n_sigmas - 1) ORC_INVALID("scheduler step_index is out of range");
    const float sig = sigmas[step_index];
    for (size_t i = 0; i < numel; ++i) out[i] = sample[i] - sig * model_output[i];
    return 0;
}

/* First-order (scheduler.cpp:175-205) or midpoint second-order (:207-260) update. */
int orc_scheduler_update(int order, const float *sigmas, size_t n_sigmas, size_t step_index,
                         const float *m0, const float *m1, const float *sample, size_t numel,
                         float *out) {
    if (n_sigmas < 2 || step_index >= n_sigmas - 1) ORC_INVALID("scheduler step_index is out of range");
    const float sigma_t = sigmas[step_index + 1], alpha_t = 1.0f - sigmas[step_index + 1];
    if (order == 1) {
        const float h = lambda_of(sigma_t) - lambda_of(sigmas[step_index]);
        const float a = sigma_t / sigmas[step_index], bc = -alpha_t * (expf(-h) - 1.0f);
        for (size_t i = 0; i < numel; ++i) out[i] = a * sample[i] + bc * m0[i];
        return 0;
    }
    if (step_index == 0) ORC_INVALID("second-order update requires at least one previous step");
    const float lt = lambda_of(sigma_t), l0 = lambda_of(sigmas[step_index]);
    const float l1 = lambda_of(sigmas[step_index - 1]);
    const float h = lt - l0, h0 = l0 - l1, r0 = h0 / h;
    const float a = sigma_t / sigmas[step_index], bc = -alpha_t * (expf(-h) - 1.0f);
    const float cc = -0.5f * alpha_t * (expf(-h) - 1.0f);
    for (size_t i = 0; i < numel; ++i) {
        const float d1 = (1.0f / r0) * (m0[i] - m1[i]);
        out[i] = a * sample[i] + bc * m0[i] + cc * d1;
    }
    return 0;
}

/* step_sana_scheduler (scheduler.cpp:272-318) with an explicit state. */
int orc_scheduler_step(const float *sigmas, size_t n_sigmas, size_t step_index, size_t lower,
                       const float *hist, size_t n_hist, const float *model_output,
                       const float *sample, size_t numel, float *out, float *hist_out,
                       size_t *n_hist_out, size_t *lower_out) {
    if (n_sigmas < 2 || step_index >= n_sigmas - 1) ORC_INVALID("scheduler step_index is out of range");
    const size_t n_steps = n_sigmas - 1;
    float *conv = (float *)malloc(numel * sizeof(float));
    orc_scheduler_convert(sigmas, n_sigmas, step_index, model_output, sample, numel, conv);
    /* history: append, keep the newest two */
    size_t nh = 0;
    if (n_hist >= 1) {
        memcpy(hist_out, hist + (n_hist - 1) * numel, numel * sizeof(float));
        nh = 1;
    }
    memcpy(hist_out + nh * numel, conv, numel * sizeof(float));
    nh += 1;
    const int last = (step_index == n_steps - 1);
    int rc;
    if (lower < 1 || last) {
        rc = orc_scheduler_update(1, sigmas, n_sigmas, step_index, conv, NULL, sample, numel, out);
    } else {
        if (nh < 2) {
            free(conv);
            ORC_INVALID("second-order update requires two model outputs");
        }
        rc = orc_scheduler_update(2, sigmas, n_sigmas, step_index, hist_out + numel, hist_out,
                                  sample, numel, out);
    }
    *n_hist_out = nh;
    *lower_out = lower < 2 ? lower + 1 : lower;
    free(conv);
    return rc;
}

/* ------------------------------------------------------------------------------------
 * Text-encoder output contract (gemma_encoder.cpp), the conditioning the denoiser reads.
 * ---------------------------------------------------------------------------------- */

/* select_rows_first_and_last (gemma_encoder.cpp:51-77): row 0, then the last keep-1 rows. */
int orc_select_rows_first_and_last(const float *in, size_t rows, size_t cols, size_t keep, float *out) {
    if (keep == 0 || keep > rows) ORC_INVALID("select_rows_first_and_last: keep must be in (0, rows]");
    memcpy(out, in, cols * sizeof(float));
    const size_t tail = keep - 1;
    memcpy(out + cols, in + (rows - tail) * cols, tail * cols * sizeof(float));
    return 0;
}

/* write_attention_bias (gemma_encoder.cpp:177-184): 0 on real tokens, (1 - 0) * -10000 after. */
static void orc_attention_bias_row(float *row, size_t real, size_t n) {
    for (size_t t = 0; t < n; ++t) {
        const float mask = t < real ? 1.0f : 0.0f;
        row[t] = (1.0f - mask) * -10000.0f;
    }
}

/* The tail of encode_prompt_pair (gemma_encoder.cpp:188-244), after the encoder ran:
 * negative [max_seq, hidden] padded straight to max_seq with negative_real real tokens;
 * positive [positive_rows, hidden] (instruction prefix + prompt, padded to positive_rows
 * with positive_real real tokens) sliced to row 0 plus its last max_seq-1 rows. Output:
 * embeddings [2, max_seq, hidden] negative first, bias [2, 1, max_seq]. The real-token
 * count after the slice counts row 0 and every kept tail row below positive_real
 * (gemma_encoder.cpp:205-215). */
int orc_prompt_pair_assemble(const float *negative, size_t negative_rows, size_t negative_real,
                             const float *positive, size_t positive_rows, size_t positive_real,
                             size_t hidden, size_t max_sequence_length, float *embeddings, float *bias) {
    const size_t L = max_sequence_length;
    if (negative_rows != L) ORC_INVALID("negative branch must be padded to max_sequence_length");
    if (negative_real > negative_rows || positive_real > positive_rows)
        ORC_INVALID("tokenized text exceeds padded_length; truncation not implemented");
    memcpy(embeddings, negative, L * hidden * sizeof(float));
    const int rc = orc_select_rows_first_and_last(positive, positive_rows, hidden, L, embeddings + L * hidden);
    if (rc) return rc;
    size_t kept_real = positive_real > 0 ? 1 : 0;
    for (size_t pos = positive_rows - (L - 1); pos < positive_rows; ++pos)
        if (pos < positive_real) ++kept_real;
    orc_attention_bias_row(bias, negative_real, L);
    orc_attention_bias_row(bias + L, kept_real, L);
    return 0;
}

/* ------------------------------------------------------------------------------------
 * VAE decoder (vae.cpp, vae_ops.cpp), NCHW fp32.
 * ---------------------------------------------------------------------------------- */

/* conv2d_same for odd k (vae_ops.cpp:203-231, :18-75): zero padding k/2,
 * out[b,o,y,x] = bias[o] + sum_{c,ky,kx} w[o,c,ky,kx] x[b,c,y+ky-k/2,x+kx-k/2]. */
static void vae_conv_same(const float *x, size_t B, size_t Cin, size_t H, size_t W, const float *w, size_t Cout,
                          size_t k, const float *bias, float *out) {
    const size_t S = H * W;
    const long r = (long)k / 2;
    const long long BO = (long long)(B * Cout);
#pragma omp parallel for schedule(dynamic, 1) if (BO * (long long)(Cin * S * k * k) > 65536)
    for (long long bo = 0; bo < BO; ++bo) {
        const size_t b = (size_t)bo / Cout, oc = (size_t)bo % Cout;
        float *o = out + (b * Cout + oc) * S;
        for (size_t s = 0; s < S; ++s) o[s] = bias ? bias[oc] : 0.0f;
        for (size_t c = 0; c < Cin; ++c) {
            const float *xi = x + (b * Cin + c) * S;
            for (size_t ky = 0; ky < k; ++ky) {
                for (size_t kx = 0; kx < k; ++kx) {
                    const float wv = w[((oc * Cin + c) * k + ky) * k + kx];
                    const long dy = (long)ky - r, dx = (long)kx - r;
                    for (size_t y = 0; y < H; ++y) {
                        const long iy = (long)y + dy;
                        if (iy < 0 || iy >= (long)H) continue;
                        const long x0 = dx < 0 ? -dx : 0, x1 = dx > 0 ? (long)W - dx : (long)W;
                        float *orow = o + y * W;
                        const float *irow = xi + (size_t)iy * W;
                        for (long xx = x0; xx < x1; ++xx) orow[xx] += wv * irow[xx + dx];
                    }
                }
            }
        }
    }
}

/* depthwise_conv2d_same (vae_ops.cpp:233-258, common_ops.cpp:484-505,658-731): taps summed
 * ky-major then kx, bias last. */
static void vae_depthwise(const float *x, size_t B, size_t C, size_t H, size_t W, const float *w, size_t k,
                          const float *bias, float *out) {
    const long r = (long)k / 2;
    const long long P = (long long)(B * C);
#pragma omp parallel for schedule(static) if (P * (long long)(H * W * k * k) > 65536)
    for (long long p = 0; p < P; ++p) {
        const size_t c = (size_t)p % C;
        const float *xi = x + (size_t)p * H * W;
        float *o = out + (size_t)p * H * W;
        for (size_t y = 0; y < H; ++y) {
            for (size_t xx = 0; xx < W; ++xx) {
                float sum = 0.0f;
                for (size_t ky = 0; ky < k; ++ky) {
                    for (size_t kx = 0; kx < k; ++kx) {
                        const long iy = (long)y + (long)ky - r, ix = (long)xx + (long)kx - r;
                        if (iy >= 0 && iy < (long)H && ix >= 0 && ix < (long)W)
                            sum += xi[(size_t)iy * W + (size_t)ix] * w[(c * k + ky) * k + kx];
                    }
                }
                if (bias) sum += bias[c];
                o[y * W + xx] = sum;
            }
        }
    }
}

/* grouped_conv2d_1x1 (vae_ops.cpp:267-326): group g maps its in_per_group input channels to
 * its out_per_group output channels. */
static void vae_grouped_1x1(const float *x, size_t B, size_t Cin, size_t S, const float *w, size_t Cout,
                            size_t groups, float *out) {
    const size_t ipg = Cin / groups, opg = Cout / groups;
    const long long BO = (long long)(B * Cout);
#pragma omp parallel for schedule(static) if (BO * (long long)(ipg * S) > 65536)
    for (long long bo = 0; bo < BO; ++bo) {
        const size_t b = (size_t)bo / Cout, oc = (size_t)bo % Cout, g = oc / opg;
        float *o = out + (b * Cout + oc) * S;
        for (size_t s = 0; s < S; ++s) o[s] = 0.0f;
        for (size_t i = 0; i < ipg; ++i) {
            const float wv = w[oc * ipg + i];
            const float *xi = x + (b * Cin + g * ipg + i) * S;
            for (size_t s = 0; s < S; ++s) o[s] += wv * xi[s];
        }
    }
}

/* rms_norm_4d_channelwise (vae_ops.cpp:495-575): per pixel over channels, fma-accumulated
 * squares in channel order, inv = 1 / sqrt(mean + eps), out = x * inv * w (+ b). */
static void vae_rms_channelwise(const float *x, size_t B, size_t C, size_t S, const float *w, const float *bias,
                                float eps, float *out) {
    float *inv = (float *)malloc(S * sizeof(float));
    for (size_t b = 0; b < B; ++b) {
        const float *xb = x + b * C * S;
        float *ob = out + b * C * S;
        for (size_t s = 0; s < S; ++s) inv[s] = 0.0f;
        for (size_t c = 0; c < C; ++c)
            for (size_t s = 0; s < S; ++s) inv[s] = fmaf(xb[c * S + s], xb[c * S + s], inv[s]);
        const float inv_c = 1.0f / (float)C;
        for (size_t s = 0; s < S; ++s) inv[s] = 1.0f / sqrtf(inv[s] * inv_c + eps);
        for (size_t c = 0; c < C; ++c) {
            for (size_t s = 0; s < S; ++s) {
                float v = xb[c * S + s] * inv[s] * w[c];
                if (bias) v += bias[c];
                ob[c * S + s] = v;
            }
        }
    }
    free(inv);
}

/* run_vae_res_block (vae_ops.cpp:587-603). */
static void vae_res_block(float *x, size_t B, size_t C, size_t H, size_t W, const float *const *t) {
    const size_t n = B * C * H * W;
    float *h = (float *)malloc(n * sizeof(float));
    float *g = (float *)malloc(n * sizeof(float));
    vae_conv_same(x, B, C, H, W, t[0], C, 3, t[1], h);
    silu_inplace(h, n);
    vae_conv_same(h, B, C, H, W, t[2], C, 3, NULL, g);
    vae_rms_channelwise(g, B, C, H * W, t[3], t[4], 1e-5f, h);
    for (size_t i = 0; i < n; ++i) x[i] = h[i] + x[i];
    free(h);
    free(g);
}

/* run_vae_multiscale_attention (vae_ops.cpp:630-808), head dim d: q, k, v 1x1 projections
 * concatenated [q | k | v] per image, a depthwise k x k and grouped 1x1 multiscale branch,
 * then per merged head g (the first 3*inner/(3d) from qkv, the rest from the branch) the
 * channels [g*3d, g*3d + 3d) of its source read as q, k, v: ReLU linear attention
 * out = (V [K;1]^T)-weighted q / (z . q + 1e-15), to_out 1x1, RMSNorm(+bias), residual. */
static void vae_attention(float *x, size_t B, size_t C, size_t H, size_t W, size_t d, size_t kms,
                          const float *const *t) {
    const size_t S = H * W, inner = C, heads = inner / d, C3 = 3 * inner;
    float *qkv = (float *)malloc(B * C3 * S * sizeof(float));
    float *tmp = (float *)malloc(B * C3 * S * sizeof(float));
    float *ms = (float *)malloc(B * C3 * S * sizeof(float));
    float *merged = (float *)malloc(B * 2 * inner * S * sizeof(float));
    for (size_t b = 0; b < B; ++b) {
        for (int j = 0; j < 3; ++j)
            orc_conv1x1(x + b * C * S, 1, C, H, W, t[j], NULL, inner, qkv + (b * C3 + (size_t)j * inner) * S);
    }
    vae_depthwise(qkv, B, C3, H, W, t[3], kms, NULL, tmp);
    vae_grouped_1x1(tmp, B, C3, S, t[4], C3, 3 * heads, ms);
    const long long BG = (long long)(B * 2 * heads);
#pragma omp parallel for schedule(dynamic, 1)
    for (long long bg = 0; bg < BG; ++bg) {
        const size_t b = (size_t)bg / (2 * heads), g = (size_t)bg % (2 * heads);
        const float *src = (g < heads ? qkv : ms) + b * C3 * S + (g % heads) * 3 * d * S;
        const float *q = src, *k = src + d * S, *v = src + 2 * d * S;
        float *sc = (float *)malloc((d + 1) * d * sizeof(float));
        for (size_t i = 0; i <= d; ++i) {
            for (size_t j = 0; j < d; ++j) {
                float acc = 0.0f;
                for (size_t s = 0; s < S; ++s) {
                    const float kv = k[j * S + s] > 0.0f ? k[j * S + s] : 0.0f;
                    acc += (i < d ? v[i * S + s] : 1.0f) * kv;
                }
                sc[i * d + j] = acc;
            }
        }
        float *o = merged + (b * 2 * heads + g) * d * S;
        for (size_t s = 0; s < S; ++s) {
            float den = 0.0f;
            for (size_t j = 0; j < d; ++j) den += sc[d * d + j] * (q[j * S + s] > 0.0f ? q[j * S + s] : 0.0f);
            den += 1e-15f;
            for (size_t i = 0; i < d; ++i) {
                float acc = 0.0f;
                for (size_t j = 0; j < d; ++j) acc += sc[i * d + j] * (q[j * S + s] > 0.0f ? q[j * S + s] : 0.0f);
                o[i * S + s] = acc / den;
            }
        }
        free(sc);
    }
    float *h = tmp;
    orc_conv1x1(merged, B, 2 * inner, H, W, t[5], NULL, C, h);
    vae_rms_channelwise(h, B, C, S, t[6], t[7], 1e-5f, ms);
    for (size_t i = 0; i < B * C * S; ++i) x[i] = ms[i] + x[i];
    free(qkv);
    free(tmp);
    free(ms);
    free(merged);
}

/* run_vae_glumb_conv (vae_ops.cpp:605-628): glumb_conv, RMSNorm(+bias), residual. */
static void vae_glumb(float *x, size_t B, size_t C, size_t H, size_t W, const float *const *t) {
    const size_t n = B * C * H * W;
    float *h = (float *)malloc(n * sizeof(float));
    float *g = (float *)malloc(n * sizeof(float));
    orc_glumb_conv(x, B, C, H, W, t[0], t[1], 8 * C, t[2], t[3], t[4], C, h);
    vae_rms_channelwise(h, B, C, H * W, t[5], t[6], 1e-5f, g);
    for (size_t i = 0; i < n; ++i) x[i] = g[i] + x[i];
    free(h);
    free(g);
}

/* run_vae_upsample_block with shortcut (vae_ops.cpp:810-821, :338-453): nearest 2x, conv,
 * then up[b,oc,2y+i,2x+j] += x[b, (4 oc + 2i + j) / repeats, y, x], repeats = 4 Cout / Cin. */
static float *vae_upsample(const float *x, size_t B, size_t Cin, size_t H, size_t W, const float *w,
                           const float *bias, size_t Cout) {
    const size_t H2 = 2 * H, W2 = 2 * W;
    float *up = (float *)malloc(B * Cin * H2 * W2 * sizeof(float));
    for (size_t p = 0; p < B * Cin; ++p)
        for (size_t y = 0; y < H2; ++y)
            for (size_t xx = 0; xx < W2; ++xx) up[(p * H2 + y) * W2 + xx] = x[(p * H + y / 2) * W + xx / 2];
    float *out = (float *)malloc(B * Cout * H2 * W2 * sizeof(float));
    vae_conv_same(up, B, Cin, H2, W2, w, Cout, 3, bias, out);
    free(up);
    const size_t rep = 4 * Cout / Cin;
    for (size_t b = 0; b < B; ++b)
        for (size_t oc = 0; oc < Cout; ++oc)
            for (size_t y = 0; y < H; ++y)
                for (size_t xx = 0; xx < W; ++xx)
                    for (size_t ij = 0; ij < 4; ++ij) {
                        const size_t ic = (oc * 4 + ij) / rep;
                        out[((b * Cout + oc) * H2 + 2 * y + ij / 2) * W2 + 2 * xx + ij % 2] +=
                            x[((b * Cin + ic) * H + y) * W + xx];
                    }
    return out;
}

static size_t vae_block_tensors(const orc_vae_block *b) {
    return (b->has_upsample ? 2u : 0u) + (size_t)b->layers * (b->is_res_block ? 5u : 15u);
}

size_t orc_vae_tensor_count(const orc_vae_dims *d) {
    size_t n = 6;
    for (int i = 0; i < d->n_blocks; ++i) n += vae_block_tensors(&d->blocks[i]);
    return n;
}

int orc_vae_decode(const orc_vae_dims *d, const float *const *t, const float *latents, size_t B, size_t h,
                   size_t w, float *out) {
    if (d->n_blocks < 1 || d->n_blocks > 8) ORC_INVALID("vae decoder must contain at least one up block");
    if (!(d->scaling_factor > 0.0f)) ORC_INVALID("vae scaling_factor must be positive");
    const int n = d->n_blocks;
    size_t first[9];
    first[0] = 6;
    for (int i = 0; i < n; ++i) first[i + 1] = first[i] + vae_block_tensors(&d->blocks[i]);
    const size_t Cl = (size_t)d->latent_channels;
    size_t C = (size_t)d->blocks[n - 1].channels, H = h, W = w;
    if (C % Cl != 0) ORC_INVALID("vae decoder conv_in output channels must be divisible by latent channels");
    /* conv_in on latents / scaling_factor, plus the repeated-channel shortcut (vae.cpp:210-241) */
    const size_t nl = B * Cl * H * W;
    float *scaled = (float *)malloc(nl * sizeof(float));
    const float inv_sf = 1.0f / d->scaling_factor;
    for (size_t i = 0; i < nl; ++i) scaled[i] = latents[i] * inv_sf;
    float *x = (float *)malloc(B * C * H * W * sizeof(float));
    vae_conv_same(scaled, B, Cl, H, W, t[0], C, 3, t[1], x);
    const size_t rep = C / Cl;
    for (size_t b = 0; b < B; ++b)
        for (size_t c = 0; c < C; ++c)
            for (size_t s = 0; s < H * W; ++s) x[(b * C + c) * H * W + s] += scaled[(b * Cl + c / rep) * H * W + s];
    free(scaled);
    for (int i = n - 1; i >= 0; --i) {
        const orc_vae_block *blk = &d->blocks[i];
        const float *const *bt = t + first[i];
        if (blk->has_upsample) {
            float *up = vae_upsample(x, B, C, H, W, bt[0], bt[1], (size_t)blk->channels);
            free(x);
            x = up;
            C = (size_t)blk->channels;
            H *= 2;
            W *= 2;
            bt += 2;
        }
        if (C != (size_t)blk->channels) ORC_INVALID("vae up block channels must match its input");
        for (int l = 0; l < blk->layers; ++l) {
            if (blk->is_res_block) {
                vae_res_block(x, B, C, H, W, bt);
                bt += 5;
            } else {
                vae_attention(x, B, C, H, W, (size_t)d->head_dim, (size_t)d->ms_kernel, bt);
                vae_glumb(x, B, C, H, W, bt + 8);
                bt += 15;
            }
        }
    }
    /* norm_out (+bias), ReLU, conv_out (vae.cpp:313-324) */
    float *y = (float *)malloc(B * C * H * W * sizeof(float));
    vae_rms_channelwise(x, B, C, H * W, t[2], t[3], 1e-5f, y);
    for (size_t i = 0; i < B * C * H * W; ++i) y[i] = y[i] > 0.0f ? y[i] : 0.0f;
    vae_conv_same(y, B, C, H, W, t[4], (size_t)d->out_channels, 3, t[5], out);
    free(x);
    free(y);
    return 0;
}
