// transformer_ops.h (cconthekeyboard/sana.cpp src/transformer_ops.h:5-50) over the C ABI.
// Shape checks and their std::invalid_argument follow transformer_ops.cpp:15-608.
#include "transformer_ops.h"

#include <stdexcept>

#include "shim.h"

using sana_shim::as_int;
using sana_shim::check;
using sana_shim::handle;
using sana_shim::opt;
using sana_shim::ptr;
using sana_shim::require;

namespace {
void require_linear(const Tensor& w, size_t in, const Tensor* b, const char* what) {
    require(w.rank() == 2 && w.dim_size(0) == in, what);
    if (b && b->numel()) require(b->numel() == w.dim_size(1), what);
}
}  // namespace

Tensor project_caption_context(const Tensor& encoder_hidden_states, const Tensor& linear_1_weight,
                               const Tensor* linear_1_bias, const Tensor& linear_2_weight, const Tensor* linear_2_bias,
                               const Tensor& norm_weight) {
    require(encoder_hidden_states.rank() == 3, "encoder_hidden_states must be rank 3");
    const size_t B = encoder_hidden_states.dim_size(0), L = encoder_hidden_states.dim_size(1);
    const size_t Din = encoder_hidden_states.dim_size(2);
    require_linear(linear_1_weight, Din, linear_1_bias, "linear_1 weight must be [in, hidden]");
    const size_t C = linear_1_weight.dim_size(1);
    require_linear(linear_2_weight, C, linear_2_bias, "linear_2 weight must be [hidden, hidden]");
    require(linear_2_weight.dim_size(1) == C && norm_weight.numel() == C, "norm weight must have hidden elements");
    Tensor out({B, L, C});
    if (out.numel() == 0) return out;
    check(sana_op_project_caption(handle(), ptr(encoder_hidden_states), as_int(B, "batch"), as_int(L, "tokens"),
                                  as_int(Din, "input dim"), ptr(linear_1_weight), opt(linear_1_bias),
                                  as_int(C, "hidden"), ptr(linear_2_weight), opt(linear_2_bias), ptr(norm_weight),
                                  out.data().data()));
    return out;
}

Tensor split_heads_3d(const Tensor& input, size_t num_heads) {
    require(input.rank() == 3, "input must be rank 3");
    require(num_heads != 0, "num_heads must be greater than 0");
    const size_t B = input.dim_size(0), T = input.dim_size(1), hidden = input.dim_size(2);
    require(hidden % num_heads == 0, "hidden size must be divisible by num_heads");
    Tensor out({B, num_heads, T, hidden / num_heads});
    if (out.numel() == 0) return out;
    check(sana_op_split_heads(handle(), ptr(input), as_int(B, "batch"), as_int(T, "tokens"), as_int(hidden, "hidden"),
                              as_int(num_heads, "heads"), out.data().data()));
    return out;
}

Tensor merge_heads_4d(const Tensor& input) {
    require(input.rank() == 4, "input must be rank 4");
    const size_t B = input.dim_size(0), H = input.dim_size(1), T = input.dim_size(2), D = input.dim_size(3);
    Tensor out({B, T, H * D});
    if (out.numel() == 0) return out;
    check(sana_op_merge_heads(handle(), ptr(input), as_int(B, "batch"), as_int(H, "heads"), as_int(T, "tokens"),
                              as_int(D, "head dim"), out.data().data()));
    return out;
}

Tensor attention_scores_4d(const Tensor& q, const Tensor& k) {
    require(q.rank() == 4, "q must be rank 4");
    require(k.rank() == 4, "k must be rank 4");
    require(q.dim_size(0) == k.dim_size(0) && q.dim_size(1) == k.dim_size(1) && q.dim_size(3) == k.dim_size(3),
            "q and k must agree in batch, heads and head_dim");
    const size_t B = q.dim_size(0), H = q.dim_size(1), Tq = q.dim_size(2), Tk = k.dim_size(2), D = q.dim_size(3);
    Tensor out({B, H, Tq, Tk});
    if (out.numel() == 0) return out;
    if (D == 0) return out;  // empty sums
    check(sana_op_attention_scores(handle(), ptr(q), ptr(k), as_int(B, "batch"), as_int(H, "heads"),
                                   as_int(Tq, "q tokens"), as_int(Tk, "k tokens"), as_int(D, "head dim"),
                                   out.data().data()));
    return out;
}

Tensor attention_values_4d(const Tensor& weights, const Tensor& v) {
    require(weights.rank() == 4, "weights must be rank 4");
    require(v.rank() == 4, "v must be rank 4");
    require(weights.dim_size(0) == v.dim_size(0) && weights.dim_size(1) == v.dim_size(1) &&
                weights.dim_size(3) == v.dim_size(2),
            "weights and v must agree in batch, heads and k_tokens");
    const size_t B = v.dim_size(0), H = v.dim_size(1), Tq = weights.dim_size(2), Tk = v.dim_size(2);
    const size_t D = v.dim_size(3);
    Tensor out({B, H, Tq, D});
    if (out.numel() == 0 || Tk == 0) return out;
    check(sana_op_attention_values(handle(), ptr(weights), ptr(v), as_int(B, "batch"), as_int(H, "heads"),
                                   as_int(Tq, "q tokens"), as_int(Tk, "k tokens"), as_int(D, "head dim"),
                                   out.data().data()));
    return out;
}

Tensor softmax_lastdim_4d(const Tensor& input) {
    require(input.rank() == 4, "input must be rank 4");
    Tensor out(input.shape());
    const size_t n = input.dim_size(3);
    if (out.numel() == 0) return out;
    check(sana_op_softmax_lastdim(handle(), ptr(input), static_cast<long long>(input.numel() / n), as_int(n, "width"),
                                  out.data().data()));
    return out;
}

Tensor attention_4d(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor* attention_bias) {
    require(q.rank() == 4 && k.rank() == 4 && v.rank() == 4, "q, k and v must be rank 4");
    require(q.dim_size(0) == k.dim_size(0) && q.dim_size(1) == k.dim_size(1) && q.dim_size(3) == k.dim_size(3),
            "q and k must agree in batch, heads and head_dim");
    require(k.same_shape(v), "k and v must have the same shape");
    const size_t B = q.dim_size(0), H = q.dim_size(1), Tq = q.dim_size(2), Tk = k.dim_size(2), D = q.dim_size(3);
    if (attention_bias)
        require(attention_bias->rank() == 3 && attention_bias->dim_size(0) == B && attention_bias->dim_size(1) == 1 &&
                    attention_bias->dim_size(2) == Tk,
                "attention_bias must have shape {batch, 1, k_tokens}");
    Tensor out(q.shape());
    if (out.numel() == 0) return out;
    check(sana_op_attention(handle(), ptr(q), ptr(k), ptr(v), as_int(B, "batch"), as_int(H, "heads"),
                            as_int(Tq, "q tokens"), as_int(Tk, "k tokens"), as_int(D, "head dim"), opt(attention_bias),
                            out.data().data()));
    return out;
}

Tensor linear_attention_4d(const Tensor& q, const Tensor& k, const Tensor& v) {
    require(q.rank() == 4 && k.rank() == 4 && v.rank() == 4, "q, k and v must be rank 4");
    require(k.same_shape(v), "k and v must have the same shape");
    require(q.dim_size(0) == k.dim_size(0) && q.dim_size(1) == k.dim_size(1) && q.dim_size(3) == k.dim_size(3),
            "q and k must agree in batch, heads and head_dim");
    const size_t B = q.dim_size(0), H = q.dim_size(1), Tq = q.dim_size(2), Tk = k.dim_size(2), D = q.dim_size(3);
    Tensor out(q.shape());
    if (out.numel() == 0) return out;
    check(sana_op_linear_attention(handle(), ptr(q), ptr(k), ptr(v), as_int(B, "batch"), as_int(H, "heads"),
                                   as_int(Tq, "q tokens"), as_int(Tk, "k tokens"), as_int(D, "head dim"),
                                   out.data().data()));
    return out;
}

Tensor attention_block_3d(const Tensor& input, const Tensor& q_weight, const Tensor* q_bias, const Tensor& k_weight,
                          const Tensor* k_bias, const Tensor& v_weight, const Tensor* v_bias, const Tensor& out_weight,
                          const Tensor* out_bias, size_t num_heads) {
    require(input.rank() == 3, "input must be rank 3");
    const size_t B = input.dim_size(0), T = input.dim_size(1), C = input.dim_size(2);
    for (const Tensor* w : {&q_weight, &k_weight, &v_weight, &out_weight})
        require(w->rank() == 2 && w->dim_size(0) == C && w->dim_size(1) == C, "projection weights must be [hidden, hidden]");
    require(num_heads != 0 && C % num_heads == 0, "hidden size must be divisible by num_heads");
    Tensor out(input.shape());
    if (out.numel() == 0) return out;
    check(sana_op_attention_block(handle(), ptr(input), as_int(B, "batch"), as_int(T, "tokens"), as_int(C, "hidden"),
                                  ptr(q_weight), opt(q_bias), ptr(k_weight), opt(k_bias), ptr(v_weight), opt(v_bias),
                                  ptr(out_weight), opt(out_bias), as_int(num_heads, "heads"), out.data().data()));
    return out;
}

Tensor cross_attention_block_3d(const Tensor& input, const Tensor& context, const Tensor* attention_bias,
                                const Tensor& q_weight, const Tensor* q_bias, const Tensor& k_weight,
                                const Tensor* k_bias, const Tensor& v_weight, const Tensor* v_bias,
                                const Tensor& out_weight, const Tensor* out_bias, size_t num_heads) {
    require(input.rank() == 3 && context.rank() == 3, "input and context must be rank 3");
    const size_t B = input.dim_size(0), T = input.dim_size(1), C = input.dim_size(2), L = context.dim_size(1);
    require(context.dim_size(0) == B && context.dim_size(2) == C, "context must be [batch, tokens, hidden]");
    for (const Tensor* w : {&q_weight, &k_weight, &v_weight, &out_weight})
        require(w->rank() == 2 && w->dim_size(0) == C && w->dim_size(1) == C, "projection weights must be [hidden, hidden]");
    require(num_heads != 0 && C % num_heads == 0, "hidden size must be divisible by num_heads");
    if (attention_bias) require(attention_bias->numel() == B * L, "attention_bias must have shape {batch, 1, k_tokens}");
    Tensor out(input.shape());
    if (out.numel() == 0) return out;
    check(sana_op_cross_attention_block(handle(), ptr(input), as_int(B, "batch"), as_int(T, "tokens"),
                                        as_int(C, "hidden"), ptr(context), as_int(L, "context tokens"),
                                        opt(attention_bias), ptr(q_weight), opt(q_bias), ptr(k_weight), opt(k_bias),
                                        ptr(v_weight), opt(v_bias), ptr(out_weight), opt(out_bias),
                                        as_int(num_heads, "heads"), out.data().data()));
    return out;
}
