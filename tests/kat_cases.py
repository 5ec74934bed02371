"""Known-answer tests of the reference, restated once and run against every implementation.

Inputs and expected values are the ones asserted in the reference's own unit tests
(cconthekeyboard/sana.cpp ``tests/test_tensor.cpp``, ``tests/test_transformer.cpp``,
``tests/test_scheduler_main.cpp``); each case cites the lines it comes from and keeps the
reference's tolerance. An implementation is any object with the methods of
``oracle/oracle.py``'s checkers (``layer_norm``, ``attention`` ...); the CPU oracle, the
compiled reference and the CUDA path (through the C ABI) all run the same cases.

A case returns a list of ``(label, got, expected, tol)``; ``tol=0`` means exact.
"""
from __future__ import annotations

import numpy as np

F = np.float32


def _a(x):
    return np.asarray(x, dtype=F)


def kat_layer_norm(impl):
    # test_tensor.cpp:92-115
    x = _a([[[1, 3], [2, 4]]])
    plain = impl.layer_norm(x, 0.0)
    affine = impl.layer_norm(x, 0.0, _a([2, 3]), _a([1, -1]))
    return [("layer_norm", plain, _a([[[-1, 1], [-1, 1]]]), 0.0),
            ("layer_norm_affine", affine, _a([[[-1, 2], [-1, 2]]]), 0.0)]


def kat_rms_norm(impl):
    # test_tensor.cpp:117-130
    out = impl.rms_norm(_a([[[3, 4], [0, 5]]]), 0.0, _a([2, 3]))
    return [("rms_norm", out, _a([[[1.6970563, 3.3941126], [0.0, 4.2426405]]]), 1e-5)]


def kat_modulate(impl):
    # test_tensor.cpp:132-148
    out = impl.modulate(_a([[[1, 2], [3, 4]]]), _a([[10, 20]]), _a([[0.5, -0.5]]))
    return [("modulate", out, _a([[[11.5, 21.0], [14.5, 22.0]]]), 0.0)]


def _conv_input():
    # test_tensor.cpp:183-190 (and 217-224 for the depthwise test)
    return _a([[[[1, 2], [3, 4]], [[10, 20], [30, 40]]]])


def kat_conv1x1(impl):
    # test_tensor.cpp:180-211
    w = _a([[1, 0], [0, 1], [1, 1]]).reshape(3, 2, 1, 1)
    out = impl.conv1x1(_conv_input(), w, _a([0, 0, -1]))
    exp = _a([[[[1, 2], [3, 4]], [[10, 20], [30, 40]], [[10, 21], [32, 43]]]])
    return [("conv1x1", out, exp, 0.0)]


def kat_depthwise3x3(impl):
    # test_tensor.cpp:214-242
    w = np.zeros((2, 1, 3, 3), F)
    w[0, 0, 1, 1] = 1.0
    w[1, 0, 1, 1] = 2.0
    out = impl.depthwise3x3(_conv_input(), w, _a([0.5, -1.0]))
    exp = _a([[[[1.5, 2.5], [3.5, 4.5]], [[19, 39], [59, 79]]]])
    return [("depthwise3x3", out, exp, 0.0)]


def _silu(x):
    x = F(x)
    return F(x / (F(1) + np.exp(-x, dtype=F)))


def _glumb_weights():
    # test_tensor.cpp:273-304 (the same weights drive the block test, test_transformer.cpp:380-404)
    w_inv = np.zeros((4, 2, 1, 1), F)
    w_inv[0, 0] = w_inv[1, 1] = w_inv[2, 0] = w_inv[3, 1] = 1.0
    w_dw = np.zeros((4, 1, 3, 3), F)
    w_dw[:, 0, 1, 1] = 1.0
    w_pt = np.zeros((2, 2, 1, 1), F)
    w_pt[0, 0] = w_pt[1, 1] = 1.0
    return w_inv, np.zeros(4, F), w_dw, np.zeros(4, F), w_pt


def kat_glumb_conv(impl):
    # test_tensor.cpp:273-313
    w_inv, b_inv, w_dw, b_dw, w_pt = _glumb_weights()
    out = impl.glumb_conv(_a([[[[1.0]], [[2.0]]]]), w_inv, b_inv, w_dw, b_dw, w_pt)
    s1, s2 = _silu(1.0), _silu(2.0)
    exp = _a([[[[s1 * _silu(s1)]], [[s2 * _silu(s2)]]]])
    return [("glumb_conv", out, exp, 1e-6)]


def kat_linear(impl):
    # test_transformer.cpp:123-146 (linear_3d_lastdim)
    x = _a([[[1, 2, 3], [4, 5, 6]]])
    w = _a([[7, 8], [9, 10], [11, 12]])
    out = impl.linear_3d(x, w, _a([1, -2]))
    return [("linear_3d", out, _a([[[59, 62], [140, 152]]]), 0.0)]


def _qkv():
    # test_transformer.cpp:180-210
    q = _a([[[[1, 0], [0, 1]]]])
    k = _a([[[[1, 2], [3, 4]]]])
    v = _a([[[[10, 20], [30, 40]]]])
    return q, k, v


def kat_attention(impl):
    # test_transformer.cpp:229-234
    q, k, v = _qkv()
    out = impl.attention(q, k, v)
    exp = _a([[[[26.088594, 36.088594], [26.088594, 36.088594]]]])
    return [("attention_4d", out, exp, 1e-5)]


def kat_linear_attention(impl):
    # test_transformer.cpp:236-241
    q, k, v = _qkv()
    out = impl.linear_attention(q, k, v)
    exp = _a([[[[25.0, 35.0], [23.333334, 33.333332]]]])
    return [("linear_attention_4d", out, exp, 1e-5)]


def kat_project_caption(impl):
    # test_transformer.cpp:243-280
    enc = _a([[[1, 2, 3, 4], [5, 6, 7, 8]]])
    w1 = np.zeros((4, 2), F)
    w1[0, 0] = w1[1, 1] = 1.0
    w2 = np.eye(2, dtype=F)
    out = impl.project_caption(enc, w1, np.zeros(2, F), w2, np.zeros(2, F), _a([1, 2]))
    exp = _a([[[0.5590534, 2.5980382], [0.9053573, 2.1728575]]])
    return [("project_caption_context", out, exp, 1e-5)]


def _eye_block():
    # test_transformer.cpp:310-330
    x = _a([[[1, 0], [0, 1]]])
    w = np.eye(2, dtype=F)
    b = np.zeros(2, F)
    return x, w, b


def kat_attention_block(impl):
    # test_transformer.cpp:332-344
    x, w, b = _eye_block()
    out = impl.attention_block(x, w, b, w, b, w, b, w, b, 1)
    return [("attention_block_3d", out, _a([[[1, 0], [0, 1]]]), 1e-5)]


def kat_cross_attention_block(impl):
    # test_transformer.cpp:346-371
    x, w, b = _eye_block()
    ctx = _a([[[2, 0], [0, 3]]])
    out = impl.cross_attention_block(x, ctx, None, w, b, w, b, w, b, w, b, 1)
    exp = _a([[[1.6088594, 0.5867110], [0.2140836, 2.6788745]]])
    return [("cross_attention_block_3d", out, exp, 1e-5)]


def block_kat_inputs(residual_only: bool):
    """The tiny one-token block of test_transformer.cpp:373-484 as a PyTorch-layout
    tensor list (see sana_b200.synthetic for the order) plus its inputs: hidden 2,
    one head each, identity (or zero, for the residual-only case) projections, the
    GLUMB weights above, zero scale_shift_table, gates 1 from the timestep vector."""
    C = 2
    w_inv, b_inv, w_dw, b_dw, w_pt = _glumb_weights()
    proj = np.zeros((C, C), F) if residual_only else np.eye(C, dtype=F)
    zb = np.zeros(C, F)
    model = [np.zeros((C, 4), F), zb, np.eye(C, dtype=F), zb,          # caption (unused)
             np.zeros((C, 1, 1, 1), F), zb,                              # patch embed (unused)
             np.zeros((C, 256), F), zb, np.zeros((C, C), F), zb,         # t-embedding (unused)
             np.zeros((6 * C, C), F), np.zeros(6 * C, F),                # t_block (unused)
             np.ones(C, F), np.zeros((2, C), F),                          # caption norm, final table
             np.zeros((1, C), F), np.zeros(1, F)]                         # proj_out (unused)
    block = [np.zeros((6, C), F), proj, proj, proj, proj, zb,
             proj, zb, proj, zb, proj, zb, proj, zb,
             w_inv, b_inv, w_dw, b_dw, w_pt]
    x = _a([[[1, 0]]])
    ctx = _a([[[2, 0], [0, 3]]])
    tmod = np.zeros((1, 12), F)
    tmod[0, [4, 5, 10, 11]] = 1.0
    return model + block, x, ctx, tmod


def kat_block_forward(impl):
    # test_transformer.cpp:373-440 and 442-484
    res = []
    for residual_only, exp in ((False, [4.3467007, -0.9475632]), (True, [1.3607715, 0.0313307])):
        tensors, x, ctx, tmod = block_kat_inputs(residual_only)
        m = impl.model(tensors, 1, 2, 1, 4, 4, 1, 1)
        out = m.block_forward(0, x, ctx, tmod)[2]
        res.append(("block_forward" + ("_residual_only" if residual_only else ""), out, _a([[exp]]), 1e-5))
    return res


def kat_scheduler(impl):
    # test_scheduler_main.cpp:27-41 (4-step schedule), 80-115 (convert, first and second order)
    ts, sg = impl.scheduler_schedule(4, 3.0)
    res = [("timesteps", ts, _a([999, 899, 749, 499]), 1e-3),
           ("sigmas", sg, _a([0.99966644, 0.89963979, 0.74962479, 0.49966654, 0.0]), 1e-6)]
    sig = _a([0.8, 0.5, 0.2, 0.0])
    conv = impl.scheduler_convert(sig, 0, _a([2.0]), _a([4.0]))
    res.append(("convert", conv, _a([2.4]), 1e-6))
    res.append(("first_order", impl.scheduler_update(1, sig, 0, conv, None, _a([4.0])), _a([3.4]), 1e-5))
    out, hist, lower = impl.scheduler_step(sig, 0, 0, [], _a([2.0]), _a([4.0]))
    res.append(("step", out, _a([3.4]), 1e-5))
    res.append(("step_history", np.concatenate(hist), _a([2.4]), 1e-6))
    res.append(("step_lower_count", _a([lower]), _a([1]), 0.0))
    sig2 = _a([0.8, 0.5, 0.2, 0.1, 0.09, 0.08, 0.07, 0.06, 0.05, 0.04, 0.03, 0.02, 0.015, 0.01, 0.005,
               0.001, 0.0])
    so = impl.scheduler_update(2, sig2, 1, _a([2.0]), _a([2.4]), _a([3.4]))
    res.append(("second_order", so, _a([2.44]), 1e-5))
    out2, hist2, lower2 = impl.scheduler_step(sig2, 1, 1, [_a([2.4]), _a([2.0])], _a([3.1]), _a([3.4]))
    res.append(("step2_history_len", _a([len(hist2)]), _a([2]), 0.0))
    res.append(("step2_lower_count", _a([lower2]), _a([2]), 0.0))
    return res


ALL_KATS = [kat_layer_norm, kat_rms_norm, kat_modulate, kat_conv1x1, kat_depthwise3x3, kat_glumb_conv,
            kat_linear, kat_attention, kat_linear_attention, kat_project_caption, kat_attention_block,
            kat_cross_attention_block, kat_block_forward, kat_scheduler]


def kat_select_rows_first_and_last(impl):
    # test_gemma_encoder.cpp:10-33: a 10x2 ramp; keep 4 -> rows 0, 7, 8, 9; keep 10 -> all; keep 1 -> row 0
    x = np.arange(20, dtype=F).reshape(10, 2)
    return [("keep4", impl.select_rows_first_and_last(x, 4), _a([[0, 1], [14, 15], [16, 17], [18, 19]]), 0.0),
            ("keep10", impl.select_rows_first_and_last(x, 10), x, 0.0),
            ("keep1", impl.select_rows_first_and_last(x, 1), _a([[0, 1]]), 0.0)]


def kat_prompt_pair(impl):
    # gemma_encoder.cpp:188-244 on a ramp: negative padded to L=4 with 2 real tokens; positive
    # padded to 7 rows with 5 real tokens -> rows 0, 4, 5, 6; real after the slice: row 0 and
    # row 4 -> bias (1 - mask) * -10000, -0.0 on real tokens
    neg = np.arange(8, dtype=F).reshape(4, 2)
    pos = 100 + np.arange(14, dtype=F).reshape(7, 2)
    emb, bias = impl.prompt_pair_assemble(neg, 2, pos, 5, 4)
    want = np.stack([neg, pos[[0, 4, 5, 6]]])
    wb = _a([[[-0.0, -0.0, -10000, -10000]], [[-0.0, -0.0, -10000, -10000]]])
    return [("embeddings", emb, want, 0.0), ("bias", bias, wb, 0.0),
            ("bias_sign", np.signbit(bias).astype(F), np.ones_like(wb), 0.0)]


# Host-side contract cases: the oracle and the library's host functions run them.
ENCODER_KATS = [kat_select_rows_first_and_last, kat_prompt_pair]


def check(results):
    """Asserts every (label, got, expected, tol) triple; tol 0 means bit-equal values."""
    for label, got, exp, tol in results:
        got = np.asarray(got, F)
        exp = np.asarray(exp, F)
        assert got.shape == exp.shape, f"{label}: shape {got.shape} != {exp.shape}"
        if tol == 0.0:
            assert np.array_equal(got, exp), f"{label}: {got.ravel()} != {exp.ravel()}"
        else:
            err = float(np.max(np.abs(got - exp)))
            assert err < tol, f"{label}: max|diff| {err} >= {tol}; got {got.ravel()} want {exp.ravel()}"
