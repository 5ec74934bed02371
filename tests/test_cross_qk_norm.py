"""The optional RMSNorm of the cross-attention query and key projections (not in the
reference's block; off by default): the oracle's restatement against an independent float64
numpy computation of the cross-attention stage, and the CUDA path against the oracle (gpu)."""
import numpy as np
import pytest

from sana_b200 import synthetic as syn

D = syn.ModelDims(n_blocks=1, hidden=64, latent_channels=4, caption_dim=48, ff_expanded=160, self_heads=4,
                  cross_heads=2)


def _setup(randn, oracle, T=16, L=12, lens=(5, 12)):
    tensors = syn.generate_model(D, randn, base_seed=7, bias_std=0.05)
    m = oracle.model(tensors, *D.as_args())
    enc = syn.encoder_states(randn, 2, L, D.caption_dim, 3)
    bias = syn.attention_bias(list(lens), L)
    ctx = m.project_caption(enc)
    _, tmod = m.time_embed([700.0, 700.0])
    x = syn._draw(randn, 2 * T * D.hidden, 9).reshape(2, T, D.hidden)
    rng = np.random.default_rng(3)
    qw = (1.0 + 0.3 * rng.standard_normal(D.hidden)).astype(np.float32)
    kw = (1.0 + 0.3 * rng.standard_normal(D.hidden)).astype(np.float32)
    return tensors, m, x, ctx, tmod, bias, qw, kw


def _block(tensors, name):
    specs = syn.model_tensor_specs(D)
    return tensors[[s[0] for s in specs].index(f"transformer_blocks.0.{name}")].astype(np.float64)


def _rms(a, w, eps):
    return a / np.sqrt((a * a).mean(-1, keepdims=True) + eps) * w


def test_oracle_cross_qk_norm_matches_float64(oracle):
    from sana_b200 import randn_torch_cpu
    tensors, m, x, ctx, tmod, bias, qw, kw = _setup(randn_torch_cpu, oracle)
    eps = 1e-6
    after_self, cross_off, _ = m.block_forward(0, x, ctx, tmod, bias)
    m.set_cross_qk_norm(0, True, qw, kw, eps)
    _, cross_on, _ = m.block_forward(0, x, ctx, tmod, bias)
    # float64 restatement of the cross-attention stage from the same after_self
    xs, c = after_self.astype(np.float64), ctx.astype(np.float64)
    q = _rms(xs @ _block(tensors, "attn2.to_q.weight").T + _block(tensors, "attn2.to_q.bias"), qw, eps)
    k = _rms(c @ _block(tensors, "attn2.to_k.weight").T + _block(tensors, "attn2.to_k.bias"), kw, eps)
    v = c @ _block(tensors, "attn2.to_v.weight").T + _block(tensors, "attn2.to_v.bias")
    H, Dh = D.cross_heads, D.hidden // D.cross_heads
    S, T, L = xs.shape[0], xs.shape[1], c.shape[1]
    qh, kh, vh = (a.reshape(S, -1, H, Dh).transpose(0, 2, 1, 3) for a in (q, k, v))
    sc = qh @ kh.transpose(0, 1, 3, 2) / np.sqrt(Dh) + bias.astype(np.float64).reshape(S, 1, 1, L)
    p = np.exp(sc - sc.max(-1, keepdims=True))
    o = (p / p.sum(-1, keepdims=True)) @ vh
    o = o.transpose(0, 2, 1, 3).reshape(S, T, H * Dh)
    want = xs + o @ _block(tensors, "attn2.to_out.0.weight").T + _block(tensors, "attn2.to_out.0.bias")
    err = np.linalg.norm(cross_on - want) / np.linalg.norm(want - xs)
    assert err < 1e-5, err
    assert np.linalg.norm(cross_on - cross_off) / np.linalg.norm(cross_off - xs) > 1e-3  # the option acts
    m.set_cross_qk_norm(0, False)
    assert np.array_equal(m.block_forward(0, x, ctx, tmod, bias)[1], cross_off)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_cuda_cross_qk_norm_matches_oracle(oracle, mode):
    """Full-size block 0 (36 x 32 self heads, 16 x 72 cross heads) with the option on: per-stage
    relative L2 <= 1e-4 (fp32 check mode) / 1e-2 (bf16) against the oracle; switching it off
    restores the reference's block."""
    from sana_b200 import SANA_MODE_BF16, SANA_MODE_F32, SanaCuda, randn_torch_cpu
    d1 = syn.ModelDims(n_blocks=1)
    tensors = syn.generate_model(d1, randn_torch_cpu, base_seed=0, bias_std=0.02)
    m = oracle.model(tensors, *d1.as_args())
    enc = syn.encoder_states(randn_torch_cpu, 2, 300, d1.caption_dim, 7)
    bias = syn.attention_bias([8, 24], 300)
    ctx = m.project_caption(enc)
    _, tmod = m.time_embed([999.0, 999.0])
    x = syn._draw(randn_torch_cpu, 2 * 1024 * d1.hidden, 400).reshape(2, 1024, d1.hidden)
    rng = np.random.default_rng(5)
    qw = (1.0 + 0.3 * rng.standard_normal(d1.hidden)).astype(np.float32)
    kw = (1.0 + 0.3 * rng.standard_normal(d1.hidden)).astype(np.float32)
    ref_off = m.block_forward(0, x, ctx, tmod, bias)
    m.set_cross_qk_norm(0, True, qw, kw, 1e-6)
    ref = m.block_forward(0, x, ctx, tmod, bias)
    g = SanaCuda(0, SANA_MODE_F32 if mode == "f32" else SANA_MODE_BF16)
    g.upload_checkpoint(d1.as_args(), tensors)
    g.set_cross_qk_norm(True, [qw], [kw], 1e-6)
    got = g.block_forward(0, x, ctx, tmod, bias)
    tol = 1e-4 if mode == "f32" else 1e-2

    def rel(a, b):
        return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))
    for a, b in zip(got, ref):
        assert rel(a, b) < tol
    assert rel(got[1] - got[0], ref[1] - ref[0]) < 10 * tol  # the cross-attention branch itself
    g.set_cross_qk_norm(False)
    off = g.block_forward(0, x, ctx, tmod, bias)
    assert rel(off[1], ref_off[1]) < tol
    g.close()
