"""Seeded synthetic inputs for the Sana-0.6B denoiser (no checkpoints or datasets here).

Weights are a random initialisation of the real architecture, listed in the order and
PyTorch layout that a checkpoint would hold them (``[out, in]`` linear weights, conv
weights ``[out, in, kh, kw]``). Values come from a torch-compatible CPU normal generator
(``torch.Generator().manual_seed(s)`` then ``torch.randn``), one seed per tensor:

* tensor ``j`` uses seed ``base_seed * 1000 + j``;
* linear/conv weights: N(0, 1) * 0.02; biases: 0 (or N(0, 1) * ``bias_std``);
* scale-shift tables: N(0, 1) / sqrt(hidden); ``caption_norm.weight``: ones.

Tensors with fewer than 16 elements take the first elements of a 16-element draw (the
torch CPU generator's block size).

The generator is injected (``randn(n, seed) -> float32[n]``) so the same spec can be
driven by the product's RNG (``sana_randn_torch_cpu`` in the C ABI), by the CPU oracle
or by the reference build; all three are bit-identical.

Model tensor list (16), per-block list (19): see ``model_tensor_specs``. The same order
is used by the C ABI's weight upload helper, the oracle and the reference wrapper.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, List, Sequence, Tuple

import numpy as np

F = np.float32
RandnFn = Callable[[int, int], np.ndarray]


@dataclass(frozen=True)
class ModelDims:
    """Architecture constants; defaults are Sana-0.6B (infer_main.cpp:366-367 heads)."""

    n_blocks: int = 28
    hidden: int = 1152
    latent_channels: int = 32
    caption_dim: int = 2304
    ff_expanded: int = 5760
    self_heads: int = 36
    cross_heads: int = 16

    def as_args(self):
        return (self.n_blocks, self.hidden, self.latent_channels, self.caption_dim, self.ff_expanded,
                self.self_heads, self.cross_heads)


MODEL_TENSORS = (
    ("caption_projection.linear_1.weight", "weight"),
    ("caption_projection.linear_1.bias", "bias"),
    ("caption_projection.linear_2.weight", "weight"),
    ("caption_projection.linear_2.bias", "bias"),
    ("patch_embed.proj.weight", "weight"),
    ("patch_embed.proj.bias", "bias"),
    ("time_embed.emb.timestep_embedder.linear_1.weight", "weight"),
    ("time_embed.emb.timestep_embedder.linear_1.bias", "bias"),
    ("time_embed.emb.timestep_embedder.linear_2.weight", "weight"),
    ("time_embed.emb.timestep_embedder.linear_2.bias", "bias"),
    ("time_embed.linear.weight", "weight"),
    ("time_embed.linear.bias", "bias"),
    ("caption_norm.weight", "ones"),
    ("scale_shift_table", "table"),
    ("proj_out.weight", "weight"),
    ("proj_out.bias", "bias"),
)

BLOCK_TENSORS = (
    ("scale_shift_table", "table"),
    ("attn1.to_q.weight", "weight"),
    ("attn1.to_k.weight", "weight"),
    ("attn1.to_v.weight", "weight"),
    ("attn1.to_out.0.weight", "weight"),
    ("attn1.to_out.0.bias", "bias"),
    ("attn2.to_q.weight", "weight"),
    ("attn2.to_q.bias", "bias"),
    ("attn2.to_k.weight", "weight"),
    ("attn2.to_k.bias", "bias"),
    ("attn2.to_v.weight", "weight"),
    ("attn2.to_v.bias", "bias"),
    ("attn2.to_out.0.weight", "weight"),
    ("attn2.to_out.0.bias", "bias"),
    ("ff.conv_inverted.weight", "weight"),
    ("ff.conv_inverted.bias", "bias"),
    ("ff.conv_depth.weight", "weight"),
    ("ff.conv_depth.bias", "bias"),
    ("ff.conv_point.weight", "weight"),
)


def model_tensor_specs(d: ModelDims) -> List[Tuple[str, Tuple[int, ...], str]]:
    C, Cl, Din, E = d.hidden, d.latent_channels, d.caption_dim, d.ff_expanded
    model_shapes = [(C, Din), (C,), (C, C), (C,), (C, Cl, 1, 1), (C,), (C, 256), (C,), (C, C), (C,),
                    (6 * C, C), (6 * C,), (C,), (2, C), (Cl, C), (Cl,)]
    block_shapes = [(6, C), (C, C), (C, C), (C, C), (C, C), (C,), (C, C), (C,), (C, C), (C,), (C, C), (C,),
                    (C, C), (C,), (E, C, 1, 1), (E,), (E, 1, 3, 3), (E,), (C, E // 2, 1, 1)]
    specs = [(n, s, k) for (n, k), s in zip(MODEL_TENSORS, model_shapes)]
    for i in range(d.n_blocks):
        specs += [(f"transformer_blocks.{i}.{n}", s, k) for (n, k), s in zip(BLOCK_TENSORS, block_shapes)]
    return specs


def _draw(randn: RandnFn, n: int, seed: int) -> np.ndarray:
    if n >= 16:
        return np.asarray(randn(n, seed), F)
    return np.asarray(randn(16, seed), F)[:n].copy()


def tensor_seed(base_seed: int, index: int) -> int:
    return base_seed * 1000 + index


def generate_tensor(spec, index: int, d: ModelDims, randn: RandnFn, base_seed: int = 0,
                    w_std: float = 0.02, bias_std: float = 0.0) -> np.ndarray:
    name, shape, kind = spec
    n = int(np.prod(shape))
    s = tensor_seed(base_seed, index)
    if kind == "ones":
        v = np.ones(n, F)
    elif kind == "bias" and bias_std == 0.0:
        v = np.zeros(n, F)
    else:
        scale = {"weight": w_std, "bias": bias_std, "table": 1.0 / math.sqrt(d.hidden)}[kind]
        v = _draw(randn, n, s) * F(scale)
    return v.reshape(shape)


def generate_model(d: ModelDims, randn: RandnFn, base_seed: int = 0, w_std: float = 0.02,
                   bias_std: float = 0.0) -> List[np.ndarray]:
    return [generate_tensor(sp, j, d, randn, base_seed, w_std, bias_std)
            for j, sp in enumerate(model_tensor_specs(d))]


def latents(randn: RandnFn, batch: int, channels: int, height: int, width: int, seed: int) -> np.ndarray:
    return _draw(randn, batch * channels * height * width, seed).reshape(batch, channels, height, width)


def encoder_states(randn: RandnFn, sequences: int, tokens: int, dim: int, seed: int) -> np.ndarray:
    return _draw(randn, sequences * tokens * dim, seed).reshape(sequences, tokens, dim)


def attention_bias(valid_lengths: Sequence[int], tokens: int) -> np.ndarray:
    """Additive caption mask [S, 1, L]: 0 for the first ``valid`` tokens, -10000 after
    (the encoder's contract, gemma_encoder.cpp:177-184)."""
    out = np.full((len(valid_lengths), 1, tokens), -10000.0, F)
    for i, v in enumerate(valid_lengths):
        out[i, 0, :v] = 0.0
    return out


def batch_valid_lengths(images: int, seed: int, lo: int = 8, hi: int = 120) -> List[int]:
    """Per-sequence valid caption lengths for a batch of images (uncond block first),
    uniform in [lo, hi] from a seeded numpy generator."""
    rng = np.random.default_rng(seed)
    return [int(v) for v in rng.integers(lo, hi + 1, size=2 * images)]
