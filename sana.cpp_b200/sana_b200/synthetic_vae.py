"""Seeded synthetic weights for the DC-AE VAE decoder the reference runs after the denoiser
(vae.h:11-73, vae.cpp:91-170): a random initialisation of the architecture, listed in the
order the C ABI's VAE upload, the oracle and the reference wrapper take them, with the
reference's GGUF tensor names (``decoder.up_blocks.<i>.<layer>....``).

Defaults are DC-AE f32c32 as Sana uses it: latent 32 channels, up blocks of
(128, 256, 512, 512, 1024, 1024) channels, three ResBlocks in the first three and three
attention + GLUMBConv layers in the last three, every block but the innermost starting with
a nearest-2x upsample conv, attention head dim 32 with a 5x5 multiscale branch, RGB out,
scaling factor 0.41407 (infer_main.cpp:369-374).

Values come from the same torch-compatible generator as the denoiser's weights: tensor j
uses seed ``base_seed * 1000 + j``; conv and linear weights N(0, 1) * 0.02, biases
N(0, 1) * 0.02, norm weights 1 + N(0, 1) * 0.1, norm biases N(0, 1) * 0.1.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Callable, List, Sequence, Tuple

import numpy as np

F = np.float32
RandnFn = Callable[[int, int], np.ndarray]


@dataclass(frozen=True)
class VaeDims:
    latent_channels: int = 32
    out_channels: int = 3
    channels: Tuple[int, ...] = (128, 256, 512, 512, 1024, 1024)
    res_blocks: Tuple[bool, ...] = (True, True, True, False, False, False)
    layers: Tuple[int, ...] = (3, 3, 3, 3, 3, 3)
    head_dim: int = 32
    ms_kernel: int = 5
    scaling_factor: float = 0.41407

    @property
    def n_blocks(self) -> int:
        return len(self.channels)

    def has_upsample(self, i: int) -> bool:
        return i < self.n_blocks - 1

    def upscale(self) -> int:
        return 2 ** (self.n_blocks - 1)


class VaeBlockStruct(ctypes.Structure):
    _fields_ = [("channels", ctypes.c_int), ("has_upsample", ctypes.c_int), ("is_res_block", ctypes.c_int),
                ("layers", ctypes.c_int)]


class VaeDimsStruct(ctypes.Structure):
    """The C layout shared by sana_vae_dims (include/sana_cuda.h), orc_vae_dims and ref_vae_dims."""
    _fields_ = [("latent_channels", ctypes.c_int), ("out_channels", ctypes.c_int), ("n_blocks", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("ms_kernel", ctypes.c_int), ("scaling_factor", ctypes.c_float),
                ("blocks", VaeBlockStruct * 8)]


def dims_struct(d: VaeDims) -> VaeDimsStruct:
    s = VaeDimsStruct(d.latent_channels, d.out_channels, d.n_blocks, d.head_dim, d.ms_kernel, d.scaling_factor)
    for i in range(d.n_blocks):
        s.blocks[i] = VaeBlockStruct(d.channels[i], int(d.has_upsample(i)), int(d.res_blocks[i]), d.layers[i])
    return s


RES_TENSORS = (("conv1.weight", "conv3"), ("conv1.bias", "bias"), ("conv2.weight", "conv3"),
               ("norm.weight", "norm_w"), ("norm.bias", "norm_b"))
ATTN_TENSORS = (("attn.to_q.weight", "lin"), ("attn.to_k.weight", "lin"), ("attn.to_v.weight", "lin"),
                ("attn.to_qkv_multiscale.0.proj_in.weight", "ms_in"),
                ("attn.to_qkv_multiscale.0.proj_out.weight", "ms_out"), ("attn.to_out.weight", "out"),
                ("attn.norm_out.weight", "norm_w"), ("attn.norm_out.bias", "norm_b"),
                ("conv_out.conv_inverted.weight", "inv"), ("conv_out.conv_inverted.bias", "inv_b"),
                ("conv_out.conv_depth.weight", "dw"), ("conv_out.conv_depth.bias", "dw_b"),
                ("conv_out.conv_point.weight", "pt"), ("conv_out.norm.weight", "norm_w"),
                ("conv_out.norm.bias", "norm_b"))


def vae_tensor_specs(d: VaeDims) -> List[Tuple[str, Tuple[int, ...], str]]:
    """(GGUF name, PyTorch shape, kind) in upload order."""
    n, ch = d.n_blocks, d.channels
    specs = [("decoder.conv_in.weight", (ch[-1], d.latent_channels, 3, 3), "w"),
             ("decoder.conv_in.bias", (ch[-1],), "b"),
             ("decoder.norm_out.weight", (ch[0],), "norm_w"),
             ("decoder.norm_out.bias", (ch[0],), "norm_b"),
             ("decoder.conv_out.weight", (d.out_channels, ch[0], 3, 3), "w"),
             ("decoder.conv_out.bias", (d.out_channels,), "b")]
    for i in range(n):
        c = ch[i]
        pre = f"decoder.up_blocks.{i}"
        base = 0
        if d.has_upsample(i):
            specs += [(f"{pre}.0.conv.weight", (c, ch[i + 1], 3, 3), "w"), (f"{pre}.0.conv.bias", (c,), "b")]
            base = 1
        for layer in range(base, base + d.layers[i]):
            lp = f"{pre}.{layer}"
            if d.res_blocks[i]:
                shapes = {"conv3": (c, c, 3, 3), "bias": (c,), "norm_w": (c,), "norm_b": (c,)}
                specs += [(f"{lp}.{nm}", shapes[k], "b" if k == "bias" else ("w" if k == "conv3" else k))
                          for nm, k in RES_TENSORS]
            else:
                shapes = {"lin": (c, c), "ms_in": (3 * c, 1, d.ms_kernel, d.ms_kernel),
                          "ms_out": (3 * c, d.head_dim, 1, 1), "out": (c, 2 * c), "norm_w": (c,), "norm_b": (c,),
                          "inv": (8 * c, c, 1, 1), "inv_b": (8 * c,), "dw": (8 * c, 1, 3, 3), "dw_b": (8 * c,),
                          "pt": (c, 4 * c, 1, 1)}
                kinds = {"inv_b": "b", "dw_b": "b", "norm_w": "norm_w", "norm_b": "norm_b"}
                specs += [(f"{lp}.{nm}", shapes[k], kinds.get(k, "w")) for nm, k in ATTN_TENSORS]
    return specs


def generate_vae(d: VaeDims, randn: RandnFn, base_seed: int = 0) -> List[np.ndarray]:
    out = []
    for j, (_, shape, kind) in enumerate(vae_tensor_specs(d)):
        n = int(np.prod(shape))
        r = randn(max(n, 16), base_seed * 1000 + j)[:n].astype(F)
        if kind == "norm_w":
            v = 1.0 + 0.1 * r
        elif kind == "norm_b":
            v = 0.1 * r
        else:
            v = 0.02 * r
        out.append(v.astype(F).reshape(shape))
    return out


def vae_flops(d: VaeDims, h: int, w: int) -> float:
    """Algorithmic FLOPs of one decode of a [1, latent, h, w] latent (2 per multiply-add):
    every convolution and projection, the multiscale depthwise and grouped convs and the
    linear attention; elementwise work not counted."""
    total = 0.0
    H, W = h, w
    n = d.n_blocks
    total += 2.0 * H * W * d.channels[-1] * d.latent_channels * 9
    for i in range(n - 1, -1, -1):
        c = d.channels[i]
        if d.has_upsample(i):
            H, W = 2 * H, 2 * W
            total += 2.0 * H * W * c * d.channels[i + 1] * 9
        P = H * W
        for _ in range(d.layers[i]):
            if d.res_blocks[i]:
                total += 2 * (2.0 * P * c * c * 9)
            else:
                heads = c // d.head_dim
                total += 2.0 * P * (3 * c) * c                       # q, k, v
                total += 2.0 * P * (3 * c) * d.ms_kernel ** 2         # depthwise
                total += 2.0 * P * (3 * c) * d.head_dim               # grouped 1x1
                total += 2 * heads * 2 * (2.0 * P * (d.head_dim + 1) * d.head_dim)  # attention, both branches
                total += 2.0 * P * c * 2 * c                          # to_out
                total += 2.0 * P * 8 * c * c + 2.0 * P * 8 * c * 9 + 2.0 * P * c * 4 * c  # GLUMBConv
    total += 2.0 * H * W * d.out_channels * d.channels[0] * 9
    return total


SMALL = VaeDims(latent_channels=8, out_channels=3, channels=(16, 32, 64), res_blocks=(True, True, False),
                layers=(1, 2, 2), head_dim=32, ms_kernel=5, scaling_factor=0.5)
