"""Writes a denoiser checkpoint as the reference's three GGUF weight files.

sana.cpp's front end reads ``model_weights.gguf`` (the transformer blocks),
``caption_weights.gguf`` (the caption projection) and ``denoiser_weights.gguf`` (patch embed,
time embedding, t_block, caption norm, final table and projection) from its weights directory
(infer_main.cpp:347-365), every tensor fp32 under its diffusers name with linear weights in
PyTorch's [out, in] layout (load_linear_weight_tensor transposes them on load). This writes a
checkpoint list in ``sana_b200.synthetic`` order into that form with the ``gguf`` package, so
synthetic or converted weights can go through ``sana_cuda_upload_gguf`` as real ones would.

    python -m sana_b200.gguf_files DIR [--blocks 28] [--vae-channels 128,256,512,512,1024,1024]

writes a random-initialised weights directory of the Sana-0.6B architecture (the four GGUF
files and a stand-in file at the text encoder's path) that the reference's front ends read with
``--weights-dir DIR`` or from ``../weights``.
"""
from __future__ import annotations

import os
from typing import Sequence

import numpy as np

from .synthetic import BLOCK_TENSORS, MODEL_TENSORS

CAPTION_FIELDS = range(0, 4)   # MODEL_TENSORS entries of caption_weights.gguf
DENOISER_FIELDS = range(4, 16)  # ... of denoiser_weights.gguf


def _write(path: str, named: Sequence) -> None:
    import gguf
    w = gguf.GGUFWriter(path, arch="sana")
    for name, arr in named:
        w.add_tensor(name, np.ascontiguousarray(arr, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def write_checkpoint_gguf(tensors: Sequence[np.ndarray], n_blocks: int, directory: str,
                          block_prefix: str = "transformer_blocks") -> dict:
    """tensors: 16 model tensors then 19 per block (synthetic order). Returns the three paths."""
    os.makedirs(directory, exist_ok=True)
    paths = {k: os.path.join(directory, f"{k}_weights.gguf") for k in ("model", "caption", "denoiser")}
    _write(paths["caption"], [(MODEL_TENSORS[i][0], tensors[i]) for i in CAPTION_FIELDS])
    _write(paths["denoiser"], [(MODEL_TENSORS[i][0], tensors[i]) for i in DENOISER_FIELDS])
    blocks = []
    for b in range(n_blocks):
        for j, (suffix, _) in enumerate(BLOCK_TENSORS):
            blocks.append((f"{block_prefix}.{b}.{suffix}", tensors[16 + 19 * b + j]))
    _write(paths["model"], blocks)
    return paths


def write_vae_gguf(dims, tensors: Sequence[np.ndarray], path: str) -> str:
    """The reference's vae_decoder_weights.gguf from VAE tensors in
    ``sana_b200.synthetic_vae`` upload order (their diffusers names, fp32, PyTorch layouts)."""
    from .synthetic_vae import vae_tensor_specs
    specs = vae_tensor_specs(dims)
    _write(path, [(name, t) for (name, _, _), t in zip(specs, tensors)])
    return path


def write_synthetic_weights(directory: str, n_blocks: int = 28, vae_channels=(128, 256, 512, 512, 1024, 1024),
                            seed: int = 0) -> dict:
    """A weights directory for the front ends: denoiser of the default ModelDims widths with
    ``n_blocks`` blocks, a decoder with ``vae_channels`` (innermost last; ResBlocks in the first
    half), normal(0, 0.02) weights drawn with numpy (fast; not the torch generator), unit norms."""
    from .synthetic import ModelDims, model_tensor_specs
    from .synthetic_vae import VaeDims, vae_tensor_specs
    rng = np.random.default_rng(seed)

    def draw(shape, kind):
        if kind in ("ones", "norm_w"):
            return np.ones(shape, np.float32)
        if kind in ("bias", "norm_b"):
            return np.zeros(shape, np.float32)
        std = 1.0 / np.sqrt(1152.0) if kind == "table" else 0.02
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))

    d = ModelDims(n_blocks=n_blocks)
    paths = write_checkpoint_gguf([draw(s, k) for _, s, k in model_tensor_specs(d)], n_blocks, directory)
    n = len(vae_channels)
    vd = VaeDims(channels=tuple(vae_channels), res_blocks=tuple(i < n // 2 for i in range(n)), layers=(3,) * n)
    paths["vae"] = os.path.join(directory, "vae_decoder_weights.gguf")
    _write(paths["vae"], [(name, draw(s, k)) for name, s, k in vae_tensor_specs(vd)])
    enc = os.path.join(directory, "gemma2_text_encoder", "gemma-2-2b-it-f32.gguf")
    os.makedirs(os.path.dirname(enc), exist_ok=True)
    with open(enc, "wb") as f:
        f.write(b"the text-encoder stand-in only opens this file\n")
    paths["gemma"] = enc
    return paths


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description="random-initialised Sana weights for the reference front ends")
    ap.add_argument("directory")
    ap.add_argument("--blocks", type=int, default=28)
    ap.add_argument("--vae-channels", default="128,256,512,512,1024,1024")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    for k, v in write_synthetic_weights(a.directory, a.blocks, [int(c) for c in a.vae_channels.split(",")],
                                        a.seed).items():
        print(k, v)
