"""Writes a denoiser checkpoint as the reference's three GGUF weight files.

sana.cpp's front end reads ``model_weights.gguf`` (the transformer blocks),
``caption_weights.gguf`` (the caption projection) and ``denoiser_weights.gguf`` (patch embed,
time embedding, t_block, caption norm, final table and projection) from its weights directory
(infer_main.cpp:347-365), every tensor fp32 under its diffusers name with linear weights in
PyTorch's [out, in] layout (load_linear_weight_tensor transposes them on load). This writes a
checkpoint list in ``sana_b200.synthetic`` order into that form with the ``gguf`` package, so
synthetic or converted weights can go through ``sana_cuda_upload_gguf`` as real ones would.
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
