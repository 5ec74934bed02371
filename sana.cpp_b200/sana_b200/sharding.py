"""Images of the batched workload sharded across ranks (one rank per GPU).

The denoiser's images are independent (each image's CFG pair of sequences only meets itself
in apply_classifier_free_guidance, transformer.cpp:570-602), so a batch splits into
contiguous image ranges with no exchange during the loop; the final latents are gathered
once at the end. Every input of an image is drawn from seeds of its global index, so an
image's result does not depend on how many ranks share the batch.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np

from . import synthetic as syn

LATENT_SEED = 42
CAPTION_SEED = 7
LENGTH_SEED = 1000


def shard_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """(first image, image count) of `rank`: contiguous, the first total % world ranks take one
    image more than the others."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if total < 0:
        raise ValueError("total must be non-negative")
    base, extra = divmod(total, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def image_valid_lengths(index: int, lo: int = 8, hi: int = 120) -> Tuple[int, int]:
    """(uncond, cond) valid caption lengths of image `index`, uniform in [lo, hi]."""
    rng = np.random.default_rng(LENGTH_SEED + index)
    u, c = rng.integers(lo, hi + 1, size=2)
    return int(u), int(c)


def image_inputs(randn, first: int, count: int, latent_shape: Sequence[int] = (32, 32, 32),
                 caption_len: int = 300, caption_dim: int = 2304):
    """Inputs of images [first, first + count) in the C ABI's batch layout: latents
    [count, Cl, H, W]; encoder states [2 count, L, D] and additive caption mask [2 count, 1, L]
    with the uncond block first; and the 2 count valid lengths in that order."""
    cl, h, w = latent_shape
    lat = np.empty((count, cl, h, w), np.float32)
    enc = np.empty((2 * count, caption_len, caption_dim), np.float32)
    lens_u: List[int] = []
    lens_c: List[int] = []
    for j in range(count):
        i = first + j
        lat[j] = syn.latents(randn, 1, cl, h, w, LATENT_SEED + 97 * i)[0]
        enc[j] = syn.encoder_states(randn, 1, caption_len, caption_dim, CAPTION_SEED + 2 * 97 * i)[0]
        enc[count + j] = syn.encoder_states(randn, 1, caption_len, caption_dim, CAPTION_SEED + 2 * 97 * i + 97)[0]
        u, c = image_valid_lengths(i)
        lens_u.append(min(u, caption_len))
        lens_c.append(min(c, caption_len))
    lens = lens_u + lens_c
    return lat, enc, syn.attention_bias(lens, caption_len), lens


def gather_images(local, total: int, world: int, group=None):
    """All-gather the ranks' image shards (dim 0 of a torch tensor, sizes from shard_range) into
    the full [total, ...] batch in image order, on every rank. Uneven shards are padded to the
    largest one for the collective and trimmed after it."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return local
    _, most = shard_range(total, world, 0)
    pad = local
    if local.shape[0] < most:
        pad = torch.zeros((most,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous(), group=group)
    return torch.cat([parts[r][: shard_range(total, world, r)[1]] for r in range(world)], dim=0)
