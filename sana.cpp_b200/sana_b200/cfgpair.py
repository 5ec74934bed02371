"""Guidance across two GPUs: pairing the ranks of a process group.

Ranks 2p and 2p+1 form pair p. Each rank exports its exchange region (a 64-byte CUDA IPC
handle), the handles travel over the process group (``all_gather_object``; any backend), each
rank maps its partner's and takes branch ``rank % 2`` (0 = the unconditional sequences of
apply_classifier_free_guidance, transformer.cpp:570-602, 1 = the conditional ones). A barrier
follows, so no rank runs a paired loop before its partner has mapped its region.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple


def pair_of(rank: int, world: int) -> Tuple[int, int, int]:
    """(pair index, branch, partner rank) of `rank`; the world size must be even."""
    if world < 2 or world % 2:
        raise ValueError(f"guidance across GPUs pairs ranks: the world size must be even, not {world}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return rank // 2, rank % 2, rank ^ 1


def pair_up(export: Callable[[], bytes], connect: Callable[[int, bytes], None], group: Optional[object] = None) -> int:
    """Exchanges handles within each pair of `group` and connects; returns this rank's branch.

    export() -> this rank's handle; connect(branch, partner_handle) maps the partner's region."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    _, branch, partner = pair_of(rank, world)
    handles = [None] * world
    dist.all_gather_object(handles, export(), group=group)
    connect(branch, handles[partner])
    dist.barrier(group)
    return branch


def connect_engine(g, capacity: int, group: Optional[object] = None) -> int:
    """pair_up for a SanaCuda handle: exports `capacity` latent elements of exchange space."""
    return pair_up(lambda: g.cfg_pair_export(capacity), g.cfg_pair_connect, group)
