"""Host-side liveness of the ranks of a multi-GPU job.

Each rank publishes a heartbeat (its step count and a wall-clock stamp) through the
torch.distributed store of its process group, and, before its next collective (the final
latent gather), checks that every peer's heartbeat is recent. A peer that never joined, or
that stopped between steps, is reported as ``PeerLost`` on the host, so the surviving ranks
leave with an error instead of entering a collective that cannot complete. The process
group's own timeout (``init_ranks``) bounds whatever the check misses. Nothing here touches
a GPU: the device-side counterpart is the bounded wait of every kernel spin
(``sana_cuda_set_wait_limit``).
"""
from __future__ import annotations

import datetime
import json
import os
import time
from typing import List, Optional


class PeerLost(RuntimeError):
    def __init__(self, ranks: List[int], what: str):
        super().__init__(f"rank(s) {ranks} {what}")
        self.ranks = ranks


class PeerWatch:
    """Heartbeats of `world` ranks under `prefix` in `store` (a torch.distributed Store)."""

    def __init__(self, store, rank: int, world: int, max_age_s: float = 60.0, prefix: str = "sana/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.max_age_s, self.prefix = max_age_s, prefix
        self.started = time.time()
        self.beat(0)

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int) -> None:
        """Publishes this rank's progress (after each completed step)."""
        self.store.set(self._key(self.rank), json.dumps({"step": int(step), "t": time.time()}))

    def check(self, now: Optional[float] = None) -> None:
        """Raises PeerLost for peers with no heartbeat within max_age_s: ranks that never
        published one (after max_age_s since this watch started) or whose last one is stale."""
        now = time.time() if now is None else now
        missing, stale = [], []
        for r in range(self.world):
            if r == self.rank:
                continue
            key = self._key(r)
            if not self.store.check([key]):
                if now - self.started > self.max_age_s:
                    missing.append(r)
                continue
            hb = json.loads(self.store.get(key))
            if now - float(hb["t"]) > self.max_age_s:
                stale.append(r)
        if missing:
            raise PeerLost(missing, f"never joined within {self.max_age_s:.1f} s")
        if stale:
            raise PeerLost(stale, f"sent no heartbeat for more than {self.max_age_s:.1f} s")


def init_ranks(backend: str, timeout_s: float, device_id=None):
    """init_process_group from the launcher's environment (RANK, WORLD_SIZE, MASTER_ADDR,
    MASTER_PORT) with a bounded timeout: a rank that never joins makes the others fail after
    `timeout_s` instead of waiting for good. Returns (rank, world, PeerWatch or None)."""
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return rank, world, None
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device_id is not None:
        kw["device_id"] = device_id
    dist.init_process_group(backend, **kw)
    store = dist.distributed_c10d._get_default_store()
    return rank, world, PeerWatch(store, rank, world, max_age_s=timeout_s)
