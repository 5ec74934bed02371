"""Failure detection on the host (no GPU): a rank that never joins, a rank that stops between
steps, and a collective whose peer has gone -- as world-size-2 gloo process groups on CPU.
The surviving rank must leave with an error within its bound, never hang."""
import datetime
import multiprocessing as mp
import os
import socket
import time

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _put_and_exit(q, item):
    """Sends `item` and leaves at once (no teardown): the queue is flushed first, since
    os._exit would drop what its feeder thread has not written yet."""
    q.put(item)
    q.close()
    q.join_thread()
    os._exit(0)


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))


def _lonely_rank(port, q):
    """Rank 0 of 2; rank 1 never starts. init_ranks must give up after its timeout."""
    _env(0, 2, port)
    from sana_b200.watchdog import init_ranks
    t0 = time.time()
    try:
        init_ranks("gloo", timeout_s=3.0)
        q.put(("joined", time.time() - t0))
    except Exception as e:  # the store or the rendezvous times out
        q.put((type(e).__name__, time.time() - t0))


def test_rank_that_never_joins_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(_free_port(), q))
    p.start()
    what, dt = q.get(timeout=120)
    p.join(timeout=60)
    assert what != "joined", "rank 0 joined a group whose rank 1 never started"
    assert dt < 60, dt


def _heartbeat_rank(rank, port, q):
    """Both ranks join; rank 1 completes one step and exits. Rank 0 keeps stepping and, before
    its next collective, its heartbeat check reports rank 1 as lost."""
    _env(rank, 2, port)
    import torch.distributed as dist
    from sana_b200.watchdog import PeerLost, init_ranks
    _, _, watch = init_ranks("gloo", timeout_s=20.0)
    watch.max_age_s = 1.0
    watch.beat(1)
    dist.barrier()
    if rank == 1:
        _put_and_exit(q, (1, "left"))  # stops without any goodbye
    t0 = time.time()
    try:
        for step in range(2, 200):
            time.sleep(0.1)
            watch.beat(step)
            watch.check()
        _put_and_exit(q, (0, "no error"))
    except PeerLost as e:
        _put_and_exit(q, (0, ("lost", e.ranks, time.time() - t0)))


def test_stopped_rank_is_reported_before_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_heartbeat_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=90) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "left"
    kind, ranks, dt = got[0]
    assert kind == "lost" and ranks == [1] and dt < 10, got[0]


def _collective_rank(rank, port, q):
    """Rank 1 exits after joining; rank 0's next all-gather must fail within the group's
    timeout rather than wait for good."""
    _env(rank, 2, port)
    import torch
    import torch.distributed as dist
    from sana_b200.sharding import gather_images
    from sana_b200.watchdog import init_ranks
    init_ranks("gloo", timeout_s=5.0)
    dist.barrier()
    if rank == 1:
        _put_and_exit(q, (1, "left"))
    t0 = time.time()
    try:
        gather_images(torch.zeros((1, 4)), 2, 2)
        _put_and_exit(q, (0, ("completed", time.time() - t0)))
    except Exception as e:
        _put_and_exit(q, (0, (type(e).__name__, time.time() - t0)))


def test_collective_with_a_lost_peer_fails_within_the_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_collective_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=90) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    kind, dt = got[0]
    assert kind != "completed" and dt < 60, got[0]


def test_peer_watch_logic_with_a_fake_store():
    from sana_b200.watchdog import PeerLost, PeerWatch

    class Store(dict):
        def set(self, k, v):
            self[k] = v

        def check(self, keys):
            return all(k in self for k in keys)

        def get(self, k):
            return self[k]

    s = Store()
    w0 = PeerWatch(s, 0, 3, max_age_s=5.0)
    w1 = PeerWatch(s, 1, 3, max_age_s=5.0)
    now = time.time()
    w0.check(now)  # rank 2 has not joined yet, but within its grace period
    with pytest.raises(PeerLost) as e:
        w0.check(now + 10)
    assert e.value.ranks == [2] and "never joined" in str(e.value)
    PeerWatch(s, 2, 3, max_age_s=5.0)
    w0.beat(3)
    w1.check(time.time())
    with pytest.raises(PeerLost) as e:
        w0.check(time.time() + 6)
    assert sorted(e.value.ranks) == [1, 2]
