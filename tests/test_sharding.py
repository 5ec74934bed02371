"""The multi-GPU batch split (sana_b200.sharding): contiguous image shards, inputs drawn per
image so that a shard does not depend on the number of ranks, and the final gather of the
latents in image order -- run here as world-size-2 process groups on the gloo backend (CPU),
the same code path bench.py runs over NCCL with one rank per GPU."""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from sana_b200.sharding import gather_images, image_inputs, shard_range


@pytest.mark.parametrize("total,world", [(16, 1), (16, 2), (16, 8), (7, 2), (5, 4), (3, 3)])
def test_shard_range_partitions_the_batch(total, world):
    ranges = [shard_range(total, world, r) for r in range(world)]
    assert ranges[0][0] == 0
    for (f0, c0), (f1, _) in zip(ranges, ranges[1:]):
        assert f1 == f0 + c0
    assert sum(c for _, c in ranges) == total
    assert max(c for _, c in ranges) - min(c for _, c in ranges) <= 1


def test_shard_range_rejects_bad_ranks():
    with pytest.raises(ValueError):
        shard_range(16, 2, 2)
    with pytest.raises(ValueError):
        shard_range(16, 0, 0)


def test_image_inputs_do_not_depend_on_the_split():
    from sana_b200 import randn_torch_cpu
    kw = dict(latent_shape=(4, 4, 4), caption_len=12, caption_dim=8)
    lat, enc, bias, lens = image_inputs(randn_torch_cpu, 0, 4, **kw)
    parts = [image_inputs(randn_torch_cpu, f, 2, **kw) for f in (0, 2)]
    assert np.array_equal(lat, np.concatenate([p[0] for p in parts]))
    # encoder rows: uncond block (images 0..3) then cond block
    enc_split = np.concatenate([parts[0][1][:2], parts[1][1][:2], parts[0][1][2:], parts[1][1][2:]])
    assert np.array_equal(enc, enc_split)
    assert lens == parts[0][3][:2] + parts[1][3][:2] + parts[0][3][2:] + parts[1][3][2:]
    assert bias.shape == (8, 1, 12) and all(8 <= v <= 12 for v in lens)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, total, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        first, count = shard_range(total, world, rank)
        # each image's "latents" are a function of its global index only
        local = torch.stack([torch.full((3, 2), float(first + j)) for j in range(count)]) if count else \
            torch.zeros((0, 3, 2))
        full = gather_images(local, total, world)
        want = torch.stack([torch.full((3, 2), float(i)) for i in range(total)])
        # the bench's timing rule: every rank reports the slowest rank's time
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, bool(torch.equal(full, want)), float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [16, 7])
def test_gather_images_world_size_2_gloo(total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, total, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(r for r, _, _ in results) == [0, 1]
    assert all(ok for _, ok, _ in results)
    assert all(t == 2.0 for _, _, t in results)
