"""Guidance across two GPUs (the latency mode of one image: the unconditional branch on one GPU,
the conditional one on another, one noise-prediction exchange per step inside the guidance +
scheduler kernel; transformer.cpp:570-602, scheduler.cpp:272-318).

* without a GPU: the pairing of ranks (sana_b200.cfgpair) over world-size-2 and -4 gloo groups,
  with stand-ins for the export / connect calls;
* on two GPUs: the paired loop against the one-GPU loop of the same image (both GPUs end with
  the same latents, equal to the one-GPU result within the bf16 tolerance), and a partner that
  never runs its loop makes the bounded wait expire (SANA_ERR_TIMEOUT) without hanging.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))


def test_pair_of():
    from sana_b200.cfgpair import pair_of
    assert pair_of(0, 2) == (0, 0, 1) and pair_of(1, 2) == (0, 1, 0)
    assert pair_of(5, 8) == (2, 1, 4)
    with pytest.raises(ValueError):
        pair_of(0, 3)
    with pytest.raises(ValueError):
        pair_of(2, 2)


def _pairing_rank(rank, world, port, q):
    _env(rank, world, port)
    import datetime

    import torch.distributed as dist
    from sana_b200.cfgpair import pair_up
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    got = {}

    def connect(branch, handle):
        got["branch"], got["handle"] = branch, handle

    branch = pair_up(lambda: bytes([rank]) * 64, connect)
    q.put((rank, branch, got["branch"], got["handle"]))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_pair_up_swaps_handles_within_pairs(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pairing_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, branch, connected_branch, handle in results:
        assert branch == connected_branch == rank % 2
        assert handle == bytes([rank ^ 1]) * 64


# --- on two GPUs -------------------------------------------------------------------------------

DIMS = dict(n_blocks=2, hidden=256, latent_channels=16, caption_dim=96, ff_expanded=640, self_heads=8,
            cross_heads=4)
STEPS = 6


def _model():
    from sana_b200 import randn_torch_cpu
    from sana_b200 import synthetic as syn
    d = syn.ModelDims(**DIMS)
    return d, syn.generate_model(d, randn_torch_cpu, base_seed=21, bias_std=0.02)


def _inputs(d):
    from sana_b200 import randn_torch_cpu
    from sana_b200 import synthetic as syn
    enc = syn.encoder_states(randn_torch_cpu, 2, 24, d.caption_dim, 5)
    bias = syn.attention_bias([6, 24], 24)
    lat = syn.latents(randn_torch_cpu, 1, d.latent_channels, 16, 16, 6)
    return lat, enc, bias


def _pair_rank(rank, port, q, partner_runs):
    try:
        _pair_rank_body(rank, port, q, partner_runs)
    except BaseException as e:  # report instead of leaving the parent waiting on the queue
        q.put((rank, f"raised {type(e).__name__}: {e}", None))
        raise


def _pair_rank_body(rank, port, q, partner_runs):
    _env(rank, 2, port)
    import datetime

    import torch
    import torch.distributed as dist
    from sana_b200 import SANA_MODE_BF16, SanaCuda, SanaError
    from sana_b200.cfgpair import connect_engine
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120))
    d, tensors = _model()
    lat, enc, bias = _inputs(d)
    g = SanaCuda(rank, SANA_MODE_BF16)
    g.upload_checkpoint(d.as_args(), tensors)
    branch = connect_engine(g, lat.size)
    dl = torch.from_numpy(lat).cuda()
    de = torch.from_numpy(np.ascontiguousarray(enc[branch:branch + 1])).cuda()
    db = torch.from_numpy(np.ascontiguousarray(bias[branch:branch + 1])).cuda()
    out = torch.empty_like(dl)
    torch.cuda.synchronize()
    if not partner_runs:
        # rank 1 stays connected but never runs its loop; rank 0's waits must expire. Rank 1
        # keeps its region (which rank 0's kernels write) until rank 0 has finished.
        if rank == 0:
            g.set_wait_limit(2_000_000)  # 2 ms
            try:
                g.denoise_loop_pair_device(dl.data_ptr(), 1, 16, 16, de.data_ptr(), 24, d.caption_dim, db.data_ptr(),
                                           out.data_ptr(), 4.5, STEPS)
                g.synchronize()
                q.put((rank, "no error", None))
            except SanaError as e:
                q.put((rank, "timeout" if e.code == 3 else f"error {e.code}", None))
            g.cfg_pair_close()
        dist.barrier()
        g.cfg_pair_close()
        dist.destroy_process_group()
        return
    results = []
    for _ in range(3):  # eager, recorded, replayed
        g.denoise_loop_pair_device(dl.data_ptr(), 1, 16, 16, de.data_ptr(), 24, d.caption_dim, db.data_ptr(),
                                   out.data_ptr(), 4.5, STEPS)
        g.synchronize()
        results.append(out.cpu().numpy())
    single = None
    if rank == 0:
        single = g.denoise_loop(lat, enc, bias, 4.5, STEPS)
    q.put((rank, results, single))
    # every paired kernel has completed on both GPUs (synchronize above) before either unmaps
    g.cfg_pair_close()
    dist.barrier()
    dist.destroy_process_group()


def _run_pair(partner_runs):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pair_rank, args=(r, port, q, partner_runs)) for r in range(2)]
    for p in procs:
        p.start()
    n = 2 if partner_runs else 1
    out = sorted((q.get(timeout=600) for _ in range(n)), key=lambda t: t[0])
    for _, what, _ in out:
        assert not (isinstance(what, str) and what.startswith("raised")), what
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


def _need_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


@pytest.mark.gpu
def test_pair_loop_matches_one_gpu():
    _need_two_gpus()
    (r0, res0, single), (r1, res1, _) = _run_pair(True)
    for a, b in zip(res0, res1):
        np.testing.assert_array_equal(a, b)  # both GPUs hold the same guided latents
    np.testing.assert_array_equal(res0[1], res0[2])  # recorded loop replays exactly
    a, b = res0[2].astype(np.float64).ravel(), single.astype(np.float64).ravel()
    cos = a @ b / (np.linalg.norm(a) * np.linalg.norm(b))
    rel = np.linalg.norm(a - b) / np.linalg.norm(b)
    print(f"pair vs one GPU: cosine {cos:.7f}, rel-L2 {rel:.2e}")
    assert cos > 0.9999 and rel < 1e-2


@pytest.mark.gpu
def test_pair_wait_expires_without_partner():
    _need_two_gpus()
    [(rank, what, _)] = _run_pair(False)
    assert rank == 0 and what == "timeout"
