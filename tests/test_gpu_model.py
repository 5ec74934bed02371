"""CUDA path, whole model pieces, through the C ABI.

* small model (hidden 64, 2 blocks): caption projection, block stages, the no-CFG forward
  and a 4-step CFG loop against the compiled reference's golden outputs;
* full-size Sana-0.6B block 0 at config-0 shapes ([2, 1024, 1152], 36x32 and 16x72 self
  heads) against the oracle: per-stage relative L2 <= 1e-2 in bf16 mode, <= 1e-4 in the
  fp32 check mode;
* full-size block 0 at config 3's 4096 tokens ([2, 4096, 1152]) and at config 2's mixed
  caption masks, against the oracle (same bars), the oracle pinned on the reference's stage
  outputs;
* the config-1 20-step image against the reference's golden latents (cosine >= 0.999), and
  properties at config-3 size (4096 tokens).
"""
import concurrent.futures as cf
import importlib.util
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
MG = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(MG)
syn = MG.syn

BLOCK_BF16 = 1e-2  # per-block relative L2, bf16 mode
BLOCK_F32 = 1e-4   # per-block relative L2, fp32 check mode


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def product_model(d, base_seed=0, bias_std=0.0):
    """The synthetic checkpoint drawn with the product's generator, tensors in parallel."""
    from sana_b200 import randn_torch_cpu
    specs = syn.model_tensor_specs(d)
    with cf.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
        return list(ex.map(lambda j: syn.generate_tensor(specs[j], j, d, randn_torch_cpu, base_seed, 0.02, bias_std),
                           range(len(specs))))


@pytest.fixture(scope="module", params=["f32", "bf16"])
def small(request):
    from sana_b200 import SANA_MODE_BF16, SANA_MODE_F32, SanaCuda, randn_torch_cpu
    g = SanaCuda(0, SANA_MODE_F32 if request.param == "f32" else SANA_MODE_BF16)
    tensors = syn.generate_model(MG.SMALL, randn_torch_cpu, base_seed=5, bias_std=0.02)
    return request.param, g.model(tensors, *MG.SMALL.as_args())


def test_small_model_matches_golden(small):
    """Every stage of the small-model recipe against the reference build's outputs, the
    timestep embedding (emb, tmod at t = 999 and 500) through its own device entry point."""
    from sana_b200 import randn_torch_cpu
    mode, m = small
    gold = np.load(os.path.join(GOLDEN, "model_small.npz"))
    got = MG.small_model_run(m, randn_torch_cpu)
    tol = {"f32": 1e-4, "bf16": 3e-2}[mode]
    for k in ("ctx", "emb", "tmod", "after_self", "after_cross", "after_ff", "noise_pred", "loop4"):
        e = rel_err(got[k], gold[k])
        assert e < tol, (mode, k, e)


def test_time_embedding_matches_oracle_at_full_size(oracle):
    """The full-size timestep embedding + t_block (256 -> 1152 -> 1152, SiLU, 1152 -> 6912) on
    the device against the oracle at the schedule's first, middle and last timesteps, as one
    batch of per-sequence timesteps."""
    from sana_b200 import SANA_MODE_BF16, SANA_MODE_F32, SanaCuda
    d1 = syn.ModelDims(n_blocks=1)
    tensors = product_model(d1, base_seed=3, bias_std=0.02)
    m = oracle.model(tensors, *d1.as_args())
    tvals = [999.0, 968.9, 500.0, 63.25, 1.0]
    want_emb, want_tmod = m.time_embed(tvals)
    for mode, tol in ((SANA_MODE_F32, 1e-5), (SANA_MODE_BF16, 1e-2)):
        g = SanaCuda(0, mode)
        g.upload_checkpoint(d1.as_args(), tensors)
        emb, tmod = g.time_embed(tvals)
        assert rel_err(emb, want_emb) < tol, (mode, rel_err(emb, want_emb))
        assert rel_err(tmod, want_tmod) < tol, (mode, rel_err(tmod, want_tmod))
        g.close()


# --- full size --------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def block0_inputs(oracle):
    d1 = syn.ModelDims(n_blocks=1)
    tensors = product_model(d1, base_seed=0)
    m = oracle.model(tensors, *d1.as_args())
    from sana_b200 import randn_torch_cpu
    enc = syn.encoder_states(randn_torch_cpu, 2, 300, d1.caption_dim, 7)
    bias = syn.attention_bias([8, 24], 300)
    ctx = m.project_caption(enc)
    emb, tmod = m.time_embed([999.0, 999.0])
    x = syn._draw(randn_torch_cpu, 2 * 1024 * d1.hidden, 400).reshape(2, 1024, d1.hidden)
    ref = m.block_forward(0, x, ctx, tmod, bias)
    return d1, tensors, x, ctx, tmod, bias, ref


def test_oracle_full_block_matches_reference_signature(block0_inputs):
    path = os.path.join(GOLDEN, "block0_full.npz")
    if not os.path.exists(path):
        pytest.skip("block0_full.npz not generated")
    g = np.load(path)
    for name, a in zip(("after_self", "after_cross", "after_ff"), block0_inputs[-1]):
        sig = MG._signature(a)
        assert rel_err(sig["row_sq"], g[f"{name}_row_sq"]) < 1e-5


@pytest.mark.parametrize("mode", ["bf16", "f32"])
def test_full_block_parity(block0_inputs, mode):
    from sana_b200 import SANA_MODE_BF16, SANA_MODE_F32, SanaCuda
    d1, tensors, x, ctx, tmod, bias, ref = block0_inputs
    g = SanaCuda(0, SANA_MODE_BF16 if mode == "bf16" else SANA_MODE_F32)
    g.upload_checkpoint(d1.as_args(), tensors)
    got = g.block_forward(0, x, ctx, tmod, bias)
    tol = BLOCK_BF16 if mode == "bf16" else BLOCK_F32
    for name, a, b in zip(("after_self", "after_cross", "after_ff"), got, ref):
        # the residual stream dominates the stage outputs; also check the branch deltas
        e = rel_err(a, b)
        assert e < tol, (mode, name, e)
    e_branch = rel_err(got[2] - x, ref[2] - x)
    assert e_branch < (5 * tol if mode == "bf16" else 10 * tol), e_branch


def test_full_block_baseline_heads(oracle):
    """BASELINE.json's literal 16 x 72 self-attention heads (the reference's callers use 36 x 32)."""
    from sana_b200 import SANA_MODE_BF16, SanaCuda, randn_torch_cpu
    d1 = syn.ModelDims(n_blocks=1, self_heads=16)
    tensors = product_model(d1, base_seed=1, bias_std=0.02)
    m = oracle.model(tensors, *d1.as_args())
    enc = syn.encoder_states(randn_torch_cpu, 2, 300, d1.caption_dim, 8)
    bias = syn.attention_bias([24, 8], 300)
    ctx = m.project_caption(enc)
    _, tmod = m.time_embed([500.0, 500.0])
    x = syn._draw(randn_torch_cpu, 2 * 1024 * d1.hidden, 401).reshape(2, 1024, d1.hidden)
    ref = m.block_forward(0, x, ctx, tmod, bias)
    g = SanaCuda(0, SANA_MODE_BF16)
    g.upload_checkpoint(d1.as_args(), tensors)
    got = g.block_forward(0, x, ctx, tmod, bias)
    for a, b in zip(got, ref):
        assert rel_err(a, b) < BLOCK_BF16


@pytest.fixture(scope="module", params=sorted(MG.BLOCK_CASES))
def block_case(request, oracle):
    """Block 0 of the full-size model on a BLOCK_CASES input of make_golden.py: config 3's
    4096-token grid ([2, 4096, 1152]) or four 1024-token sequences with mixed caption masks
    (valid lengths 17, 120, 64, 9), with the oracle's stage outputs."""
    from sana_b200 import randn_torch_cpu
    d1 = syn.ModelDims(n_blocks=1)
    tensors = product_model(d1, base_seed=0)
    m = oracle.model(tensors, *d1.as_args())
    x, ctx, tmod, bias = MG.block_case_inputs(m, randn_torch_cpu, request.param)
    return request.param, d1, tensors, x, ctx, tmod, bias, m.block_forward(0, x, ctx, tmod, bias)


def test_block_case_oracle_matches_reference_signature(block_case):
    """The oracle's stage outputs against the reference build's (tests/golden/<case>.npz)."""
    name, *_, ref = block_case
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    for stage, a in zip(("after_self", "after_cross", "after_ff"), ref):
        sig = MG._signature(a)
        assert rel_err(sig["head"], g[f"{stage}_head"]) < 1e-5, (name, stage)
        assert rel_err(sig["row_sum"], g[f"{stage}_row_sum"]) < 1e-4, (name, stage)
        assert rel_err(sig["row_sq"], g[f"{stage}_row_sq"]) < 1e-5, (name, stage)


@pytest.mark.parametrize("mode", ["bf16", "f32"])
def test_block_case_parity(block_case, mode):
    """Per-stage parity at config 3's 4096 tokens and at config 2's mixed masks: relative L2
    <= 1e-2 in bf16 mode and <= 1e-4 in the fp32 check mode, as for the 1024-token block."""
    from sana_b200 import SANA_MODE_BF16, SANA_MODE_F32, SanaCuda
    name, d1, tensors, x, ctx, tmod, bias, ref = block_case
    g = SanaCuda(0, SANA_MODE_BF16 if mode == "bf16" else SANA_MODE_F32)
    g.upload_checkpoint(d1.as_args(), tensors)
    got = g.block_forward(0, x, ctx, tmod, bias)
    tol = BLOCK_BF16 if mode == "bf16" else BLOCK_F32
    for stage, a, b in zip(("after_self", "after_cross", "after_ff"), got, ref):
        e = rel_err(a, b)
        assert e < tol, (name, mode, stage, e)
    e_branch = rel_err(got[2] - x, ref[2] - x)
    assert e_branch < (5 * tol if mode == "bf16" else 10 * tol), (name, e_branch)
    g.close()


@pytest.fixture(scope="module")
def full_gpu():
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    d = syn.ModelDims()
    tensors = product_model(d, base_seed=0)
    g = SanaCuda(0, SANA_MODE_BF16)
    g.upload_checkpoint(d.as_args(), tensors)
    del tensors
    return g


def test_loop20_matches_reference_golden(full_gpu):
    path = os.path.join(GOLDEN, "loop20_full.npz")
    if not os.path.exists(path):
        pytest.skip("loop20_full.npz not generated")
    from sana_b200 import randn_torch_cpu
    gold = np.load(path)["latents"]
    enc = syn.encoder_states(randn_torch_cpu, 2, 300, 2304, 7)
    bias = syn.attention_bias([8, 24], 300)
    lat = syn.latents(randn_torch_cpu, 1, 32, 32, 32, 42)
    out = full_gpu.denoise_loop(lat, enc, bias, 4.5, 20)
    assert np.isfinite(out).all()
    c = cosine(out, gold)
    assert c >= 0.999, c
    # the captured-graph replay gives the same result as the first (eager) call
    out2 = full_gpu.denoise_loop(lat, enc, bias, 4.5, 20)
    assert np.array_equal(out, out2)


def test_forward_config0_matches_reference_golden(full_gpu):
    path = os.path.join(GOLDEN, "forward_full.npz")
    if not os.path.exists(path):
        pytest.skip("forward_full.npz not generated")
    from sana_b200 import randn_torch_cpu
    gold = np.load(path)["noise_pred"]
    enc = syn.encoder_states(randn_torch_cpu, 2, 300, 2304, 7)
    bias = syn.attention_bias([8, 24], 300)
    lat = syn.latents(randn_torch_cpu, 2, 32, 32, 32, 42)
    ctx = full_gpu.project_caption_model(enc)
    out = full_gpu.forward(lat, 999.0, ctx, bias)
    print(f"config-0 forward vs reference: cosine {cosine(out, gold):.6f}, rel-L2 {rel_err(out, gold):.3e}")
    assert cosine(out, gold) >= 0.999
    assert rel_err(out, gold) < 1e-2  # measured 4.6e-3 over the 28 blocks in bf16


def test_batched_loop_images_are_independent(full_gpu):
    """Config-2 style batch: each image of a batch gets the latents it would get alone."""
    from sana_b200 import randn_torch_cpu
    B, L = 3, 300
    lens = syn.batch_valid_lengths(B, 11)
    enc = syn.encoder_states(randn_torch_cpu, 2 * B, L, 2304, 21)
    bias = syn.attention_bias(lens, L)
    lat = syn.latents(randn_torch_cpu, B, 32, 32, 32, 22)
    batch = full_gpu.denoise_loop(lat, enc, bias, 4.5, 4)
    for i in range(B):
        idx = [i, B + i]
        one = full_gpu.denoise_loop(lat[i:i + 1], enc[idx], bias[idx], 4.5, 4)
        assert cosine(batch[i], one[0]) > 0.9999


@pytest.mark.parametrize("pairs,hidden,pos_rows,L", [(3, 2304, 324, 300), (2, 30, 12, 5), (1, 2304, 300, 300)])
def test_prompt_pairs_device_matches_oracle(oracle, pairs, hidden, pos_rows, L):
    """The encoder output contract assembled on the device equals the reference's host tail
    (restated in the oracle) pair by pair, bit for bit, mask signs included."""
    import torch
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    g = SanaCuda(0, SANA_MODE_BF16)
    rng = np.random.default_rng(pairs * 131 + hidden)
    neg = rng.standard_normal((pairs, L, hidden)).astype(np.float32)
    pos = rng.standard_normal((pairs, pos_rows, hidden)).astype(np.float32)
    neg_real = [int(v) for v in rng.integers(0, L + 1, pairs)]
    pos_real = [int(v) for v in rng.integers(0, pos_rows + 1, pairs)]
    pos_real[0] = pos_rows
    enc, bias = g.prompt_pairs_device(torch.from_numpy(neg).cuda(), neg_real, torch.from_numpy(pos).cuda(), pos_real, L)
    torch.cuda.synchronize()
    enc, bias = enc.cpu().numpy(), bias.cpu().numpy()
    for p in range(pairs):
        e, b = oracle.prompt_pair_assemble(neg[p], neg_real[p], pos[p], pos_real[p], L)
        for half, row in ((0, p), (1, pairs + p)):
            assert np.array_equal(enc[row].view(np.uint32), e[half].view(np.uint32))
            assert np.array_equal(bias[row].view(np.uint32), b[half].view(np.uint32))
    with pytest.raises(ValueError, match="exceeds padded_length"):
        g.prompt_pairs_device(torch.from_numpy(neg).cuda(), [L + 1] * pairs, torch.from_numpy(pos).cuda(), pos_real, L)
    if pairs == 3:  # buffers offset by one float (not 16-byte aligned): the scalar copy, same result
        nb = torch.zeros(neg.size + 1, dtype=torch.float32, device="cuda")
        pb = torch.zeros(pos.size + 1, dtype=torch.float32, device="cuda")
        nb[1:] = torch.from_numpy(neg.ravel()).cuda()
        pb[1:] = torch.from_numpy(pos.ravel()).cuda()
        enc2, bias2 = g.prompt_pairs_device(nb[1:].view(neg.shape), neg_real, pb[1:].view(pos.shape), pos_real, L)
        torch.cuda.synchronize()
        assert np.array_equal(enc2.cpu().numpy(), enc) and np.array_equal(bias2.cpu().numpy(), bias)
    if pairs == 1:  # more pairs than one launch takes
        many = torch.zeros((65, L, hidden), dtype=torch.float32, device="cuda")
        many_pos = torch.zeros((65, pos_rows, hidden), dtype=torch.float32, device="cuda")
        with pytest.raises(ValueError, match="prompt pair count"):
            g.prompt_pairs_device(many, [1] * 65, many_pos, [1] * 65, L)


def test_loop_from_device_assembled_prompts(full_gpu, oracle):
    """Two prompt pairs assembled on the device feed the device loop directly; the result
    equals the host loop on the host-assembled conditioning (negatives first)."""
    import torch
    from sana_b200 import randn_torch_cpu
    B, L, D, rows = 2, 300, 2304, 324
    neg = randn_torch_cpu(B * L * D, 71).reshape(B, L, D)
    pos = randn_torch_cpu(B * rows * D, 72).reshape(B, rows, D)
    neg_real, pos_real = [9, 17], [60, 324]
    lat = syn.latents(randn_torch_cpu, B, 32, 32, 32, 73)
    enc_h = np.empty((2 * B, L, D), np.float32)
    bias_h = np.empty((2 * B, 1, L), np.float32)
    for p in range(B):
        e, b = oracle.prompt_pair_assemble(neg[p], neg_real[p], pos[p], pos_real[p], L)
        enc_h[p], enc_h[B + p], bias_h[p], bias_h[B + p] = e[0], e[1], b[0], b[1]
    host = full_gpu.denoise_loop(lat, enc_h, bias_h, 4.5, 3)
    enc_d, bias_d = full_gpu.prompt_pairs_device(torch.from_numpy(neg).cuda(), neg_real, torch.from_numpy(pos).cuda(),
                                                 pos_real, L)
    lat_d = torch.from_numpy(lat).cuda()
    out_d = torch.empty_like(lat_d)
    full_gpu.denoise_loop_device(lat_d.data_ptr(), B, 32, 32, enc_d.data_ptr(), L, D, bias_d.data_ptr(),
                                 out_d.data_ptr(), 4.5, 3)
    torch.cuda.synchronize()
    assert np.array_equal(out_d.cpu().numpy(), host)


def test_highres_step_is_finite_and_consistent(full_gpu):
    """Config 3 (64 x 64 latent, 4096 tokens): one step through the loop API and through
    the single-step API agree."""
    from sana_b200 import randn_torch_cpu
    enc = syn.encoder_states(randn_torch_cpu, 2, 300, 2304, 7)
    bias = syn.attention_bias([8, 24], 300)
    lat = syn.latents(randn_torch_cpu, 1, 32, 64, 64, 43)
    one_step = full_gpu.denoise_loop(lat, enc, bias, 4.5, 1)
    assert np.isfinite(one_step).all()
    ctx = full_gpu.project_caption_model(enc)
    from sana_b200 import scheduler_schedule
    ts, sg = scheduler_schedule(1)
    lat2, si, lo, hist = full_gpu.denoise_step(lat, ctx, bias, 4.5, float(ts[0]), sg, 0, 0, [])
    assert si == 1 and lo == 1 and len(hist) == 1
    assert cosine(lat2, one_step) > 0.9999


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_gguf_upload_matches_pointer_upload(tmp_path, mode):
    """The reference's three GGUF weight files, mapped and uploaded straight into the device
    cache (sana_cuda_upload_gguf), give the same model as the pointer-table upload of the same
    checkpoint: identical denoising-loop latents and caption projection, in both modes."""
    from sana_b200 import SANA_MODE_BF16, SANA_MODE_F32, SanaCuda, randn_torch_cpu
    from sana_b200.gguf_files import write_checkpoint_gguf
    d = syn.ModelDims(n_blocks=3, hidden=128, latent_channels=8, caption_dim=96, ff_expanded=320, self_heads=4,
                      cross_heads=2)
    tensors = syn.generate_model(d, randn_torch_cpu, base_seed=11, bias_std=0.02)
    paths = write_checkpoint_gguf(tensors, d.n_blocks, str(tmp_path))
    m = SANA_MODE_F32 if mode == "f32" else SANA_MODE_BF16
    a, b = SanaCuda(0, m), SanaCuda(0, m)
    a.upload_checkpoint(d.as_args(), tensors)
    dims = b.upload_gguf(paths["model"], paths["caption"], paths["denoiser"], d.self_heads, d.cross_heads)
    assert dims == tuple(d.as_args())
    enc = syn.encoder_states(randn_torch_cpu, 2, 20, d.caption_dim, 3)
    bias = syn.attention_bias([5, 12], 20)
    lat = syn.latents(randn_torch_cpu, 1, d.latent_channels, 8, 8, 4)
    assert np.array_equal(a.denoise_loop(lat, enc, bias, 4.5, 4), b.denoise_loop(lat, enc, bias, 4.5, 4))
    assert np.array_equal(a.project_caption_model(enc), b.project_caption_model(enc))


def test_gguf_upload_errors_follow_the_loaders(tmp_path):
    """A missing tensor is the loaders' invalid_argument (ValueError here); a non-fp32 tensor
    or a wrong shape is a runtime error (SanaError), as weights_io.cpp / transformer.cpp raise."""
    import gguf
    from sana_b200 import SanaCuda, SanaError, randn_torch_cpu
    from sana_b200.gguf_files import write_checkpoint_gguf
    d = syn.ModelDims(n_blocks=1, hidden=64, latent_channels=4, caption_dim=48, ff_expanded=160, self_heads=2,
                      cross_heads=2)
    tensors = syn.generate_model(d, randn_torch_cpu, base_seed=2)
    paths = write_checkpoint_gguf(tensors, d.n_blocks, str(tmp_path))
    g = SanaCuda(0)

    def rewrite(path, fn):
        r = gguf.GGUFReader(path)
        items = [(t.name, np.array(t.data).reshape(tuple(int(x) for x in reversed(t.shape)))) for t in r.tensors]
        del r
        w = gguf.GGUFWriter(path, arch="sana")
        for name, arr in fn(items):
            w.add_tensor(name, arr)
        w.write_header_to_file()
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()

    rewrite(paths["denoiser"], lambda items: [x for x in items if x[0] != "proj_out.bias"])
    with pytest.raises(ValueError, match="weight name not found"):
        g.upload_gguf(paths["model"], paths["caption"], paths["denoiser"], 2, 2)
    write_checkpoint_gguf(tensors, d.n_blocks, str(tmp_path))
    rewrite(paths["caption"], lambda items: [(n, a.astype(np.float16) if n.endswith("linear_2.weight") else a)
                                             for n, a in items])
    with pytest.raises(SanaError, match="only float32"):
        g.upload_gguf(paths["model"], paths["caption"], paths["denoiser"], 2, 2)
    write_checkpoint_gguf(tensors, d.n_blocks, str(tmp_path))
    rewrite(paths["model"], lambda items: [(n, a[:, :32] if n.endswith("attn1.to_q.weight") else a) for n, a in items])
    with pytest.raises(SanaError, match="has shape"):
        g.upload_gguf(paths["model"], paths["caption"], paths["denoiser"], 2, 2)


@pytest.mark.parametrize("cfg", [dict(solver_heun=1), dict(solver_order=1),
                                 dict(num_train_timesteps=500, flow_shift=2.0, solver_heun=1)])
def test_loop_with_scheduler_config_equals_stepped_loop(cfg):
    """run_full_denoising_loop_with_cfg with a non-default SanaSchedulerConfig: the captured
    device loop (sana_cuda_denoise_loop_config) equals the loop run step by step through
    run_full_denoising_step_with_cfg (sana_cuda_denoise_step_config), whose scheduler
    arithmetic the scheduler-config tests hold against the reference. The graph replay of the
    second call equals the eager first call."""
    from sana_b200 import SANA_MODE_F32, SanaCuda, randn_torch_cpu, scheduler_schedule_config
    g = SanaCuda(0, SANA_MODE_F32)
    tensors = syn.generate_model(MG.SMALL, randn_torch_cpu, base_seed=5, bias_std=0.02)
    g.upload_checkpoint(MG.SMALL.as_args(), tensors)
    d = MG.SMALL
    enc = syn.encoder_states(randn_torch_cpu, 2, 12, d.caption_dim, 3)
    bias = syn.attention_bias([5, 12], 12)
    lat = syn.latents(randn_torch_cpu, 1, d.latent_channels, 4, 4, 4)
    n = 5
    loop = g.denoise_loop_config(cfg, lat, enc, bias, 4.5, n)
    assert np.array_equal(g.denoise_loop_config(cfg, lat, enc, bias, 4.5, n), loop)  # graph replay
    ts, sg = scheduler_schedule_config(n, **cfg)
    ctx = g.project_caption_model(enc)
    x, step, lower, hist = lat, 0, 0, []
    for _ in range(n):
        x, step, lower, hist = g.denoise_step_config(cfg, x, ctx, bias, 4.5, float(ts[step]), sg, step, lower, hist)
    order = cfg.get("solver_order", 2)
    assert step == n and lower == min(n, order) and len(hist) == min(n, order)
    assert rel_err(x, loop) < 1e-6
    # the default config differs from these (the configs change the trajectory)
    assert rel_err(g.denoise_loop(lat, enc, bias, 4.5, n), loop) > 1e-5
