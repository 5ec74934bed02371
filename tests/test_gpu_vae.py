"""The VAE decoder on the GPU (vae.cpp:243-325 run_vae_decode, vae_ops.cpp) through the C ABI,
against the reference build's golden outputs (tests/golden/vae.npz) and the oracle.

Tolerances: fp32 check mode follows the reference to rounding (rel-L2 <= 1e-4); the bf16
product path keeps activations in bf16 between ops with fp32 accumulation (rel-L2 <= 2e-2,
cosine >= 0.999)."""
import importlib.util
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
MG = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(MG)

TOL = {"f32": 1e-4, "bf16": 2e-2}


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def decoder(mode, dims, seed):
    from sana_b200 import SANA_MODE_BF16, SANA_MODE_F32, SanaCuda, randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    g = SanaCuda(0, SANA_MODE_F32 if mode == "f32" else SANA_MODE_BF16)
    g.vae_upload(dims, sv.generate_vae(dims, randn_torch_cpu, seed))
    return g


def latents(dims, B, h, w, seed):
    from sana_b200 import randn_torch_cpu
    return MG.sv_latents(randn_torch_cpu, B, dims.latent_channels, h, w, seed)


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_vae_small_matches_reference_golden(mode):
    from sana_b200 import synthetic_vae as sv
    g = decoder(mode, sv.SMALL, MG.VAE_SMALL_SEED)
    out = g.vae_decode(latents(sv.SMALL, 2, 4, 6, MG.VAE_SMALL_SEED))
    gold = np.load(os.path.join(GOLDEN, "vae.npz"))["small"]
    e = rel_err(out, gold)
    print(f"vae small {mode}: rel-L2 {e:.3e}")
    assert e < TOL[mode]
    assert g.vae_last_launches() > 10


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_vae_dcae_dims_match_reference_golden(mode):
    """DC-AE f32c32's structure (1024-channel attention levels down to 128-channel ResBlocks)
    at 2 x 2 latents: a 64 x 64 image."""
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims()
    g = decoder(mode, dims, MG.VAE_FULL_SEED)
    out = g.vae_decode(latents(dims, 1, 2, 2, MG.VAE_FULL_SEED))
    gold = np.load(os.path.join(GOLDEN, "vae.npz"))["full_2x2"]
    e, c = rel_err(out, gold), cosine(out, gold)
    print(f"vae dc-ae 2x2 {mode}: rel-L2 {e:.3e} cosine {c:.6f}")
    assert e < TOL[mode] and c > 0.999


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_vae_fresh_structures_match_oracle(mode, oracle):
    """A 3x3 multiscale kernel, attention between ResBlock levels, odd latent sizes."""
    from sana_b200 import randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims(latent_channels=4, out_channels=3, channels=(16, 64, 32), res_blocks=(True, False, True),
                      layers=(2, 1, 1), head_dim=32, ms_kernel=3, scaling_factor=0.7)
    g = decoder(mode, dims, 41)
    lat = latents(dims, 1, 3, 5, 41)
    out = g.vae_decode(lat)
    want = oracle.vae_decode(dims, sv.generate_vae(dims, randn_torch_cpu, 41), lat)
    e = rel_err(out, want)
    print(f"vae fresh {mode}: rel-L2 {e:.3e}")
    assert e < TOL[mode]


def test_vae_dcae_8x8_matches_oracle(oracle):
    """bf16 product path at 8 x 8 latents (a 256 x 256 image), every level wide enough for
    the tensor-core GEMM tiles."""
    from sana_b200 import randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims()
    g = decoder("bf16", dims, 7)
    lat = latents(dims, 1, 8, 8, 7)
    out = g.vae_decode(lat)
    want = oracle.vae_decode(dims, sv.generate_vae(dims, randn_torch_cpu, 7), lat)
    e, c = rel_err(out, want), cosine(out, want)
    print(f"vae dc-ae 8x8 bf16: rel-L2 {e:.3e} cosine {c:.6f}")
    assert e < TOL["bf16"] and c > 0.999


def test_vae_implicit_convolutions_match_patch_gemm(oracle, monkeypatch):
    """The tensor-core implicit 3x3 convolutions and the sub-pixel upsample convs give the
    same decode as the patch-gather path, and both follow the oracle. 8 x 8 latents through
    64/64/128-channel levels: implicit tiles of 16- and 32-pixel rows, one low-resolution
    grid too small for them (patch path)."""
    from sana_b200 import randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims(latent_channels=8, out_channels=3, channels=(64, 64, 128), res_blocks=(True, True, False),
                      layers=(2, 1, 1), head_dim=32, ms_kernel=5, scaling_factor=0.5)
    g = decoder("bf16", dims, 11)
    lat = latents(dims, 2, 8, 8, 11)
    implicit = g.vae_decode(lat)
    monkeypatch.setenv("SANA_VAE_CONV", "im2col")
    patch = g.vae_decode(lat)
    monkeypatch.delenv("SANA_VAE_CONV")
    want = oracle.vae_decode(dims, sv.generate_vae(dims, randn_torch_cpu, 11), lat)
    e1, e2, c = rel_err(implicit, want), rel_err(patch, want), cosine(implicit, patch)
    print(f"vae implicit vs oracle {e1:.3e}, patch vs oracle {e2:.3e}, implicit vs patch cosine {c:.7f}")
    assert e1 < TOL["bf16"] and e2 < TOL["bf16"] and c > 0.9999


def test_vae_pixel_pair_convolutions_match_single_pixel_rows(monkeypatch):
    """The 64- and 128-channel levels run their 3x3 and sub-pixel convolutions with two pixels
    per product row (zero taps padding each pixel's kernel); the single-pixel rows give the
    same decode."""
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims(latent_channels=8, out_channels=3, channels=(64, 64, 128), res_blocks=(True, True, False),
                      layers=(2, 1, 1), head_dim=32, ms_kernel=5, scaling_factor=0.5)
    g = decoder("bf16", dims, 12)
    lat = latents(dims, 2, 8, 8, 12)
    pairs = g.vae_decode(lat)
    monkeypatch.setenv("SANA_VAE_PAIR", "0")
    single = g.vae_decode(lat)
    c = cosine(pairs, single)
    print(f"vae pixel pairs vs single rows: cosine {c:.8f}, identical {np.array_equal(pairs, single)}")
    assert c > 0.99999


def test_vae_batch_images_are_independent():
    from sana_b200 import synthetic_vae as sv
    g = decoder("bf16", sv.SMALL, 5)
    lat = latents(sv.SMALL, 3, 4, 4, 5)
    both = g.vae_decode(lat)
    for i in range(3):
        one = g.vae_decode(lat[i:i + 1])
        assert cosine(both[i], one[0]) > 0.99999


def test_vae_1024_image_is_deterministic_and_finite():
    """Sana's image size: 32 x 32 latents through DC-AE f32c32 -> 1024 x 1024 RGB."""
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims()
    g = decoder("bf16", dims, 3)
    lat = latents(dims, 1, 32, 32, 3)
    a = g.vae_decode(lat)
    b = g.vae_decode(lat)
    assert a.shape == (1, 3, 1024, 1024)
    assert np.isfinite(a).all() and float(np.std(a)) > 1e-3
    assert np.array_equal(a, b)


def test_vae_1024_implicit_matches_patch_gemm(monkeypatch):
    """At Sana's size every 3x3 and upsample conv takes the implicit tensor-core path; the
    patch-gather path computes the same image."""
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims()
    g = decoder("bf16", dims, 3)
    lat = latents(dims, 1, 32, 32, 3)
    a = g.vae_decode(lat)
    monkeypatch.setenv("SANA_VAE_CONV", "im2col")
    b = g.vae_decode(lat)
    c = cosine(a, b)
    print(f"vae 1024 implicit vs patch: cosine {c:.7f} rel-L2 {rel_err(a, b):.3e}")
    assert c > 0.9999


def test_vae_argument_errors():
    from sana_b200 import SANA_MODE_BF16, SanaCuda, SanaError, randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    g = SanaCuda(0, SANA_MODE_BF16)
    with pytest.raises(SanaError):
        g.vae_dims = sv.SMALL
        g.vae_decode(latents(sv.SMALL, 1, 2, 2, 1))  # no weights uploaded
    bad = sv.VaeDims(latent_channels=8, channels=(16, 32, 64), res_blocks=(True, True, False), layers=(1, 1, 1),
                     head_dim=16)
    with pytest.raises(ValueError, match="head dim"):
        g.vae_upload(bad, sv.generate_vae(bad, randn_torch_cpu, 1))
    bad = sv.VaeDims(latent_channels=6, channels=(16, 32, 64), res_blocks=(True, True, False), layers=(1, 1, 1))
    with pytest.raises(ValueError, match="divisible by latent channels"):
        g.vae_upload(bad, sv.generate_vae(bad, randn_torch_cpu, 1))


def test_vae_gguf_upload_matches_pointer_upload(tmp_path):
    """vae_decoder_weights.gguf written under the reference's names loads into the same decoder
    as the pointer table (load_vae_weights' structure discovery, vae.cpp:64-170)."""
    from sana_b200 import SANA_MODE_BF16, SanaCuda, randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    from sana_b200.gguf_files import write_vae_gguf
    dims = sv.VaeDims(latent_channels=8, out_channels=3, channels=(16, 32, 64), res_blocks=(True, True, False),
                      layers=(3, 3, 3), head_dim=32, ms_kernel=5, scaling_factor=0.41407)
    tensors = sv.generate_vae(dims, randn_torch_cpu, 13)
    path = write_vae_gguf(dims, tensors, str(tmp_path / "vae_decoder_weights.gguf"))
    lat = latents(dims, 1, 4, 4, 13)
    a = SanaCuda(0, SANA_MODE_BF16)
    a.vae_upload(dims, tensors)
    b = SanaCuda(0, SANA_MODE_BF16)
    got = b.vae_upload_gguf(path, 0.41407)
    import dataclasses
    assert abs(got.scaling_factor - dims.scaling_factor) < 1e-7
    assert dataclasses.replace(got, scaling_factor=dims.scaling_factor) == dims
    assert np.array_equal(a.vae_decode(lat), b.vae_decode(lat))


def test_vae_gguf_errors_follow_the_loader(tmp_path):
    from sana_b200 import SANA_MODE_BF16, SanaCuda, SanaError, randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    from sana_b200.gguf_files import _write
    dims = sv.VaeDims(latent_channels=8, out_channels=3, channels=(16, 32, 64), res_blocks=(True, True, False),
                      layers=(3, 3, 3))
    specs = sv.vae_tensor_specs(dims)
    tensors = sv.generate_vae(dims, randn_torch_cpu, 2)
    g = SanaCuda(0, SANA_MODE_BF16)
    missing = str(tmp_path / "missing.gguf")
    _write(missing, [(n, t) for (n, _, _), t in zip(specs, tensors) if n != "decoder.conv_out.bias"])
    with pytest.raises(ValueError, match="weight name not found"):
        g.vae_upload_gguf(missing)
    bad = str(tmp_path / "bad.gguf")
    _write(bad, [(n, t if n != "decoder.conv_in.bias" else t[:-1]) for (n, _, _), t in zip(specs, tensors)])
    with pytest.raises(SanaError, match="shape"):
        g.vae_upload_gguf(bad)


def test_vae_device_entry_and_batch_on_the_implicit_path():
    """Two images of 16 x 16 latents through DC-AE f32c32 (every level from 128 x 128 up takes
    the implicit tensor-core convolutions and pixel pairs): the device-pointer entry point gives
    the host entry point's image, and each image of the batch is the one it gets alone."""
    import torch
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims()
    g = decoder("bf16", dims, 17)
    lat = latents(dims, 2, 16, 16, 17)
    host = g.vae_decode(lat)
    d_lat = torch.from_numpy(lat).cuda()
    d_out = torch.empty((2, 3, 512, 512), dtype=torch.float32, device="cuda")
    g.vae_decode_device(d_lat.data_ptr(), 2, 16, 16, d_out.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy(), host)
    # alone, an image's linear attention splits its token sums differently (the split depends on
    # the batch), so bf16 roundings differ slightly: the denoiser's batch criterion applies
    for i in range(2):
        one = g.vae_decode(lat[i:i + 1])
        c, e = cosine(host[i], one[0]), rel_err(host[i], one[0])
        print(f"vae batch image {i}: cosine {c:.7f} rel-L2 {e:.2e}")
        assert c > 0.9999 and e < 1e-2, (i, c, e)
