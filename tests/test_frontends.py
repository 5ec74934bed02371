"""The reference's own front ends on this host layer.

* ``tests/bench_full_pipeline.cpp`` and ``src/infer_main.cpp`` of the reference, compiled
  unmodified against host/include and lib/libsana_shim.so + lib/libsana_frontend.so
  (sana.cpp_b200/build.py build_reference_frontends; the executables travel in lib/);
* the loaders they call (load_weight_index, load_denoiser_weights, load_vae_weights: the
  reference's transformer.cpp:166-488, vae.cpp:12-160, weights_io.cpp) through
  tests/cpp/test_frontend.cpp, against the GGUF files the test writes;
* the npy reader / writer and the JSON index of weights_io.h, the encoder stand-in's contract
  (gemma_encoder.cpp:156-244) and the error messages of all of these.

On the GPU: the unmodified benchmark prints its timing summary, and the unmodified CLI writes an
image equal to the Python API's decode of the same conditioning.
"""
import os
import shutil
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, reference_root

PKG = os.path.join(ROOT, "sana.cpp_b200")
LIB = os.path.join(PKG, "lib")
GEMMA_REL = os.path.join("gemma2_text_encoder", "gemma-2-2b-it-f32.gguf")


def _pkg_build():
    if PKG not in sys.path:
        sys.path.insert(0, PKG)
    import build as pkg_build  # sana.cpp_b200/build.py
    return pkg_build


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    b = _pkg_build()
    if not (os.path.exists(b.SHIM_SO) and os.path.exists(b.FRONTEND_SO)):
        b.build_shim()
        b.build_frontend()
    out = str(tmp_path_factory.mktemp("frontend") / "test_frontend")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(PKG, "host", "include"), os.path.join(ROOT, "tests", "cpp", "test_frontend.cpp"),
           os.path.join(PKG, "host", "tensor.cpp"), "-L", LIB, "-lsana_shim", "-lsana_frontend", "-lsana_cuda",
           f"-Wl,-rpath,{LIB}", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "warning" not in r.stderr, r.stderr
    return out


def call(driver, *args):
    r = subprocess.run([driver, *map(str, args)], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout.strip()


@pytest.fixture(scope="module")
def frontends():
    """{name: executable} of the reference's front ends built against this host layer."""
    b = _pkg_build()
    exes = {name: os.path.join(LIB, name) for name in b.REFERENCE_FRONTENDS.values()}
    if all(os.path.exists(e) for e in exes.values()):
        return exes
    ref = reference_root()
    if not ref or not os.path.isdir(os.path.join(ref, "src")):
        pytest.skip("reference front ends not built and the reference tree is absent")
    built = b.build_reference_frontends(ref)
    return {b.REFERENCE_FRONTENDS[k]: v for k, v in built.items()}


# --- loaders -------------------------------------------------------------------------------

SMALL_MODEL = dict(n_blocks=12, hidden=64, latent_channels=8, caption_dim=48, ff_expanded=160, self_heads=4,
                   cross_heads=2)


def _write_model(directory, d, seed=3, bias_std=0.05):
    from sana_b200 import gguf_files, randn_torch_cpu
    from sana_b200 import synthetic as syn
    tensors = syn.generate_model(d, randn_torch_cpu, base_seed=seed, bias_std=bias_std)
    return tensors, gguf_files.write_checkpoint_gguf(tensors, d.n_blocks, str(directory))


def test_denoiser_loader_matches_the_files(driver, tmp_path):
    pytest.importorskip("gguf")
    from sana_b200 import synthetic as syn
    d = syn.ModelDims(**SMALL_MODEL)
    tensors, paths = _write_model(tmp_path / "w", d)
    out = tmp_path / "out"
    out.mkdir()
    msg = call(driver, "denoiser", paths["model"], paths["caption"], paths["denoiser"], d.self_heads, d.cross_heads, out)
    assert msg == "", msg
    meta = (out / "meta.txt").read_text().split("\n")
    assert int(meta[0]) == d.n_blocks
    assert all(line == f"{d.self_heads} {d.cross_heads}" for line in meta[1:1 + d.n_blocks])

    def got(name):
        return np.load(out / f"{name}.npy")

    def linear(t):  # load_linear_weight_tensor: [out, in] -> [in, out]
        return t.T

    model = dict(zip([n for n, _ in syn.MODEL_TENSORS], tensors[:16]))
    np.testing.assert_array_equal(got("caption.linear_1_weight"), linear(model["caption_projection.linear_1.weight"]))
    np.testing.assert_array_equal(got("caption.linear_2_bias"), model["caption_projection.linear_2.bias"])
    np.testing.assert_array_equal(got("patch_embed_weight"), model["patch_embed.proj.weight"])
    np.testing.assert_array_equal(got("time_embed_linear_1_weight"),
                                  linear(model["time_embed.emb.timestep_embedder.linear_1.weight"]))
    np.testing.assert_array_equal(got("time_projection_weight"), linear(model["time_embed.linear.weight"]))
    np.testing.assert_array_equal(got("final_scale_shift_table"), model["scale_shift_table"])
    np.testing.assert_array_equal(got("proj_out_weight"), linear(model["proj_out.weight"]))
    # blocks in numeric order (10 and 11 after 9), linear weights transposed, zero q/k/v biases
    # and unit / zero norm affines filled in
    for i in range(d.n_blocks):
        blk = dict(zip([n for n, _ in syn.BLOCK_TENSORS], tensors[16 + 19 * i:16 + 19 * (i + 1)]))
        p = f"blocks.{i}."
        np.testing.assert_array_equal(got(p + "scale_shift_table"), blk["scale_shift_table"])
        np.testing.assert_array_equal(got(p + "q_weight"), linear(blk["attn1.to_q.weight"]))
        np.testing.assert_array_equal(got(p + "cross_v_weight"), linear(blk["attn2.to_v.weight"]))
        np.testing.assert_array_equal(got(p + "cross_k_bias"), blk["attn2.to_k.bias"])
        np.testing.assert_array_equal(got(p + "ff_depth_weight"), blk["ff.conv_depth.weight"])
        np.testing.assert_array_equal(got(p + "ff_point_weight"), blk["ff.conv_point.weight"])
        np.testing.assert_array_equal(got(p + "q_bias"), np.zeros(d.hidden, np.float32))
        np.testing.assert_array_equal(got(p + "attn_norm_gamma"), np.ones(d.hidden, np.float32))
        np.testing.assert_array_equal(got(p + "mlp_norm_beta"), np.zeros(d.hidden, np.float32))


def test_denoiser_loader_errors(driver, tmp_path):
    pytest.importorskip("gguf")
    from sana_b200 import gguf_files
    from sana_b200 import synthetic as syn
    d = syn.ModelDims(**dict(SMALL_MODEL, n_blocks=2))
    tensors, paths = _write_model(tmp_path / "w", d)
    args = ["denoiser", paths["model"], paths["caption"], paths["denoiser"]]
    assert call(driver, *args, 0, 2, tmp_path) == "invalid_argument: self_num_heads must be greater than 0"
    assert call(driver, *args, 5, 2, tmp_path) == \
        "runtime_error: self attention hidden size must be divisible by self_num_heads"
    # the caption file has no blocks; a missing tensor; an unreadable file
    assert call(driver, "denoiser", paths["caption"], paths["caption"], paths["denoiser"], 4, 2, tmp_path) == \
        "invalid_argument: weight index does not contain any prefixed model blocks"
    assert call(driver, "denoiser", paths["model"], paths["denoiser"], paths["denoiser"], 4, 2, tmp_path) == \
        "invalid_argument: weight name not found in weight index"
    missing = str(tmp_path / "absent.gguf")
    assert call(driver, "denoiser", missing, paths["caption"], paths["denoiser"], 4, 2, tmp_path) == \
        f"runtime_error: failed to open gguf weight file: {missing}"
    # a caption projection whose output width is not the blocks' hidden size
    bad = list(tensors)
    wide = d.hidden + 8
    bad[0:4] = [np.zeros((wide, d.caption_dim), np.float32), np.zeros(wide, np.float32),
                np.zeros((wide, wide), np.float32), np.zeros(wide, np.float32)]
    bad_paths = gguf_files.write_checkpoint_gguf(bad, d.n_blocks, str(tmp_path / "bad"))
    assert call(driver, "denoiser", paths["model"], bad_paths["caption"], paths["denoiser"], 4, 2, tmp_path) == \
        "invalid_argument: caption output hidden size must match model block hidden size"


def test_vae_loader_structure(driver, tmp_path):
    pytest.importorskip("gguf")
    from sana_b200 import gguf_files, randn_torch_cpu
    from sana_b200 import synthetic_vae as sv
    dims = sv.VaeDims(latent_channels=8, channels=(16, 32, 32, 64), res_blocks=(True, True, False, False),
                      layers=(3, 3, 3, 3))
    tensors = sv.generate_vae(dims, randn_torch_cpu, 5)
    path = gguf_files.write_vae_gguf(dims, tensors, str(tmp_path / "vae_decoder_weights.gguf"))
    out = tmp_path / "out"
    out.mkdir()
    assert call(driver, "vae", path, out) == ""
    meta = (out / "meta.txt").read_text().split("\n")
    assert meta[0].split() == ["4", "0.41407", "32"]
    named = {name: t for (name, _, _), t in zip(sv.vae_tensor_specs(dims), tensors)}
    for i in range(dims.n_blocks):
        up, res, n_res, n_attn = map(int, meta[1 + i].split())
        assert up == int(dims.has_upsample(i))
        assert res == int(dims.res_blocks[i])
        assert (n_res, n_attn) == ((3, 0) if dims.res_blocks[i] else (0, 3))
        first = 1 if up else 0
        last = f"decoder.up_blocks.{i}.{first + 2}"
        if up:
            np.testing.assert_array_equal(np.load(out / f"up.{i}.upsample_conv_weight.npy"),
                                          named[f"decoder.up_blocks.{i}.0.conv.weight"])
        if res:
            np.testing.assert_array_equal(np.load(out / f"up.{i}.last.conv2_weight.npy"), named[last + ".conv2.weight"])
        else:
            q = named[last + ".attn.to_q.weight"]
            np.testing.assert_array_equal(np.load(out / f"up.{i}.last.to_q_weight_conv1x1.npy"),
                                          q.reshape(*q.shape, 1, 1))
            np.testing.assert_array_equal(np.load(out / f"up.{i}.last.proj_in_weight.npy"),
                                          named[last + ".attn.to_qkv_multiscale.0.proj_in.weight"])
    np.testing.assert_array_equal(np.load(out / "conv_in_weight.npy"), named["decoder.conv_in.weight"])


# --- weights_io ------------------------------------------------------------------------------

def test_npy_round_trip(driver, tmp_path):
    a = np.random.default_rng(1).standard_normal((3, 5, 7)).astype(np.float32)
    src = tmp_path / "a.npy"
    np.save(src, a)
    assert call(driver, "npy_copy", src, tmp_path / "b.npy") == ""
    raw = (tmp_path / "b.npy").read_bytes()
    header_len = int.from_bytes(raw[8:10], "little")
    assert (10 + header_len) % 16 == 0  # payload on a 16-byte boundary, as numpy writes it
    np.testing.assert_array_equal(np.load(tmp_path / "b.npy"), a)
    # format 2.0 headers, 1-D shapes
    v = np.arange(40, dtype=np.float32)
    with open(tmp_path / "v2.npy", "wb") as f:
        np.lib.format.write_array(f, v, version=(2, 0))
    assert call(driver, "npy_copy", tmp_path / "v2.npy", tmp_path / "v.npy") == ""
    np.testing.assert_array_equal(np.load(tmp_path / "v.npy"), v)
    # the reference's refusals
    np.save(tmp_path / "f64.npy", a.astype(np.float64))
    assert call(driver, "npy_copy", tmp_path / "f64.npy", tmp_path / "x.npy") == \
        "runtime_error: only little-endian float32 npy tensors are supported"
    np.save(tmp_path / "fort.npy", np.asfortranarray(a[0]))
    assert call(driver, "npy_copy", tmp_path / "fort.npy", tmp_path / "x.npy") == \
        "runtime_error: fortran-order npy tensors are not supported"
    (tmp_path / "junk.npy").write_bytes(b"not an npy file")
    assert call(driver, "npy_copy", tmp_path / "junk.npy", tmp_path / "x.npy") == \
        "runtime_error: invalid npy magic header"


def test_json_index_and_linear_weights(driver, tmp_path):
    w = np.random.default_rng(2).standard_normal((6, 4)).astype(np.float32)
    np.save(tmp_path / "w.npy", w)
    (tmp_path / "index.json").write_text(
        '{\n  "lin.weight": {"file": "w.npy", "shape": [6, 4], "dtype": "float32"},\n'
        '  "bad.shape": {"file": "w.npy", "shape": [4, 6], "dtype": "float32"},\n'
        '  "half": {"dtype": "float16", "file": "w.npy", "shape": [6, 4]}\n}\n')
    idx = tmp_path / "index.json"
    assert call(driver, "index_tensor", idx, tmp_path, "lin.weight", tmp_path / "o.npy") == ""
    np.testing.assert_array_equal(np.load(tmp_path / "o.npy"), w)
    assert call(driver, "index_tensor", idx, tmp_path, "lin.weight", tmp_path / "t.npy", "linear") == ""
    np.testing.assert_array_equal(np.load(tmp_path / "t.npy"), w.T)
    assert call(driver, "index_tensor", idx, tmp_path, "bad.shape", tmp_path / "x.npy") == \
        "runtime_error: loaded weight tensor shape does not match index metadata"
    assert call(driver, "index_tensor", idx, tmp_path, "half", tmp_path / "x.npy") == \
        "runtime_error: only float32 saved weights are supported"
    assert call(driver, "index_tensor", idx, tmp_path, "nope", tmp_path / "x.npy") == \
        "invalid_argument: weight name not found in weight index"
    (tmp_path / "bad.json").write_text('{"a": {"file": "w.npy", "size": 3}}')
    assert call(driver, "index_tensor", tmp_path / "bad.json", tmp_path, "a", tmp_path / "x.npy") == \
        "runtime_error: unexpected field in weight index"
    (tmp_path / "empty.json").write_text("{ }")
    assert call(driver, "index_tensor", tmp_path / "empty.json", tmp_path, "a", tmp_path / "x.npy") == \
        "invalid_argument: weight name not found in weight index"


def test_gguf_index_refuses_half_tensors(driver, tmp_path):
    gguf = pytest.importorskip("gguf")
    path = str(tmp_path / "h.gguf")
    wr = gguf.GGUFWriter(path, arch="sana")
    wr.add_tensor("h", np.ones((4, 8), np.float16))
    wr.add_tensor("f", np.arange(12, dtype=np.float32).reshape(3, 4))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    assert call(driver, "index_tensor", path, "", "h", tmp_path / "x.npy") == \
        "runtime_error: only float32 saved weights are supported"
    assert call(driver, "index_tensor", path, "", "f", tmp_path / "f.npy") == ""
    np.testing.assert_array_equal(np.load(tmp_path / "f.npy"), np.arange(12, dtype=np.float32).reshape(3, 4))


# --- the encoder stand-in's contract -----------------------------------------------------------

def test_prompt_pair_contract(driver, tmp_path):
    gemma = tmp_path / "gemma.gguf"
    gemma.write_bytes(b"stand-in")
    out = tmp_path / "p"
    out.mkdir()
    assert call(driver, "prompt", "a house by the lake", "", 300, gemma, out) == ""
    emb, bias = np.load(out / "embeddings.npy"), np.load(out / "bias.npy")
    assert emb.shape == (2, 300, 2304) and bias.shape == (2, 1, 300)
    # negative: the beginning token only; positive: 24 prefix tokens + 5 words, cut to row 0 and
    # the last 299 of its 322 rows (rows 23..321), of which rows 23..28 are real
    assert (bias[0, 0] == 0).sum() == 1 and (bias[1, 0] == 0).sum() == 1 + 6
    assert set(np.unique(bias)) <= {0.0, -10000.0}
    assert np.isfinite(emb).all() and abs(float(emb.std()) - 1.0) < 0.01
    again = tmp_path / "q"
    again.mkdir()
    assert call(driver, "prompt", "a house by the lake", "", 300, gemma, again) == ""
    np.testing.assert_array_equal(np.load(again / "embeddings.npy"), emb)
    assert call(driver, "prompt", "a house by the lake", "", 300, tmp_path / "absent.gguf", out) == \
        f"runtime_error: failed to load Gemma-2 GGUF: {tmp_path / 'absent.gguf'}"
    long_prompt = " ".join(["word"] * 400)
    assert call(driver, "prompt", long_prompt, "", 300, gemma, out) == \
        "invalid_argument: tokenized text exceeds padded_length; truncation not implemented"
    # a zero-length sequence: the positive text cannot fit its padded length (prefix + L - 2)
    assert call(driver, "prompt", "x", "", 0, gemma, out) == \
        "invalid_argument: tokenized text exceeds padded_length; truncation not implemented"


def test_select_rows_first_and_last(driver, tmp_path):
    a = np.arange(10 * 3, dtype=np.float32).reshape(10, 3)
    np.save(tmp_path / "a.npy", a)
    assert call(driver, "select", tmp_path / "a.npy", 4, tmp_path / "s.npy") == ""
    np.testing.assert_array_equal(np.load(tmp_path / "s.npy"), a[[0, 7, 8, 9]])
    assert call(driver, "select", tmp_path / "a.npy", 11, tmp_path / "s.npy") == \
        "invalid_argument: select_rows_first_and_last: keep must be in (0, rows]"


# --- the reference's front ends ------------------------------------------------------------------

def test_reference_frontends_built_unmodified(frontends, tmp_path):
    r = subprocess.run([frontends["sana_infer"], "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.startswith("Usage:"), r.stdout + r.stderr
    # no weights: both stop where the reference stops, at the text encoder's model file
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([frontends["sana_infer"], "--prompt", "x"], capture_output=True, text=True, timeout=60,
                       cwd=tmp_path, env=env)
    assert r.returncode == 1
    assert "Error: failed to load Gemma-2 GGUF: ../weights/gemma2_text_encoder/gemma-2-2b-it-f32.gguf" in r.stderr
    r = subprocess.run([frontends["sana_infer"], "--bogus"], capture_output=True, text=True, timeout=60,
                       cwd=tmp_path, env=env)
    assert r.returncode == 1 and "Error: unknown option: --bogus" in r.stderr


# Test model for the GPU runs: the real widths (hidden 1152, 36 / 16 heads, which the front ends
# hard-code; caption 2304; 32 latent channels at 32x32) with 2 blocks, and a narrow six-block VAE
# (x32 upsampling to the 1024x1024 image the front ends ask for).
FRONTEND_BLOCKS = 2


def _frontend_weights(root, n_blocks=FRONTEND_BLOCKS):
    from sana_b200 import gguf_files, randn_torch_cpu
    from sana_b200 import synthetic as syn
    from sana_b200 import synthetic_vae as sv
    weights = root / "weights"
    d = syn.ModelDims(n_blocks=n_blocks)
    tensors = syn.generate_model(d, randn_torch_cpu, base_seed=11, bias_std=0.02)
    paths = gguf_files.write_checkpoint_gguf(tensors, d.n_blocks, str(weights))
    del tensors
    vd = sv.VaeDims(channels=(16, 32, 32, 64, 64, 128), layers=(3,) * 6)
    paths["vae"] = gguf_files.write_vae_gguf(vd, sv.generate_vae(vd, randn_torch_cpu, 12),
                                             str(weights / "vae_decoder_weights.gguf"))
    (weights / GEMMA_REL).parent.mkdir(parents=True)
    (weights / GEMMA_REL).write_bytes(b"the text-encoder stand-in only opens this file")
    run = root / "run"
    run.mkdir()
    return paths, run


@pytest.mark.gpu
def test_reference_bench_full_pipeline_runs(frontends, tmp_path):
    pytest.importorskip("gguf")
    _, run = _frontend_weights(tmp_path)
    r = subprocess.run([frontends["bench_full_pipeline"], "1", "2"], capture_output=True, text=True, timeout=900,
                       cwd=run)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    summary = dict(line.split(":", 1) for line in r.stdout.split("=== timing summary ===")[1].strip().split("\n"))
    assert int(summary["iters"]) == 2
    assert float(summary["transformer_ms_avg"].split()[0]) > 0
    assert float(summary["vae_ms_avg"]) > 0


def _read_ppm(path):
    raw = open(path, "rb").read()
    magic, dims, maxval, rest = raw.split(b"\n", 3)
    assert magic == b"P6" and maxval == b"255"
    w, h = map(int, dims.split())
    return np.frombuffer(rest, np.uint8).reshape(h, w, 3)


@pytest.mark.gpu
def test_reference_infer_matches_python_api(frontends, tmp_path):
    pytest.importorskip("gguf")
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    paths, run = _frontend_weights(tmp_path)
    steps = 4
    r = subprocess.run([frontends["sana_infer"], "--weights-dir", "../weights", "--prompt", "a house by the lake",
                        "--steps", str(steps), "--output", "out.ppm"], capture_output=True, text=True, timeout=900,
                       cwd=run)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    image = _read_ppm(run / "out.ppm")
    assert image.shape == (1024, 1024, 3)

    cond = run / ".sana_conditioning" / "out_seed42"
    enc = np.load(cond / "caption_projection_input.npy")
    bias = np.load(cond / "encoder_attention_mask.npy")
    lat = np.load(cond / "initial_latent.npy")
    assert enc.shape == (2, 300, 2304) and bias.shape == (2, 1, 300) and lat.shape == (1, 32, 32, 32)
    g = SanaCuda(0, SANA_MODE_BF16)
    g.upload_gguf(paths["model"], paths["caption"], paths["denoiser"], 36, 16)
    g.vae_upload_gguf(paths["vae"], 0.41407)
    decoded = g.vae_decode(g.denoise_loop(lat, enc, bias, 4.5, steps))
    want = np.round(np.clip(decoded[0] * 0.5 + 0.5, 0.0, 1.0) * 255.0).astype(np.uint8).transpose(1, 2, 0)
    diff = np.abs(image.astype(np.int32) - want.astype(np.int32))
    print(f"sana_infer vs Python API: max {diff.max()} levels, mean {diff.mean():.4f}")
    assert diff.max() <= 2 and diff.mean() < 0.05
