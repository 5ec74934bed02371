"""GGUF weight files (the reference's model/caption/denoiser_weights.gguf, weights_io.cpp:134-164,
325-377): the library's own reader against files written by the ``gguf`` package (llama.cpp's
writer, the one the reference's loader comment names), and its failure modes. No GPU: the
reader is host code of libsana_cuda.so."""
import os
import struct

import numpy as np
import pytest

from sana_b200 import SanaError, gguf_index


def _write(path, tensors, kv=None, alignment=None):
    gguf = pytest.importorskip("gguf")
    w = gguf.GGUFWriter(path, arch="sana")
    if alignment:
        w.add_custom_alignment(alignment)
    for k, (kind, v) in (kv or {}).items():
        getattr(w, "add_" + kind)(k, v)
    for name, arr in tensors:
        w.add_tensor(name, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_reader_matches_the_gguf_writer(tmp_path):
    rng = np.random.default_rng(0)
    tensors = [("a.weight", rng.standard_normal((7, 5)).astype(np.float32)),
               ("a.bias", rng.standard_normal(7).astype(np.float32)),
               ("conv.weight", rng.standard_normal((6, 3, 3, 3)).astype(np.float32)),
               ("table", rng.standard_normal((2, 9)).astype(np.float32)),
               ("half", rng.standard_normal((4, 8)).astype(np.float16))]
    kv = {"general.name": ("string", "sana test"), "x.count": ("uint32", 7), "x.big": ("uint64", 1 << 40),
          "x.neg": ("int64", -3), "x.f": ("float32", 0.5), "x.d": ("float64", 0.25), "x.flag": ("bool", True),
          "x.names": ("array", ["q", "k", "v"]), "x.nums": ("array", [1, 2, 3]),
          "x.nested": ("array", [[1, 2], [3]])}
    path = str(tmp_path / "w.gguf")
    _write(path, tensors, kv)
    idx = gguf_index(path)
    assert list(idx) == [n for n, _ in tensors]
    for name, arr in tensors:
        typ, shape, data = idx[name]
        assert shape == arr.shape
        assert typ == (1 if arr.dtype == np.float16 else 0)
        assert np.array_equal(data, arr)


@pytest.mark.parametrize("alignment", [32, 64, 256])
def test_reader_honours_alignment(tmp_path, alignment):
    rng = np.random.default_rng(alignment)
    tensors = [(f"t{i}", rng.standard_normal(n).astype(np.float32)) for i, n in enumerate((3, 17, 64, 5))]
    path = str(tmp_path / "a.gguf")
    _write(path, tensors, alignment=alignment)
    idx = gguf_index(path)
    for name, arr in tensors:
        assert np.array_equal(idx[name][2], arr)


def test_reader_agrees_with_gguf_reader(tmp_path):
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(1)
    tensors = [(f"blk.{i}.w", rng.standard_normal((3 + i, 2 * i + 1)).astype(np.float32)) for i in range(6)]
    path = str(tmp_path / "r.gguf")
    _write(path, tensors)
    theirs = {t.name: np.asarray(t.data) for t in gguf.GGUFReader(path).tensors}
    ours = gguf_index(path)
    assert set(theirs) == set(ours)
    for name, arr in theirs.items():
        assert np.array_equal(ours[name][2].reshape(-1), arr.reshape(-1))


def test_reader_rejects_malformed_files(tmp_path):
    path = str(tmp_path / "ok.gguf")
    _write(path, [("w", np.ones((4, 4), np.float32))])
    raw = open(path, "rb").read()
    bad_magic = str(tmp_path / "magic.gguf")
    open(bad_magic, "wb").write(b"GGUX" + raw[4:])
    with pytest.raises(SanaError, match="bad magic"):
        gguf_index(bad_magic)
    bad_version = str(tmp_path / "version.gguf")
    open(bad_version, "wb").write(raw[:4] + struct.pack("<I", 9) + raw[8:])
    with pytest.raises(SanaError, match="unsupported version"):
        gguf_index(bad_version)
    truncated = str(tmp_path / "short.gguf")
    open(truncated, "wb").write(raw[: len(raw) - 8])
    with pytest.raises(SanaError, match="past the end|truncated"):
        gguf_index(truncated)
    with pytest.raises(SanaError, match="failed to open"):
        gguf_index(str(tmp_path / "missing.gguf"))


def test_checkpoint_writer_uses_the_reference_names(tmp_path):
    from sana_b200 import synthetic as syn
    from sana_b200.gguf_files import write_checkpoint_gguf
    d = syn.ModelDims(n_blocks=2, hidden=64, latent_channels=8, caption_dim=48, ff_expanded=160, self_heads=2,
                      cross_heads=2)
    specs = syn.model_tensor_specs(d)
    tensors = [np.full(s, i, np.float32) for i, (_, s, _) in enumerate(specs)]
    paths = write_checkpoint_gguf(tensors, d.n_blocks, str(tmp_path))
    names = set()
    for p in paths.values():
        names |= set(gguf_index(p))
    assert names == {n for n, _, _ in specs}
    blocks = gguf_index(paths["model"])
    assert blocks["transformer_blocks.1.ff.conv_point.weight"][1] == (64, 80, 1, 1)
