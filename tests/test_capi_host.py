"""The C-ABI library without a GPU: it loads, exports every function include/sana_cuda.h
declares, and its host-only entry points (torch-compatible generator, scheduler schedule)
agree bit-for-bit with the oracle, the reference build and the golden fixtures. Nothing here
launches a kernel."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

HEADER = os.path.join(ROOT, "include", "sana_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sana_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from sana_b200 import load_library
    return load_library()


def test_library_exports_every_declared_function(lib):
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_randn_matches_oracle_and_golden(oracle):
    from sana_b200 import randn_torch_cpu
    g = np.load(os.path.join(GOLDEN, "rng.npz"))
    assert np.array_equal(randn_torch_cpu(17, 3).view(np.uint32), g["r17_3"].view(np.uint32))
    assert np.array_equal(randn_torch_cpu(1000, 42).view(np.uint32), g["r1000_42"].view(np.uint32))
    assert np.array_equal(randn_torch_cpu(100003, 9)[-64:].view(np.uint32), g["r100003_9"].view(np.uint32))
    for n, s in ((16, 0), (1152 * 6 + 7, 12345), (2304, 2**33 + 5)):
        assert np.array_equal(randn_torch_cpu(n, s), oracle.randn(n, s))
    with pytest.raises(ValueError):
        randn_torch_cpu(15, 0)


def test_schedule_matches_golden():
    from sana_b200 import scheduler_schedule
    g = np.load(os.path.join(GOLDEN, "scheduler_20.npz"))
    ts, sg = scheduler_schedule(20, 3.0)
    assert np.array_equal(ts, g["timesteps"]) and np.array_equal(sg, g["sigmas"])
    ts4, sg4 = scheduler_schedule(4, 3.0)  # test_scheduler_main.cpp:27-41
    np.testing.assert_allclose(ts4, [999, 899, 749, 499], atol=1e-3)
    np.testing.assert_allclose(sg4, [0.99966644, 0.89963979, 0.74962479, 0.49966654, 0.0], atol=1e-6)
    with pytest.raises(ValueError):
        scheduler_schedule(0)


def test_schedule_matches_reference_build(reference):
    from sana_b200 import scheduler_schedule
    for n, shift in ((1, 3.0), (7, 3.0), (20, 1.0), (50, 4.5)):
        a = scheduler_schedule(n, shift)
        b = reference.scheduler_schedule(n, shift)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_synthetic_weights_use_the_product_generator(oracle):
    """The synthetic checkpoint recipe gives identical tensors whichever generator drives it."""
    from sana_b200 import randn_torch_cpu
    from sana_b200 import synthetic as syn
    d = syn.ModelDims(n_blocks=1, hidden=32, latent_channels=4, caption_dim=24, ff_expanded=64,
                      self_heads=2, cross_heads=2)
    a = syn.generate_model(d, randn_torch_cpu, base_seed=3, bias_std=0.02)
    b = syn.generate_model(d, oracle.randn, base_seed=3, bias_std=0.02)
    assert len(a) == 16 + 19
    for x, y in zip(a, b):
        assert x.shape == y.shape and np.array_equal(x, y)


def test_handle_errors_are_reported_without_a_device(lib):
    """Creating a handle where no device exists returns an error code and a message (no
    crash, no fallback). Skipped where a GPU is present."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from sana_b200 import SanaCuda, SanaError
    with pytest.raises(SanaError):
        SanaCuda(0)
    assert lib.sana_cuda_synchronize(None) == 1
