"""The C-ABI library without a GPU: it loads, exports every function include/sana_cuda.h
declares, and its host-only entry points (torch-compatible generator, scheduler schedule)
agree bit-for-bit with the oracle, the reference build and the golden fixtures. Nothing here
launches a kernel."""
import ctypes
import os
import re
import types

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


def test_schedule_configs_match_reference_build():
    """build_sana_scheduler_timesteps for other configs (num_train_timesteps, flow_shift,
    solver settings) bit for bit against the reference's schedules, and its refusals."""
    from sana_b200 import scheduler_schedule_config
    from test_oracle_pin import scheduler_cases
    n_checked = 0
    for cfg, _, _, explicit, want in scheduler_cases():
        if explicit is not None:
            continue
        ts, sg = scheduler_schedule_config(len(want["ts"]), **cfg)
        assert np.array_equal(ts, want["ts"]) and np.array_equal(sg.view(np.uint32), want["sg"].view(np.uint32)), cfg
        n_checked += 1
    assert n_checked >= 8
    for bad in ({"solver_order": 0}, {"solver_order": 3}, {"use_flow_sigmas": 0}, {"final_sigmas_zero": 0},
                {"num_train_timesteps": 0}):
        with pytest.raises(ValueError):
            scheduler_schedule_config(4, **bad)
    with pytest.raises(ValueError):
        scheduler_schedule_config(0)


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


# --- the text-encoder output contract (host functions; gemma_encoder.cpp:51-77,177-244) ----

@pytest.mark.parametrize("case", ["kat_select_rows_first_and_last", "kat_prompt_pair"])
def test_encoder_contract_kats(case):
    import kat_cases as K
    import sana_b200
    K.check(getattr(K, case)(sana_b200))


@pytest.mark.parametrize("neg_real,pos_rows,pos_real,L", [
    (8, 324, 40, 300),     # the encoder's shapes: 26-token instruction prefix + 300 - 2
    (0, 300, 0, 300),      # empty prompts: no real token at all
    (300, 300, 300, 300),  # every row real, no slice
    (1, 9, 9, 3),          # tail fully real
    (2, 12, 7, 5),         # real tokens end before the kept tail
])
def test_prompt_pair_matches_oracle(oracle, neg_real, pos_rows, pos_real, L):
    from sana_b200 import prompt_pair_assemble
    rng = np.random.default_rng(pos_rows * 7 + L)
    hidden = 24
    neg = rng.standard_normal((L, hidden)).astype(np.float32)
    pos = rng.standard_normal((pos_rows, hidden)).astype(np.float32)
    e1, b1 = prompt_pair_assemble(neg, neg_real, pos, pos_real, L)
    e2, b2 = oracle.prompt_pair_assemble(neg, neg_real, pos, pos_real, L)
    assert np.array_equal(e1.view(np.uint32), e2.view(np.uint32))
    assert np.array_equal(b1.view(np.uint32), b2.view(np.uint32))
    assert np.array_equal(e1[0], neg) and np.array_equal(e1[1, 0], pos[0])
    assert np.array_equal(e1[1, 1:], pos[pos_rows - (L - 1):])


@pytest.mark.parametrize("bad", ["keep0", "keep_gt_rows", "neg_rows", "neg_real", "pos_real", "pos_short"])
def test_encoder_contract_errors(oracle, bad):
    from sana_b200 import prompt_pair_assemble, select_rows_first_and_last
    x = np.zeros((10, 2), np.float32)
    neg, pos = np.zeros((4, 2), np.float32), np.zeros((7, 2), np.float32)
    calls = {
        "keep0": (lambda m: m.select_rows_first_and_last(x, 0), "keep must be in"),
        "keep_gt_rows": (lambda m: m.select_rows_first_and_last(x, 11), "keep must be in"),
        "neg_rows": (lambda m: m.prompt_pair_assemble(np.zeros((5, 2), np.float32), 1, pos, 1, 4), "padded"),
        "neg_real": (lambda m: m.prompt_pair_assemble(neg, 5, pos, 1, 4), "exceeds padded_length"),
        "pos_real": (lambda m: m.prompt_pair_assemble(neg, 1, pos, 8, 4), "exceeds padded_length"),
        "pos_short": (lambda m: m.prompt_pair_assemble(neg, 1, pos[:3], 1, 4), "keep must be in"),
    }
    fn, msg = calls[bad]
    lib = types.SimpleNamespace(select_rows_first_and_last=select_rows_first_and_last,
                                prompt_pair_assemble=prompt_pair_assemble)
    for impl in (lib, oracle):
        with pytest.raises(ValueError, match=msg):
            fn(impl)
