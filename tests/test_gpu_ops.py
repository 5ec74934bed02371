"""CUDA path, single operations, through the C ABI (include/sana_cuda.h).

* the tcgen05 tensor-core GEMM against float64 products of the same bf16-rounded
  operands (only accumulation error remains), and the CUDA-core GEMM in fp32;
* the reference's own known-answer tests in the fp32 check mode (reference tolerances);
* every op against the golden fixtures the compiled reference produced
  (fp32 check mode: relative L2 <= 1e-5; bf16 mode: <= 2e-2);
* edge cases of the reference's op contracts against the oracle.
"""
import ctypes
import importlib.util
import os

import numpy as np
import pytest

import kat_cases as K
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
MG = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(MG)

F32_TOL = 1e-5   # fp32 check mode, relative L2 to the reference
BF16_TOL = 2e-2  # bf16 operands / activations, fp32 accumulation


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_round(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def gpu_f32():
    from sana_b200 import SANA_MODE_F32, SanaCuda
    return SanaCuda(0, SANA_MODE_F32)


@pytest.fixture(scope="module")
def gpu_bf16():
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    return SanaCuda(0, SANA_MODE_BF16)


# --- GEMM -----------------------------------------------------------------------------------
GEMM_SHAPES = [(128, 64, 128), (256, 128, 256), (300, 136, 200), (1, 64, 32), (77, 1152, 16), (640, 512, 1152),
               (2048, 1152, 3456), (1000, 2880, 1152), (517, 2304, 1152), (2048, 1152, 5760)]


@pytest.mark.parametrize("M,K,N", GEMM_SHAPES)
def test_tensor_core_gemm(gpu_bf16, M, K, N):
    from sana_b200 import gemm_counts
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    tc0, _ = gemm_counts()
    out = gpu_bf16.linear_3d(x, w, b)
    tc1, _ = gemm_counts()
    assert tc1 == tc0 + 1, "the tensor-core path did not run"
    ref = bf16_round(x).astype(np.float64) @ bf16_round(w).astype(np.float64) + b
    assert rel_err(out, ref) < 1e-5 + 2e-6 * np.sqrt(K)


@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (3, 5, 7), (64, 64, 64), (130, 300, 70), (512, 1152, 1152)])
def test_cuda_core_gemm_fp32(gpu_f32, M, K, N):
    from sana_b200 import gemm_counts
    rng = np.random.default_rng(M + K + N)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((K, N)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    _, s0 = gemm_counts()
    out = gpu_f32.linear_3d(x, w, b)
    _, s1 = gemm_counts()
    assert s1 == s0 + 1
    ref = x.astype(np.float64) @ w.astype(np.float64) + b
    assert rel_err(out, ref) < 1e-6


@pytest.mark.parametrize("act", [1, 2], ids=["silu", "gelu_tanh"])
def test_gemm_activation_epilogue(gpu_bf16, act):
    """Bias + SiLU / GELU-tanh fused into the tensor-core epilogue (the FF-inverted and
    caption projections), over pre-activations from -120 to 120: every bf16 output within
    its own rounding (2^-8 relative) of the float64 activation of the same bf16 product."""
    import torch
    M, K, N = 256, 64, 384
    rng = np.random.default_rng(act)
    x = bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    w = bf16_round((rng.standard_normal((N, K)) * 0.3).astype(np.float32))
    b = np.linspace(-120, 120, N).astype(np.float32)
    pre = x.astype(np.float64) @ w.astype(np.float64).T + b
    if act == 1:
        ref = pre / (1 + np.exp(-pre))
    else:
        ref = 0.5 * pre * (1 + np.tanh(np.sqrt(2 / np.pi) * (pre + 0.044715 * pre ** 3)))
    A = torch.from_numpy(x).to("cuda", torch.bfloat16)
    B = torch.from_numpy(w).to("cuda", torch.bfloat16)
    bias = torch.from_numpy(b).cuda()
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    gpu_bf16.gemm_device(A.data_ptr(), B.data_ptr(), M, N, K, out.data_ptr(), bias.data_ptr(), act)
    gpu_bf16.synchronize()
    got = out.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - ref)
    bound = 2.0 ** -8 * np.abs(ref) + 1e-6
    assert (err <= bound).all(), float((err / bound).max())


def test_silu_epilogue_fp32_accuracy(gpu_bf16):
    """The tensor-core SiLU epilogue at full precision: pre-activations x in [-80, 80] (bf16
    values, passed through an exact product), fp32 output against float64 x / (1 + e^-x).
    Its reciprocal (bit-pattern estimate + two Newton steps, <= 6.7e-6; host-checked in
    test_numerics_host.py) and the fast exponential (whose argument rounding grows with |x|)
    keep the relative error below 1.5e-5 over the whole range the epilogue clamps to."""
    import ctypes
    import torch
    M, K, N = 2048, 16, 16
    x = bf16_round(np.linspace(-80.0, 80.0, M).astype(np.float32))
    a = np.zeros((M, K), np.float32)
    a[:, 0] = x
    w = np.zeros((N, K), np.float32)
    w[:, 0] = 1.0
    A = torch.from_numpy(a).to("cuda", torch.bfloat16)
    B = torch.from_numpy(w).to("cuda", torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    vp = ctypes.c_void_p
    gpu_bf16._call("sana_op_gemm_f32out_device", vp(A.data_ptr()), vp(B.data_ptr()), ctypes.c_int(M),
                   ctypes.c_int(N), ctypes.c_int(K), None, ctypes.c_int(1), vp(out.data_ptr()))
    gpu_bf16.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    xd = x.astype(np.float64)[:, None]
    ref = xd / (1.0 + np.exp(-xd))
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-300)
    assert np.isfinite(got).all()
    assert rel.max() <= 1.5e-5, float(rel.max())


def _dwglu_f64(x, w, b):
    """Depthwise 3x3 (zero padding) + bias over [S, H, W, E] tokens, split into the value and
    gate halves (common_ops.cpp:484-505 and 745-758), in float64."""
    S, H, W, E = x.shape
    xp = np.zeros((S, H + 2, W + 2, E))
    xp[:, 1:-1, 1:-1] = x
    acc = np.zeros((S, H, W, E))
    for ky in range(3):
        for kx in range(3):
            acc += xp[:, ky:ky + H, kx:kx + W] * w[:, ky * 3 + kx]
    acc += b
    return acc[..., :E // 2], acc[..., E // 2:]


@pytest.mark.parametrize("S,H,W,E,gscale", [(2, 32, 32, 5760, 1.0), (1, 64, 64, 256, 1.0), (3, 7, 40, 80, 1.0),
                                            (1, 1, 1, 16, 1.0), (2, 9, 33, 128, 40.0)])
def test_depthwise_glu_device(gpu_bf16, S, H, W, E, gscale):
    """The bf16 streaming depthwise+GLU kernel on device buffers (config-2 channel count, two
    column stripes, a partial channel slice, a single pixel, gates reaching +-100): every bf16
    output within its own rounding (2^-8) of the float64 result of the same bf16 inputs, plus
    the hardware tanh's error (2^-10 relative) carried through silu(g) = g (1 + tanh(g/2)) / 2."""
    import ctypes

    import torch
    rng = np.random.default_rng(S * 1000 + H * 10 + W + E)
    x = bf16_round(rng.standard_normal((S, H, W, E)).astype(np.float32))
    w = (rng.standard_normal((E, 9)) * 0.3).astype(np.float32)
    b = rng.standard_normal(E).astype(np.float32)
    w[E // 2:] *= gscale
    b[E // 2:] *= gscale
    v, g = _dwglu_f64(x.astype(np.float64), w.astype(np.float64), b.astype(np.float64))
    sig = 1.0 / (1.0 + np.exp(-g))
    ref = v * g * sig
    xt = torch.from_numpy(x).to("cuda", torch.bfloat16)
    wt, bt = torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda()
    out = torch.empty(S, H, W, E // 2, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    vp = ctypes.c_void_p
    gpu_bf16._call("sana_op_depthwise_glu_device", vp(xt.data_ptr()), ctypes.c_int(S), ctypes.c_int(H),
                   ctypes.c_int(W), ctypes.c_int(E), vp(wt.data_ptr()), vp(bt.data_ptr()), vp(out.data_ptr()))
    gpu_bf16.synchronize()
    got = out.float().cpu().numpy().astype(np.float64)
    tanh_err = 2.0 ** -10 * np.abs(v * g / 2) * np.abs(2 * sig - 1)
    bound = 2.0 ** -8 * np.abs(ref) + tanh_err + 1e-5 * np.abs(v) + 1e-6
    err = np.abs(got - ref)
    assert (err <= bound).all(), float((err / bound).max())


@pytest.mark.parametrize("rows,C,rps", [(32768 // 8, 1152, 1024), (45, 1152, 7), (33, 256, 5), (19, 384, 19),
                                         (10, 1000, 3)])
def test_ln_modulate_device(gpu_bf16, rows, C, rps):
    """layer_norm + modulate on device rows (the register path for widths of 128 k, blocks whose
    rows span several sequences, and the generic path for other widths) against float64: every
    bf16 output within its own rounding of the exact value."""
    import ctypes

    import torch
    rng = np.random.default_rng(rows + C + rps)
    x = (rng.standard_normal((rows, C)) * 3 + 1.5).astype(np.float32)
    S = -(-rows // rps)
    mod = (rng.standard_normal((S, 6, C)) * 0.5).astype(np.float32)
    xd = x.astype(np.float64)
    mean = xd.mean(axis=1, keepdims=True)
    var = ((xd - mean) ** 2).mean(axis=1, keepdims=True)
    seq = np.arange(rows) // rps
    shift, scale = mod[seq, 3].astype(np.float64), mod[seq, 4].astype(np.float64)
    ref = (xd - mean) / np.sqrt(var + 1e-6) * (1 + scale) + shift
    xt, mt = torch.from_numpy(x).cuda(), torch.from_numpy(mod).cuda()
    out = torch.empty(rows, C, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    gpu_bf16._call("sana_op_ln_modulate_device", ctypes.c_void_p(xt.data_ptr()), ctypes.c_longlong(rows),
                   ctypes.c_int(C), ctypes.c_int(rps), ctypes.c_void_p(mt.data_ptr()), ctypes.c_longlong(6 * C),
                   ctypes.c_int(3), ctypes.c_int(4), ctypes.c_float(1e-6), ctypes.c_void_p(out.data_ptr()))
    gpu_bf16.synchronize()
    got = out.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - ref)
    bound = 2.0 ** -8 * np.abs(ref) + 1e-5 * (1 + np.abs(ref))
    assert (err <= bound).all(), float((err / bound).max())


@pytest.mark.parametrize("M,N,K,rpg,copy", [(4096 + 96, 1152, 1152, 1024, True), (3000, 1152, 2880, 700, False),
                                             (1000, 384, 128, 300, True), (2304, 200, 64, 2304, True)])
def test_gemm_residual_epilogue(gpu_bf16, M, N, K, rpg, copy):
    """out = resid + gate[row / rows_per_gate] * (A B^T + bias) with an optional bf16 copy (the
    out-projection, cross-out and FF-point epilogues): CTA-pair and single-CTA kernels, ragged
    row and column tiles, TMA-stored and element-wise column batches, against float64 of the
    same bf16 operands."""
    import ctypes

    import torch
    rng = np.random.default_rng(M + N + K)
    a = bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    w = bf16_round((rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    b = rng.standard_normal(N).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32)
    g = rng.standard_normal((-(-M // rpg), N)).astype(np.float32)
    ref = r + g[np.arange(M) // rpg] * (a.astype(np.float64) @ w.astype(np.float64).T + b)
    A, B = torch.from_numpy(a).to("cuda", torch.bfloat16), torch.from_numpy(w).to("cuda", torch.bfloat16)
    bt, rt, gt = (torch.from_numpy(x).cuda() for x in (b, r, g))
    out = torch.empty(M, N, device="cuda")
    out2 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16) if copy else None
    torch.cuda.synchronize()
    vp = ctypes.c_void_p
    gpu_bf16._call("sana_op_gemm_residual_device", vp(A.data_ptr()), vp(B.data_ptr()), ctypes.c_int(M),
                   ctypes.c_int(N), ctypes.c_int(K), vp(bt.data_ptr()), vp(rt.data_ptr()), vp(gt.data_ptr()),
                   ctypes.c_int(rpg), vp(out.data_ptr()), vp(out2.data_ptr()) if copy else None)
    gpu_bf16.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    scale = np.abs(g[np.arange(M) // rpg]) * (np.abs(a) @ np.abs(w).T + np.abs(b))
    assert (np.abs(got - ref) <= 1e-5 * scale + 1e-5 * np.abs(ref) + 1e-6).all()
    if copy:
        got2 = out2.float().cpu().numpy().astype(np.float64)
        assert (np.abs(got2 - got) <= 2.0 ** -8 * np.abs(got) + 1e-30).all()


@pytest.mark.parametrize("M,N,K", [(4096, 1152, 1152), (4096, 3456, 1152), (2048, 5760, 1152), (2304, 1152, 2880),
                                   (4096, 1152, 128), (8192, 3456, 1152)])
def test_gemm_short_m_shapes(gpu_bf16, M, N, K):
    """The projections at the per-GPU batch of 4 and 8 GPUs (2048 and 4096 rows), with K up to
    the FF point projection's 2880, and config 4's QKV: fp32 output against float64 of the same
    bf16 operands, bit-identical across calls."""
    import ctypes
    import torch
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    a = bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    w = bf16_round((rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    b = rng.standard_normal(N).astype(np.float32)
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b
    A, B = torch.from_numpy(a).to("cuda", torch.bfloat16), torch.from_numpy(w).to("cuda", torch.bfloat16)
    bt = torch.from_numpy(b).cuda()
    outs = []
    vp = ctypes.c_void_p
    for _ in range(2):
        out = torch.full((M, N), float("nan"), device="cuda")
        torch.cuda.synchronize()
        gpu_bf16._call("sana_op_gemm_f32out_device", vp(A.data_ptr()), vp(B.data_ptr()), ctypes.c_int(M),
                       ctypes.c_int(N), ctypes.c_int(K), vp(bt.data_ptr()), ctypes.c_int(0), vp(out.data_ptr()))
        gpu_bf16.synchronize()
        outs.append(out.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    got = outs[0].astype(np.float64)
    scale = np.abs(a).astype(np.float64) @ np.abs(w).astype(np.float64).T + np.abs(b)
    assert (np.abs(got - ref) <= 1e-5 * scale + 1e-6).all(), float((np.abs(got - ref) / (scale + 1e-6)).max())


def test_bounded_wait_times_out_and_handle_recovers():
    """Failure detection without a fault: a device wait on a flag that nothing sets gives up
    after the handle's wait limit (1 ms here), the call returns SANA_ERR_TIMEOUT, and the same
    handle then runs a tensor-core GEMM correctly and passes the wait once the flag is set."""
    import time

    import torch
    from sana_b200 import SANA_MODE_BF16, SanaCuda, SanaError
    g = SanaCuda(0, SANA_MODE_BF16)
    assert g.wait_limit() == 2_000_000_000
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    g.set_wait_limit(1_000_000)
    t0 = time.perf_counter()
    with pytest.raises(SanaError) as e:
        g.selftest_wait(flag.data_ptr(), 1)
    assert e.value.code == 3, e.value  # SANA_ERR_TIMEOUT
    assert time.perf_counter() - t0 < 1.0
    with pytest.raises(ValueError):
        g.set_wait_limit(10)
    g.set_wait_limit(2_000_000_000)
    rng = np.random.default_rng(9)
    a = bf16_round(rng.standard_normal((2048, 256)).astype(np.float32))
    w = bf16_round((rng.standard_normal((512, 256)) * 0.05).astype(np.float32))
    A, B = torch.from_numpy(a).to("cuda", torch.bfloat16), torch.from_numpy(w).to("cuda", torch.bfloat16)
    out = torch.empty(2048, 512, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    g.gemm_device(A.data_ptr(), B.data_ptr(), 2048, 512, 256, out.data_ptr())
    g.synchronize()
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    assert rel_err(out.float().cpu().numpy(), ref) < 5e-3
    flag.fill_(1)
    torch.cuda.synchronize()
    g.selftest_wait(flag.data_ptr(), 1)
    g.close()


def test_gemm_repeatable(gpu_bf16):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((1024, 1152)).astype(np.float32)
    w = rng.standard_normal((1152, 1152)).astype(np.float32)
    a = gpu_bf16.linear_3d(x, w)
    b = gpu_bf16.linear_3d(x, w)
    assert np.array_equal(a, b)


def test_handles_on_two_devices_in_one_process():
    """Handles on two GPUs of one process: the tensor-core GEMM and the depthwise stream kernel
    (both above the default shared-memory limit, set up per device) give the same bits on
    each device. Needs two visible GPUs."""
    import torch
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    gen = torch.Generator(device="cpu").manual_seed(3)
    A = torch.randn(4096, 1152, generator=gen).to(torch.bfloat16)
    B = (torch.randn(1152, 1152, generator=gen) * 0.02).to(torch.bfloat16)
    H = torch.randn(2 * 32 * 32, 640, generator=gen).to(torch.bfloat16)
    w = torch.randn(640 * 9, generator=gen) * 0.1
    b = torch.randn(640, generator=gen) * 0.1
    outs = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            g = SanaCuda(dev, SANA_MODE_BF16)
            a, bb, h = A.cuda(dev), B.cuda(dev), H.cuda(dev)
            wd, bd = w.cuda(dev), b.cuda(dev)
            out = torch.empty(4096, 1152, dtype=torch.bfloat16, device=f"cuda:{dev}")
            glu = torch.empty(2 * 32 * 32, 320, dtype=torch.bfloat16, device=f"cuda:{dev}")
            g.gemm_device(a.data_ptr(), bb.data_ptr(), 4096, 1152, 1152, out.data_ptr())
            g._call("sana_op_depthwise_glu_device", ctypes.c_void_p(h.data_ptr()), ctypes.c_int(2), ctypes.c_int(32),
                    ctypes.c_int(32), ctypes.c_int(640), ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(bd.data_ptr()),
                    ctypes.c_void_p(glu.data_ptr()))
            torch.cuda.synchronize(dev)
            outs.append((out.cpu(), glu.cpu()))
            g.close()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    ref = (A.float() @ B.float().T)
    assert float((outs[0][0].float() - ref).norm() / ref.norm()) < 1e-2


# --- the reference's known-answer tests ------------------------------------------------------
@pytest.mark.parametrize("case", K.ALL_KATS, ids=lambda f: f.__name__)
def test_reference_kats_fp32_mode(gpu_f32, case):
    K.check(case(gpu_f32))


# --- ops against the reference's outputs -----------------------------------------------------
@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_ops_match_golden(request, mode, oracle):
    g = request.getfixturevalue("gpu_" + mode)
    gold = np.load(os.path.join(GOLDEN, "ops_small.npz"))
    tol = F32_TOL if mode == "f32" else BF16_TOL
    for name, meth, args in MG.ops_cases(oracle.randn):
        out = getattr(g, meth)(*args)
        assert out.shape == gold[name].shape, name
        e = rel_err(out, gold[name])
        assert e < tol, (name, e)


# --- edge cases of the op contracts (against the oracle) -------------------------------------
def test_attention_all_keys_masked(gpu_f32, gpu_bf16, oracle):
    """Every key masked: the reference's softmax still runs over all keys, each score
    carrying the -10000 bias (its fp32 rounding at that magnitude included); no key may
    be dropped."""
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((2, 2, 5, 8)).astype(np.float32) for _ in range(3))
    bias = np.full((2, 1, 5), -10000.0, np.float32)
    ref = oracle.attention(q, k, v, bias)
    assert rel_err(ref, oracle.attention(q, k, v)) < 1e-2  # close to, not equal to, unmasked
    assert rel_err(gpu_f32.attention(q, k, v, bias), ref) < F32_TOL
    assert rel_err(gpu_bf16.attention(q, k, v, bias), ref) < BF16_TOL


def test_attention_mask_with_holes_and_soft_bias(gpu_f32, oracle):
    rng = np.random.default_rng(2)
    q = rng.standard_normal((2, 3, 9, 16)).astype(np.float32)
    k, v = (rng.standard_normal((2, 3, 12, 16)).astype(np.float32) for _ in range(2))
    bias = rng.standard_normal((2, 1, 12)).astype(np.float32)
    bias[0, 0, [1, 4, 11]] = -10000.0
    bias[1, 0, 6:] = -10000.0
    assert rel_err(gpu_f32.attention(q, k, v, bias), oracle.attention(q, k, v, bias)) < F32_TOL


@pytest.mark.parametrize("D,Tq,Tk", [(1, 3, 5), (32, 200, 130), (72, 129, 257), (128, 16, 16)])
def test_linear_attention_shapes(gpu_f32, gpu_bf16, oracle, D, Tq, Tk):
    rng = np.random.default_rng(D)
    q = rng.standard_normal((2, 3, Tq, D)).astype(np.float32)
    k, v = (rng.standard_normal((2, 3, Tk, D)).astype(np.float32) for _ in range(2))
    ref = oracle.linear_attention(q, k, v)
    assert rel_err(gpu_f32.linear_attention(q, k, v), ref) < F32_TOL
    assert rel_err(gpu_bf16.linear_attention(q, k, v), ref) < BF16_TOL


def test_linear_attention_all_negative_queries(gpu_f32):
    """relu(q) = 0: numerator 0, denominator 1e-15, output exactly 0 (transformer_ops.cpp:532)."""
    q = -np.ones((1, 1, 4, 2), np.float32)
    k = np.ones((1, 1, 4, 2), np.float32)
    v = np.arange(8, dtype=np.float32).reshape(1, 1, 4, 2)
    assert np.array_equal(gpu_f32.linear_attention(q, k, v), np.zeros_like(q))


@pytest.mark.parametrize("H,W", [(1, 1), (1, 7), (5, 7), (32, 32)])
def test_depthwise_and_glumb_grids(gpu_f32, gpu_bf16, oracle, H, W):
    rng = np.random.default_rng(H * 31 + W)
    img = rng.standard_normal((2, 16, H, W)).astype(np.float32)
    w = rng.standard_normal((16, 1, 3, 3)).astype(np.float32)
    b = rng.standard_normal(16).astype(np.float32)
    assert rel_err(gpu_f32.depthwise3x3(img, w, b), oracle.depthwise3x3(img, w, b)) < F32_TOL
    wi = (rng.standard_normal((32, 16, 1, 1)) * 0.3).astype(np.float32)
    bi = rng.standard_normal(32).astype(np.float32)
    wd = (rng.standard_normal((32, 1, 3, 3)) * 0.3).astype(np.float32)
    bd = rng.standard_normal(32).astype(np.float32)
    wp = (rng.standard_normal((12, 16, 1, 1)) * 0.3).astype(np.float32)
    ref = oracle.glumb_conv(img, wi, bi, wd, bd, wp)
    assert rel_err(gpu_f32.glumb_conv(img, wi, bi, wd, bd, wp), ref) < F32_TOL
    assert rel_err(gpu_bf16.glumb_conv(img, wi, bi, wd, bd, wp), ref) < BF16_TOL


def test_norms_degenerate_rows(gpu_f32, oracle):
    x = np.zeros((1, 3, 5), np.float32)
    x[0, 1] = 7.0  # constant row: zero variance
    x[0, 2] = np.arange(5, dtype=np.float32)
    for eps in (1e-6, 1e-5):
        np.testing.assert_allclose(gpu_f32.layer_norm(x, eps), oracle.layer_norm(x, eps), rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(gpu_f32.rms_norm(x, eps), oracle.rms_norm(x, eps), rtol=1e-5, atol=1e-6)


def test_invalid_arguments_raise(gpu_f32):
    with pytest.raises(ValueError):
        gpu_f32.attention_block(np.ones((1, 2, 3), np.float32), *[np.eye(3, dtype=np.float32), None] * 4, 2)
    with pytest.raises(ValueError):
        gpu_f32.scheduler_update(2, np.array([0.5, 0.2, 0.0], np.float32), 0, np.ones(1, np.float32),
                                 np.ones(1, np.float32), np.ones(1, np.float32))
    with pytest.raises(ValueError):
        gpu_f32.block_forward(0, np.ones((1, 2, 2), np.float32), np.ones((1, 2, 2), np.float32),
                              np.ones((1, 12), np.float32))


def test_scheduler_trajectory_matches_golden(gpu_f32, oracle):
    """step_sana_scheduler through the device kernel over a 20-step schedule."""
    g = np.load(os.path.join(GOLDEN, "scheduler_20.npz"))
    _, sg = gpu_f32.scheduler_schedule(20, 3.0)
    mo = MG.syn._draw(oracle.randn, 20 * 64, 300).reshape(20, 64)
    x = MG.syn._draw(oracle.randn, 64, 301)
    hist, lower = [], 0
    for s in range(20):
        x, hist, lower = gpu_f32.scheduler_step(sg, s, lower, hist, mo[s], x)
        assert rel_err(x, g["samples"][s]) < 1e-6, s


def test_scheduler_configs_match_reference(gpu_f32):
    """step_sana_scheduler for every configuration the reference accepts (heun / midpoint,
    solver_order 1, lower_order_final off, variance-preserving sigmas, other
    num_train_timesteps), through the device update, against the reference's trajectories."""
    from test_oracle_pin import scheduler_cases
    for cfg, mo, x0, _, want in scheduler_cases():
        sg = want["sg"]
        x, hist, lower, step = x0, [], 0, 0
        for s in range(len(mo)):
            x, hist, lower, step = gpu_f32.scheduler_step_config(cfg, sg, step, lower, hist, mo[s], x)
            assert rel_err(x, want["samples"][s]) < 1e-6, (cfg, s)
        n = len(mo)
        assert step == n and lower == min(n, cfg["solver_order"]) and len(hist) == min(n, cfg["solver_order"])
    heun = dict(solver_heun=1)
    with pytest.raises(ValueError):
        gpu_f32.scheduler_step_config(dict(solver_order=3), want["sg"], 0, 0, [], mo[0], x0)
    # second order at step 0 is refused as the reference refuses it
    with pytest.raises(ValueError):
        gpu_f32.scheduler_update_config(heun, 2, want["sg"], 0, mo[0], mo[0], x0)


@pytest.mark.parametrize("D", [72, 64, 32])
def test_cross_attention_key_counts(gpu_bf16, oracle, D):
    """The tensor-core cross-attention at valid lengths of 1, 17, 128, 129, 255 and 300 keys
    (64-key chunks full, partial and single-key), a query count that leaves a partial
    128-query tile, and six sequences."""
    from sana_b200 import synthetic as syn
    rng = np.random.default_rng(D)
    lens = (1, 17, 128, 129, 255, 300)
    S, H, Tq, L = len(lens), 3, 1024 + 64, 300
    q = rng.standard_normal((S, H, Tq, D)).astype(np.float32)
    k, v = (rng.standard_normal((S, H, L, D)).astype(np.float32) for _ in range(2))
    bias = syn.attention_bias(lens, L)
    ref = oracle.attention(q, k, v, bias)
    got = gpu_bf16.attention(q, k, v, bias)
    for s in range(S):
        assert rel_err(got[s], ref[s]) < BF16_TOL, (D, lens[s], rel_err(got[s], ref[s]))


def test_cross_attention_two_tile_blocks(gpu_bf16):
    """Config 2's cross-attention grid (32 sequences x 16 heads x 1024 queries, 300 caption
    tokens), where each block takes two query tiles that share the keys and values: valid
    lengths on both sides of the two-chunk limit (kept in shared memory up to 128 live keys,
    streamed again beyond), against float64 softmax over the live keys of the same bf16
    operands (masked keys carry exactly zero weight, transformer_ops.cpp:357-388)."""
    from sana_b200 import synthetic as syn
    rng = np.random.default_rng(11)
    S, H, Tq, L, D = 32, 16, 1024, 300, 72
    lens = [(8, 24, 64, 65, 120, 128, 129, 200, 300, 1)[i % 10] for i in range(S)]
    q = bf16_round(rng.standard_normal((S, H, Tq, D)).astype(np.float32))
    k = bf16_round(rng.standard_normal((S, H, L, D)).astype(np.float32))
    v = bf16_round(rng.standard_normal((S, H, L, D)).astype(np.float32))
    got = gpu_bf16.attention(q, k, v, syn.attention_bias(lens, L))
    scale = 1.0 / np.sqrt(D)
    for s in range(S):
        n = lens[s]
        sc = np.einsum("htd,hkd->htk", q[s].astype(np.float64), k[s, :, :n].astype(np.float64)) * scale
        sc -= sc.max(axis=-1, keepdims=True)
        p_ = np.exp(sc)
        p_ /= p_.sum(axis=-1, keepdims=True)
        ref = np.einsum("htk,hkd->htd", p_, v[s, :, :n].astype(np.float64))
        assert rel_err(got[s], ref) < BF16_TOL, (s, n, rel_err(got[s], ref))


@pytest.mark.parametrize("D,Tq,L,lens", [(72, 1024, 300, (8, 24)), (72, 100, 300, (300, 1)), (32, 77, 70, (70, 65)),
                                        (64, 130, 129, (64, 129)), (128, 40, 20, (20, 3))])
def test_cross_attention_tensor_core_shapes(gpu_bf16, oracle, D, Tq, L, lens):
    """The bf16 tensor-core cross-attention at the model's shape (16 heads x 72, 300 caption
    tokens, short valid prefixes) and at chunk-boundary key counts."""
    from sana_b200 import synthetic as syn
    rng = np.random.default_rng(D * 3 + L)
    q = rng.standard_normal((2, 4, Tq, D)).astype(np.float32)
    k, v = (rng.standard_normal((2, 4, L, D)).astype(np.float32) for _ in range(2))
    bias = syn.attention_bias(lens, L)
    ref = oracle.attention(q, k, v, bias)
    assert rel_err(gpu_bf16.attention(q, k, v, bias), ref) < BF16_TOL
