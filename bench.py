"""Throughput benchmark of the B200 Sana-0.6B denoiser (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

Workload: 16 images x CFG (32 sequences of 1024 tokens), 20-step
DPM-Solver++ loop with guidance 4.5, caption states [300, 2304] with valid lengths drawn
from 8..120; seeded random-init weights of the real architecture (synthetic: there are no
checkpoints or datasets here). The 16 images are sharded across the ranks in contiguous
ranges (sana_b200.sharding), weights replicated, every image's inputs drawn from seeds of its
own index; the final latents are NCCL-gathered into the full batch on every rank after each
loop (the path's only collective). Total work is fixed as N grows ("strong" scaling).

    python bench.py --microbench [--op NAME,...]     (one GPU)
    torchrun --nproc-per-node 2 bench.py --gpus 2 --cfg-pair   (latency mode, configs[1])

One bench step = one full denoising loop over the rank's batch (caption projection,
cross-K/V for all blocks, 20 denoiser steps, CFG + scheduler), replayed from a CUDA graph.
`value` is images/s over all ranks with inputs resident in HBM, timed with CUDA events on
the launching stream (L2 flushed between iterations, untimed), max over ranks; `e2e` is the
same through the reference-facing C ABI call with pinned host buffers (host<->device
copies inside the timed region). Rank 0 prints one JSON line.

--impl reference times the reference's own CPU implementation (oracle/_ref, compiled from
the reference's sources; the CPU oracle when that build is absent) on this host's cores:
one block_forward of one sequence per thread, extrapolated to images/s.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "sana.cpp_b200")]

METRIC = "denoiser steps/sec & images/sec (Sana-0.6B 1024px, 20 steps, CFG) at 1/2/4/8 B200"
NUM_STEPS = 20
GUIDANCE = 4.5
CAPTION_LEN = 300
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum of one FF-inverted projection launch at the
# default workload (M=32768, K=1152, N=5760), copied from an ncu capture of that kernel; the
# JSON line names the capture it came from. Not measured by this script.
FF_INVERTED_TRAFFIC = {"bytes": 88_987_904 + 329_661_952,
                       "source": "ncu --set full capture of gemm_tc2_kernel<256,0,0,0> at M=32768 K=1152 N=5760 "
                                 "(profiles/gemm_tc2_ff_inverted_config2.md)"}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ------------------------------------------------------------------------------------------
# Synthetic workload
# ------------------------------------------------------------------------------------------
def make_weights(dims, seed=0, randn=None):
    """The synthetic checkpoint, drawn with `randn` (the product's torch-compatible generator by
    default; the CPU arms pass their own checker's, so that their process maps no product
    library)."""
    from sana_b200 import synthetic as syn
    if randn is None:
        from sana_b200 import randn_torch_cpu as randn
    specs = syn.model_tensor_specs(dims)
    workers = min(32, len(os.sched_getaffinity(0)))
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        return list(ex.map(lambda j: syn.generate_tensor(specs[j], j, dims, randn, seed), range(len(specs))))


def make_inputs(first, count):
    """Images [first, first + count) of the synthetic batch (sana_b200.sharding.image_inputs)."""
    from sana_b200 import randn_torch_cpu
    from sana_b200.sharding import image_inputs
    return image_inputs(randn_torch_cpu, first, count, (32, 32, 32), CAPTION_LEN, 2304)


def loop_flops(images, lens, C=1152, E=5760, T=1024, n_blocks=28, Hs=36, steps=NUM_STEPS, Din=2304, Cl=32):
    """Algorithmic FLOPs of one denoising loop (multiply-add = 2): per step and sequence the
    block GEMMs, linear attention, cross-attention at each sequence's valid key count and the
    depthwise conv; once per loop the caption projection and cross-K/V (hoisted)."""
    D = C // Hs
    S = 2 * images
    gemm_block = 2 * T * C * (3 * C + C + C + C + E) + 2 * T * (E // 2) * C
    lin = 2 * T * D * D * 2 * Hs + 2 * T * D * Hs
    dw = 2 * 9 * T * E
    xattn = sum(4 * T * L * C for L in lens)  # q k^T and p v over the valid keys of each sequence
    per_step = S * n_blocks * (gemm_block + lin + dw) + n_blocks * xattn + S * (2 * T * Cl * C * 2)
    once = S * CAPTION_LEN * (2 * Din * C + 2 * C * C) + n_blocks * S * CAPTION_LEN * 2 * C * 2 * C
    gemm_only = steps * S * n_blocks * gemm_block
    return steps * per_step + once, gemm_only


def kernel_classes(images, lens, C=1152, E=5760, T=1024, Hs=36, Cl=32):
    """Algorithmic work per launch of each profiled kernel class: ("flop", FLOPs) for the
    tensor-core projections, ("byte", HBM bytes read + written with bf16 activations) for the
    memory-bound kernels."""
    S = 2 * images
    M = S * T
    D = C // Hs
    xbytes = sum(2 * T * L * C * 2 for L in lens)  # not used as a rate basis; cross-attn is FLOP-rated below
    return {
        "gemm_qkv": ("flop", 2.0 * M * C * 3 * C),
        "gemm_out": ("flop", 2.0 * M * C * C),
        "gemm_cross_q": ("flop", 2.0 * M * C * C),
        "gemm_cross_out": ("flop", 2.0 * M * C * C),
        "gemm_ff_inverted": ("flop", 2.0 * M * C * E),
        "gemm_ff_point": ("flop", 2.0 * M * (E // 2) * C),
        "cross_attention": ("flop", float(sum(4 * T * L * C for L in lens))),
        # q, k, v read + output written
        "linear_attention": ("byte", 2.0 * M * 3 * C + 2.0 * M * C),
        # SiLU-ed inverted output read, GLU output written
        "depthwise_glu": ("byte", 2.0 * M * E + 2.0 * M * (E // 2)),
        # fp32 residual read, bf16 modulated row written
        "ln_modulate": ("byte", 4.0 * M * C + 2.0 * M * C),
    }


# ------------------------------------------------------------------------------------------
# Clock sampling during the timed region
# ------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *exc):
        if self.p:
            self.p.terminate()
            self.p.wait(timeout=10)

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines()]
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9 and r[0].strip() == self.gpu]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


def vae_cpu_sample(vd, threads=None):
    """The reference's run_vae_decode (oracle/_ref; the oracle port without it) on this host:
    one decode of 4 x 4 latents (a 128 x 128 image) per thread, all threads at once, scaled
    to the 1024 x 1024 decode by algorithmic FLOPs (the decoder's work is linear in pixels)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, Reference
    from sana_b200 import synthetic_vae as sv
    impl, kind = (Reference(), "reference") if Reference.available() else (Oracle(), "port")
    threads = 1 if kind == "port" else (threads or min(64, len(os.sched_getaffinity(0))))
    tensors = sv.generate_vae(vd, impl.randn, 3)
    lats = [impl.randn(vd.latent_channels * 16, 900 + i).reshape(1, vd.latent_channels, 4, 4)
            for i in range(threads)]
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda x: impl.vae_decode(vd, tensors, x), lats))
    dt = time.perf_counter() - t0
    scale = sv.vae_flops(vd, 32, 32) / sv.vae_flops(vd, 4, 4)
    ms_per_image = dt * 1000.0 * scale / threads
    return {"value": round(ms_per_image, 1), "unit": "ms per 1024x1024 image (throughput)", "cores": threads,
            "kind": kind, "sample": f"{threads} decodes of 4x4 latents in {dt:.1f} s, scaled by FLOPs x{scale:.0f}"}


# ------------------------------------------------------------------------------------------
# CPU baseline (the reference's own code) — a bounded sample on this host's cores
# ------------------------------------------------------------------------------------------
def cpu_sample(threads=None):
    """One reference block_forward of one 1024-token sequence per thread, all threads at
    once; returns (images_per_s, seconds, threads, kind). Weights and inputs come from the
    checker's own torch-compatible generator (the same draws as the product's)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, Reference
    from sana_b200 import synthetic as syn
    impl, kind = (Reference(), "reference") if Reference.available() else (Oracle(), "port")
    randn_torch_cpu = impl.randn
    d1 = syn.ModelDims(n_blocks=1)
    tensors = make_weights(d1, randn=randn_torch_cpu)
    model = impl.model(tensors, *d1.as_args())
    del tensors
    threads = threads or min(64, len(os.sched_getaffinity(0)))
    if kind == "port":
        threads = 1  # the oracle parallelises internally
    enc = syn.encoder_states(randn_torch_cpu, 1, CAPTION_LEN, 2304, 7)
    ctx = model.project_caption(enc)
    _, tmod = model.time_embed([999.0])
    bias = syn.attention_bias([24], CAPTION_LEN)
    xs = [syn._draw(randn_torch_cpu, 1024 * 1152, 500 + i).reshape(1, 1024, 1152) for i in range(threads)]
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda x: model.block_forward(0, x, ctx, tmod, bias), xs))
    dt = time.perf_counter() - t0
    seq_blocks_per_s = threads / dt
    images_per_s = seq_blocks_per_s / (2 * 28 * NUM_STEPS)
    return images_per_s, dt, threads, kind


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    W, K = args.warmup, args.steps
    vals, secs = [], []
    kind, threads = "reference", 0
    for i in range(W + K):
        v, dt, threads, kind = cpu_sample()
        if i >= W:
            vals.append(v)
            secs.append(dt)
    value = statistics.mean(vals)
    sample = (f"one reference block_forward of one 1024-token sequence per thread ({threads} threads at once), "
              f"extrapolated x2 sequences x28 blocks x{NUM_STEPS} steps per image")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": K, "warmup": W, "ms_per_step": 1000 * statistics.mean(secs), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args),
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def config_dict(args):
    per = [f"{(args.images + args.gpus - 1 - r) // args.gpus}" for r in range(args.gpus)]
    return {"workload": f"config2: {args.images} images x CFG ({2 * args.images} sequences x 1024 tokens) sharded "
                        f"over {args.gpus} GPU(s), {NUM_STEPS}-step DPM-Solver++ loop, guidance {GUIDANCE}",
            "global_batch": args.images, "images_per_gpu": "/".join(per), "seq_len": 1024,
            "caption_tokens": CAPTION_LEN, "caption_valid_lengths": "uniform 8..120 (seeded per image)",
            "self_attention": "36 heads x 32 (linear)", "cross_attention": "16 heads x 72 (softmax)",
            "parallelism": f"images sharded over {args.gpus} GPU(s), weights replicated, final latents gathered",
            "l2": "flushed between timed iterations (256 MiB write, untimed)"}


# ------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------
def gemm_roofline(g, torch, stream, M, peak_tflops):
    """The dominant kernel (tcgen05 GEMM) alone at the step's shapes: algorithmic FLOPs per
    launch / CUDA-event launch time, FLOP-weighted over the block's six projections."""
    shapes = [(M, 3456, 1152), (M, 1152, 1152), (M, 1152, 1152), (M, 1152, 1152), (M, 5760, 1152), (M, 1152, 2880)]
    tot_f, tot_ms, per = 0.0, 0.0, []
    dev = torch.device("cuda")
    for (m, n, k) in shapes:
        A = torch.randn(m, k, device=dev, dtype=torch.bfloat16)
        B = torch.randn(n, k, device=dev, dtype=torch.bfloat16) * 0.02
        C = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        torch.cuda.synchronize()
        for _ in range(3):
            g.gemm_device(A.data_ptr(), B.data_ptr(), m, n, k, C.data_ptr())
        reps = 10
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.gemm_device(A.data_ptr(), B.data_ptr(), m, n, k, C.data_ptr())
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        f = 2.0 * m * n * k
        per.append({"shape": [m, n, k], "ms": round(ms, 4), "tflops": round(f / ms / 1e9, 1)})
        tot_f += f
        tot_ms += ms
        del A, B, C
    achieved = tot_f / tot_ms / 1e9
    return achieved, per


MICRO_OPS = ("qkv_gemm", "linear_attention_16x72", "linear_attention_36x32", "depthwise_glu", "cross_attention",
             "ff_inverted_config2", "linear_attention_config2", "depthwise_glu_config2", "cross_attention_config2",
             "out_proj_config2", "ff_point_config2", "ln_modulate_config2", "vae_decode_1024")


def run_microbench(args):
    """BASELINE configs[4], the op-level microbenchmark: 4096 tokens, batch 2, hidden 1152,
    bf16 activations N(0,1), each op through its device entry point of the C ABI and against
    its roofline: (a) ReLU linear attention 16 x 72 (and the model's 36 x 32), (b) depthwise
    3x3 + SiLU-GLU on 5760 -> 2880 channels, (c) the QKV projection M=8192, K=1152, N=3456,
    (d) cross-attention to 300 unmasked caption tokens. Also three kernels at the loop's
    config-2 size (32 sequences x 1024 tokens): the FF-inverted projection M=32768, K=1152,
    N=5760 with bias and SiLU, linear attention 36 x 32 and depthwise+GLU on 32 x 32 images.
    L2 is flushed (256 MiB write, untimed) before every timed launch; the median of --steps
    launches is reported. One JSON line per op."""
    import torch
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    ops = MICRO_OPS if not args.op else tuple(args.op.split(","))
    bad = [o for o in ops if o not in MICRO_OPS]
    if bad:
        raise SystemExit(f"unknown --op {bad}; choose from {MICRO_OPS}")
    torch.cuda.set_device(0)
    g = SanaCuda(0, SANA_MODE_BF16)
    st = torch.cuda.Stream()
    g.set_stream(st.cuda_stream)
    for line in microbench_lines(g, st, ops, args.steps, args.warmup, args.no_cpu_baseline):
        print(json.dumps(line), flush=True)
    g.close()


CONFIG4_OPS = ("linear_attention_16x72", "linear_attention_36x32", "depthwise_glu", "qkv_gemm", "cross_attention")


def microbench_lines(g, st, ops, steps, warmup, no_cpu_baseline=True):
    """The microbenchmark of each op in `ops` on handle g (stream st): a list of dicts."""
    import ctypes
    import torch
    pk, pk_kind = peaks()
    g.lib.sana_op_linear_attention_workspace.restype = ctypes.c_size_t
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    lines = []
    vp, I = ctypes.c_void_p, ctypes.c_int
    S, T, C, E, L = 2, 4096, 1152, 5760, CAPTION_LEN
    gen = torch.Generator(device="cpu").manual_seed(4)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=gen) * scale).to(device="cuda", dtype=torch.bfloat16)

    def timed(fn):
        times = []
        with torch.cuda.stream(st):
            for _ in range(warmup):
                fn()
            for _ in range(steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                fn()
                e1.record(st)
                e1.synchronize()
                times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    def report(name, what, ms, work, bound, extra=None):
        if bound == "hbm":
            ach, peak, unit = work / ms / 1e6, pk["hbm_gbs"], "GB/s"
        else:
            ach, peak, unit = work / ms / 1e9, pk["bf16_tflops"], "TFLOP/s"
        lines.append({"microbench": name, "workload": what, "ms": round(ms, 4), "bound": bound,
                      "algorithmic": work, "achieved": round(ach, 1), "peak": peak, "unit": unit,
                      "frac": round(ach / peak, 3), "peak_source": f"{pk_kind} (burst: op timed alone)",
                      "steps": steps, "warmup": warmup, "l2": "flushed before every launch", **(extra or {})})

    for name in ops:
        if name == "vae_decode_1024":
            # the DC-AE f32c32 decoder after the loop (vae.cpp:243): 32 x 32 latents -> 1024 x 1024
            from sana_b200 import randn_torch_cpu
            from sana_b200 import synthetic_vae as sv
            vd = sv.VaeDims()
            g.vae_upload(vd, sv.generate_vae(vd, randn_torch_cpu, 3))
            lat = torch.randn(1, vd.latent_channels, 32, 32, generator=gen).cuda()
            img = torch.empty(1, vd.out_channels, 1024, 1024, device="cuda")
            ms = timed(lambda: g.vae_decode_device(lat.data_ptr(), 1, 32, 32, img.data_ptr()))
            report(name, "DC-AE f32c32 decode, latents [1,32,32,32] -> image [1,3,1024,1024], bf16 activations "
                         f"({g.vae_last_launches()} launches)", ms, sv.vae_flops(vd, 32, 32), "tensor",
                   extra=None if no_cpu_baseline else {"cpu_baseline": vae_cpu_sample(vd)})
            continue
        S, T = (32, 1024) if name.endswith("config2") else (2, 4096)
        side = int(round(T ** 0.5))
        if name.startswith("linear_attention"):
            heads, D = (16, 72) if name.endswith("16x72") else (36, 32)
            qkv = rnd(S * T, 3 * C)
            part = torch.empty(g.lib.sana_op_linear_attention_workspace(I(S), I(T), I(heads), I(D)) // 4,
                               device="cuda", dtype=torch.float32)
            out = torch.empty(S * T, C, device="cuda", dtype=torch.bfloat16)
            ms = timed(lambda: g._call("sana_op_linear_attention_device", vp(qkv.data_ptr()), I(S), I(T), I(heads),
                                       I(D), vp(part.data_ptr()), vp(out.data_ptr())))
            report(name, f"q,k,v [{S},{heads},{T},{D}] bf16 -> o", ms, 2.0 * S * T * 4 * C, "hbm")
        elif name.startswith("depthwise_glu"):
            h = rnd(S * T, E)
            w = (torch.randn(E * 9, generator=gen) * 0.02).cuda()
            b = torch.zeros(E, device="cuda")
            out = torch.empty(S * T, E // 2, device="cuda", dtype=torch.bfloat16)
            ms = timed(lambda: g._call("sana_op_depthwise_glu_device", vp(h.data_ptr()), I(S), I(side), I(side), I(E),
                                       vp(w.data_ptr()), vp(b.data_ptr()), vp(out.data_ptr())))
            report(name, f"[{S},{side},{side},{E}] -> [{S},{side},{side},{E // 2}] bf16", ms,
                   2.0 * S * T * (E + E // 2), "hbm")
        elif name == "qkv_gemm":
            M, N, K = S * T, 3 * C, C
            A, B = rnd(M, K), rnd(N, K, scale=0.02)
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            ms = timed(lambda: g.gemm_device(A.data_ptr(), B.data_ptr(), M, N, K, out.data_ptr()))
            report(name, f"M={M} K={K} N={N} bf16 -> bf16", ms, 2.0 * M * N * K, "tensor")
        elif name == "ff_inverted_config2":
            M, N, K = S * T, E, C
            A, B = rnd(M, K), rnd(N, K, scale=0.02)
            bias = torch.zeros(N, device="cuda")
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            ms = timed(lambda: g.gemm_device(A.data_ptr(), B.data_ptr(), M, N, K, out.data_ptr(), bias.data_ptr(), 1))
            report(name, f"M={M} K={K} N={N} +bias, SiLU, bf16 out", ms, 2.0 * M * N * K, "tensor")
        elif name == "ln_modulate_config2":
            # layer_norm + AdaLN modulate of the residual stream (norm1 / norm2 of every block)
            M = S * T
            x = torch.randn(M, C, generator=gen).cuda()
            mod = torch.randn(S, 6 * C, generator=gen).cuda()
            out = torch.empty(M, C, device="cuda", dtype=torch.bfloat16)
            ms = timed(lambda: g._call("sana_op_ln_modulate_device", vp(x.data_ptr()), ctypes.c_longlong(M), I(C), I(T),
                                       vp(mod.data_ptr()), ctypes.c_longlong(6 * C), I(0), I(1), ctypes.c_float(1e-6),
                                       vp(out.data_ptr())))
            byts = 4.0 * M * C + 2.0 * M * C
            report(name, f"[{M},{C}] fp32 -> bf16 ({byts / 1e6:.0f} MB)", ms, byts, "hbm")
        elif name in ("out_proj_config2", "ff_point_config2"):
            # the self-attention output projection: fp32 residual + gate x (A W^T + b), bf16 copy;
            # the FF point projection: the same from the 2880 GLU channels, no copy
            copy = name == "out_proj_config2"
            M, N, K = S * T, C, (C if copy else E // 2)
            A, Bw = rnd(M, K), rnd(N, K, scale=0.02)
            bias = torch.zeros(N, device="cuda")
            resid = torch.randn(M, N, generator=gen).cuda()
            gate = torch.randn(S, N, generator=gen).cuda()
            out = torch.empty(M, N, device="cuda")
            out2 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16) if copy else None
            ms = timed(lambda: g._call("sana_op_gemm_residual_device", vp(A.data_ptr()), vp(Bw.data_ptr()), I(M),
                                       I(N), I(K), vp(bias.data_ptr()), vp(resid.data_ptr()), vp(gate.data_ptr()),
                                       I(T), vp(out.data_ptr()), vp(out2.data_ptr()) if copy else None))
            byts = 2.0 * M * K + 2.0 * N * K + 4.0 * M * N * 2 + (2.0 * M * N if copy else 0.0)
            report(name, f"M={M} K={K} N={N}: fp32 residual read + fp32{' and bf16' if copy else ''} out "
                         f"({byts / 1e6:.0f} MB; {2.0 * M * N * K / 1e9:.0f} GFLOP)", ms, byts, "hbm")
        elif name.startswith("cross_attention"):
            heads, D = 16, 72
            q, kv = rnd(S * T, C), rnd(S * L, 2 * C)
            kvl = torch.empty(S, device="cuda", dtype=torch.int32)
            out = torch.empty(S * T, C, device="cuda", dtype=torch.bfloat16)
            if name.endswith("config2"):  # the loop's caption masks: valid lengths uniform in 8..120
                from sana_b200.sharding import image_valid_lengths
                lens = [v for i in range(S // 2) for v in image_valid_lengths(i)]
                from sana_b200 import synthetic as syn
                bias = torch.from_numpy(syn.attention_bias(lens, L).reshape(S, L)).cuda()
                what = f"q [{S},{heads},{T},{D}], k/v {L} keys, valid lengths 8..120 (mean {sum(lens) / S:.0f})"
            else:
                lens, bias, what = [L] * S, None, f"q [{S},{heads},{T},{D}], k/v {L} keys, no mask"
            ms = timed(lambda: g._call("sana_op_cross_attention_device", vp(q.data_ptr()), vp(kv.data_ptr()),
                                       vp(bias.data_ptr()) if bias is not None else None, vp(kvl.data_ptr()), I(S),
                                       I(T), I(L), I(heads), I(D), vp(out.data_ptr())))
            report(name, what, ms, 4.0 * T * C * sum(lens), "tensor")
    del flush
    return lines


def run_cuda(args):
    import torch
    import torch.distributed as dist
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    from sana_b200 import synthetic as syn

    from sana_b200.watchdog import init_ranks
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    # a bounded process-group timeout and host heartbeats: a rank that never joins or stops
    # ends the others with an error instead of a wait for good
    rank, world, watch = init_ranks("nccl", timeout_s=300.0, device_id=torch.device("cuda", local))
    dims = syn.ModelDims()
    t0 = time.time()
    tensors = make_weights(dims)
    g = SanaCuda(local, SANA_MODE_BF16)
    g.upload_checkpoint(dims.as_args(), tensors)
    del tensors
    log(f"[rank {rank}] weights ready in {time.time() - t0:.1f}s")

    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    g.set_stream(stream.cuda_stream)
    from sana_b200.sharding import gather_images, shard_range
    total = args.images
    if total < world:
        raise SystemExit(f"--images {total} is smaller than the number of ranks {world}")
    first, B = shard_range(total, world, rank)
    lat, enc, bias, lens = make_inputs(first, B)
    d_lat = torch.from_numpy(lat).cuda()
    d_enc = torch.from_numpy(enc).cuda()
    d_bias = torch.from_numpy(bias).cuda()
    d_out = torch.empty_like(d_lat)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()

    def step():
        g.denoise_loop_device(d_lat.data_ptr(), B, 32, 32, d_enc.data_ptr(), CAPTION_LEN, 2304,
                              d_bias.data_ptr(), d_out.data_ptr(), GUIDANCE, NUM_STEPS)
        if world > 1:
            gather_images(d_out, total, world)

    for i in range(args.warmup):
        step()
        if watch:
            torch.cuda.synchronize()
            watch.beat(i + 1)
            watch.check()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- timed: K steps, CUDA events on the launching stream, L2 flushed between ----
    gpu_index = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] if os.environ.get(
        "CUDA_VISIBLE_DEVICES") else str(local)
    events = []
    with ClockSampler(gpu_index) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        wall0 = time.perf_counter()
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
            events.append((e0, e1))
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        wall = time.perf_counter() - wall0
    ms = sum(a.elapsed_time(b) for a, b in events)
    launches = g.last_launch_count()
    if watch:
        watch.beat(args.warmup + args.steps)
        watch.check()
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    images_per_s = total / (ms_per_step / 1000.0)
    flops, gemm_flops = loop_flops(B, lens)
    pk, pk_kind = peaks()

    # ---- e2e: the reference-facing C ABI call with pinned host buffers ----
    h_lat = torch.from_numpy(lat).pin_memory()
    h_enc = torch.from_numpy(enc).pin_memory()
    h_bias = torch.from_numpy(bias).pin_memory()
    h_out = torch.empty_like(h_lat).pin_memory()

    def e2e_step():
        g.denoise_loop_ptrs(h_lat.data_ptr(), B, 32, 32, h_enc.data_ptr(), CAPTION_LEN, 2304, h_bias.data_ptr(),
                            h_out.data_ptr(), GUIDANCE, NUM_STEPS)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t1 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    h2d = h_lat.numel() * 4 + h_enc.numel() * 4 + h_bias.numel() * 4
    d2h = h_out.numel() * 4

    # ---- roofline of the dominant kernel, measured live: one eager loop with CUDA events ----
    from sana_b200 import gemm_counts
    tc0, simt0 = gemm_counts()
    prof = g.profile_loop_device(d_lat.data_ptr(), B, 32, 32, d_enc.data_ptr(), CAPTION_LEN, 2304,
                                 d_bias.data_ptr(), d_out.data_ptr(), GUIDANCE, NUM_STEPS)
    torch.cuda.synchronize()
    tc1, simt1 = gemm_counts()
    classes = kernel_classes(B, lens)
    gemm_names = [k for k, v in classes.items() if v[0] == "flop"]
    gemm_ms = sum(prof[k][1] for k in gemm_names if k in prof)
    gemm_fl = sum(classes[k][1] * prof[k][0] for k in gemm_names if k in prof)
    achieved = gemm_fl / (gemm_ms / 1e3) / 1e12
    # the dominant kernel: the FF-inverted projection (the loop's largest launch)
    ff_n, ff_total_ms = prof.get("gemm_ff_inverted", (0, 0.0))
    ff_flops = classes["gemm_ff_inverted"][1]
    ff_ms_launch = ff_total_ms / max(ff_n, 1)
    ff_achieved = ff_flops / (ff_ms_launch / 1e3) / 1e12 if ff_n else None
    loop_ms = sum(v[1] for v in prof.values())
    breakdown = {}
    for k, (n, ms_k) in sorted(prof.items(), key=lambda kv: -kv[1][1]):
        e = {"launches": n, "ms_per_loop": round(ms_k, 3), "share": round(ms_k / loop_ms, 4)}
        if k in classes:
            kind, per_launch = classes[k]
            rate = per_launch * n / (ms_k / 1e3)
            if kind == "flop":
                e["tflops"] = round(rate / 1e12, 1)
            else:
                e["gbs"] = round(rate / 1e9, 1)
                e["frac_hbm"] = round(rate / 1e9 / pk["hbm_gbs"], 3)
        breakdown[k] = e
    _, per_shape = gemm_roofline(g, torch, stream, 2 * B * 1024, pk["bf16_tflops"])

    # BASELINE configs[4], the op-level microbenchmark, at one GPU (after the timed region)
    micro = None
    if world == 1 and not args.no_microbench:
        micro = [{k: v for k, v in m.items() if k not in ("steps", "warmup", "l2", "peak_source")}
                 for m in microbench_lines(g, stream, CONFIG4_OPS, 5, 3)]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, dt, threads, kind = cpu_sample()
        cpu = {"value": v, "unit": "images/s", "cores": threads, "kind": kind,
               "sample": f"one reference block_forward of one 1024-token sequence per thread ({threads} threads, "
                         f"{dt:.1f} s), extrapolated x2 sequences x28 blocks x{NUM_STEPS} steps per image"}

    if rank == 0:
        clocks = clk.summary()
        out = {
            "metric": METRIC, "value": images_per_s, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded random-init Sana-0.6B weights, N(0,1) latents and caption states",
            "config": config_dict(args),
            "denoiser_steps_per_s": images_per_s * NUM_STEPS,
            "wall_s_timed_region": wall,
            "roofline": {"bound": "tensor",
                         "kernel": "gemm_tc2_kernel<256> FF-inverted projection (tcgen05.mma.cta_group::2, "
                                   "256x256 tiles, TMA, TMEM accumulators, +bias +SiLU epilogue)",
                         "achieved": ff_achieved, "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                         "frac": ff_achieved / pk["bf16_tflops_sustained"],
                         "algorithmic_per_launch": ff_flops, "launches": ff_n, "avg_launch_ms": ff_ms_launch,
                         "peak_source": f"{pk_kind} bf16_tflops_sustained (kernel timed inside the loop)",
                         "measured": "CUDA events around every launch of one eager loop on the launch stream",
                         "traffic": FF_INVERTED_TRAFFIC["bytes"] if B == 16 else None, "traffic_unit": "bytes",
                         "traffic_source": (FF_INVERTED_TRAFFIC["source"] + ", copied, not measured in this run")
                         if B == 16 else "no capture at this per-GPU batch",
                         "all_block_gemms": {"achieved": achieved, "unit": "TFLOP/s",
                                             "frac": achieved / pk["bf16_tflops_sustained"]},
                         "isolated_per_shape": per_shape},
            "kernels": breakdown,
            "gemm_dispatch_per_loop": {"tensor_core": tc1 - tc0, "cuda_core": simt1 - simt0},
            "microbench_config4": None if micro is None else {
                "ops": micro, "timing": "median of 5 launches after 3 warm-up, L2 flushed before each, "
                                        "peaks are the burst figures (ops timed alone)"},
            "model_flops": {"per_loop_tflop": flops / 1e12, "achieved_tflops": flops / (ms_per_step / 1e3) / 1e12,
                            "frac_of_sustained_peak": flops / (ms_per_step / 1e3) / 1e12 / pk["bf16_tflops_sustained"],
                            "gemm_share_of_flops": gemm_flops / flops},
            "cpu_baseline": cpu,
            "e2e": {"value": total / e2e_s, "unit": "images/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_cfg_pair(args):
    """--cfg-pair: the latency mode. Ranks 2p / 2p+1 run the unconditional / conditional
    branch of the same images (configs[1]: one image per pair by default) and meet once per
    step inside the guidance kernel over NVLink peer memory (sana_b200.cfgpair). `value` is
    images/s over all pairs; `latency_ms` is one image's 20-step loop. Rank 0 also times the
    one-GPU loop of the same images and reports how far the paired result is from it."""
    import torch
    import torch.distributed as dist
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    from sana_b200 import synthetic as syn
    from sana_b200.cfgpair import connect_engine, pair_of
    from sana_b200.watchdog import init_ranks
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    rank, world, watch = init_ranks("nccl", timeout_s=300.0, device_id=torch.device("cuda", local))
    pair, branch, _ = pair_of(rank, world)
    pairs = world // 2
    B = args.images if args.images else 1
    dims = syn.ModelDims()
    tensors = make_weights(dims)
    g = SanaCuda(local, SANA_MODE_BF16)
    g.upload_checkpoint(dims.as_args(), tensors)
    del tensors
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    g.set_stream(stream.cuda_stream)
    lat, enc, bias, lens = make_inputs(pair * B, B)
    assert connect_engine(g, lat.size) == branch
    d_lat = torch.from_numpy(lat).cuda()
    d_enc = torch.from_numpy(np.ascontiguousarray(enc[branch * B:(branch + 1) * B])).cuda()
    d_bias = torch.from_numpy(np.ascontiguousarray(bias[branch * B:(branch + 1) * B])).cuda()
    d_out = torch.empty_like(d_lat)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def step():
        g.denoise_loop_pair_device(d_lat.data_ptr(), B, 32, 32, d_enc.data_ptr(), CAPTION_LEN, 2304,
                                   d_bias.data_ptr(), d_out.data_ptr(), GUIDANCE, NUM_STEPS)

    for i in range(args.warmup):
        step()
        g.synchronize()
        if watch:
            watch.beat(i + 1)
            watch.check()
    dist.barrier()
    gpu_index = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] if os.environ.get(
        "CUDA_VISIBLE_DEVICES") else str(local)
    events = []
    with ClockSampler(gpu_index) as clk:
        torch.cuda.synchronize()
        dist.barrier()
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
            events.append((e0, e1))
        g.synchronize()
        dist.barrier()
    ms = sum(a.elapsed_time(b) for a, b in events) / args.steps
    launches = g.last_launch_count()
    t = torch.tensor([ms], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    paired = d_out.cpu().numpy()

    # e2e through the Python API: pinned host inputs in, result out, every step
    h_lat = torch.from_numpy(lat).pin_memory()
    h_enc = torch.from_numpy(np.ascontiguousarray(enc[branch * B:(branch + 1) * B])).pin_memory()
    h_bias = torch.from_numpy(np.ascontiguousarray(bias[branch * B:(branch + 1) * B])).pin_memory()
    h_out = torch.empty_like(h_lat).pin_memory()

    def e2e_step():
        d_lat.copy_(h_lat, non_blocking=True)
        d_enc.copy_(h_enc, non_blocking=True)
        d_bias.copy_(h_bias, non_blocking=True)
        step()
        h_out.copy_(d_out, non_blocking=True)
        stream.synchronize()

    e2e_step()
    dist.barrier()
    t1 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t1) / args.steps
    t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())
    g.synchronize()
    g.cfg_pair_close()
    dist.barrier()

    single = None
    if rank == 0:
        # the same images on one GPU, both branches in one batch
        s_enc, s_bias = torch.from_numpy(enc).cuda(), torch.from_numpy(bias).cuda()
        s_out = torch.empty_like(d_lat)

        def one_gpu():
            g.denoise_loop_device(d_lat.data_ptr(), B, 32, 32, s_enc.data_ptr(), CAPTION_LEN, 2304,
                                  s_bias.data_ptr(), s_out.data_ptr(), GUIDANCE, NUM_STEPS)
        d_lat.copy_(torch.from_numpy(lat))
        for _ in range(args.warmup):
            one_gpu()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            flush.zero_()
            one_gpu()
        e1.record(stream)
        e1.synchronize()
        ref = s_out.cpu().numpy().astype(np.float64).ravel()
        a = paired.astype(np.float64).ravel()
        single = {"ms": e0.elapsed_time(e1) / args.steps,
                  "cosine": float(a @ ref / (np.linalg.norm(a) * np.linalg.norm(ref))),
                  "rel_l2": float(np.linalg.norm(a - ref) / np.linalg.norm(ref))}
        out = {
            "metric": METRIC, "mode": "cfg_pair (latency)", "value": pairs * B / (ms / 1e3), "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "latency_ms": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded random-init Sana-0.6B weights, N(0,1) latents and caption states",
            "config": {"workload": f"config1: {B} image(s) per GPU pair, unconditional branch on one GPU and "
                                   f"conditional on the other, {NUM_STEPS}-step DPM-Solver++ loop, guidance "
                                   f"{GUIDANCE}; one {B * 32 * 1024 * 4 // 1024} KB noise exchange per step and "
                                   "direction over NVLink inside the guidance kernel",
                       "global_batch": pairs * B, "seq_len": 1024, "caption_tokens": CAPTION_LEN,
                       "parallelism": f"{pairs} pair(s) x 2 CFG branches",
                       "l2": "flushed between timed iterations (256 MiB write, untimed)"},
            "one_gpu_same_images": {"ms": single["ms"], "speedup": single["ms"] / ms,
                                    "paired_vs_one_gpu_cosine": single["cosine"],
                                    "paired_vs_one_gpu_rel_l2": single["rel_l2"]},
            "e2e": {"value": pairs * B / e2e_s, "unit": "images/s",
                    "h2d_bytes_per_step": 2 * (h_lat.numel() + h_enc.numel() + h_bias.numel()) * 4,
                    "d2h_bytes_per_step": 2 * h_out.numel() * 4,
                    "note": "Python API (torch copies from pinned host memory + the paired loop), both ranks"},
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--images", type=int, default=16, help="images (x2 CFG sequences) in the batch, over all GPUs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-microbench", action="store_true", help="skip the config-4 op lines of the 1-GPU run")
    ap.add_argument("--microbench", action="store_true",
                    help="op-level microbenchmark (BASELINE configs[4]) instead of the loop; one GPU")
    ap.add_argument("--op", default="", help="with --microbench: comma-separated subset of " + ",".join(MICRO_OPS))
    ap.add_argument("--cfg-pair", action="store_true",
                    help="latency mode: each pair of ranks splits one batch's CFG branches (--images per pair, "
                         "default 1)")
    args = ap.parse_args()
    if args.cfg_pair and args.impl == "cuda":
        if args.images == 16 and "--images" not in sys.argv:
            args.images = 1
        run_cfg_pair(args)
    elif args.microbench:
        run_microbench(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_cuda(args)


if __name__ == "__main__":
    main()
