"""Generates the golden fixtures in this folder by running the reference itself.

The reference (cconthekeyboard/sana.cpp ``src/*.cpp``, unmodified) is compiled by
``oracle/Makefile`` into ``oracle/_ref/libsana_ref.so``; this script drives it through
``oracle/oracle.py``'s ``Reference`` binding on seeded synthetic inputs and stores the
outputs as small ``.npz`` files. Weights and inputs are not stored: they are re-created
from the seeds recorded in each file with the torch-compatible generator, which the
tests show is bit-identical across the reference, the oracle and the product.

Usage (from the repo root, after ``make -C oracle``):
    python tests/golden/make_golden.py small      # ops, small model, scheduler (seconds)
    python tests/golden/make_golden.py block      # one full-size block (~10 s)
    python tests/golden/make_golden.py blocks     # block 0 at 4096 tokens and at mixed masks (~1 min)
    python tests/golden/make_golden.py forward    # config 0: one CFG-batch forward (~4 min)
    python tests/golden/make_golden.py loop       # config 1: 20-step loop (~80 min)
    python tests/golden/make_golden.py vae        # VAE decoder: small dims, DC-AE dims at 2x2 (~1 min)
    python tests/golden/make_golden.py scheduler  # scheduler configurations (+ tests/cpp/scheduler_configs.inc)
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "sana.cpp_b200")]

from oracle import Reference  # noqa: E402
from sana_b200 import synthetic as syn  # noqa: E402

# Small model used by the fast parity cases: every dimension differs, heads divide
# the hidden size, the token grid is 4 x 4.
SMALL = syn.ModelDims(n_blocks=2, hidden=64, latent_channels=4, caption_dim=48, ff_expanded=160,
                      self_heads=4, cross_heads=2)
FULL = syn.ModelDims()


def ops_cases(rnd):
    """Seeded op-level cases: (name, method, args). Inputs use seeds 100.. ."""
    d = lambda n, s: syn._draw(rnd, n, s)  # noqa: E731
    x = d(2 * 8 * 24, 100).reshape(2, 8, 24)
    w = d(24 * 16, 101).reshape(24, 16) * np.float32(0.2)
    g, be = d(24, 103), d(24, 104)
    sh, sc = d(2 * 24, 105).reshape(2, 24), d(2 * 24, 106).reshape(2, 24)
    q = d(2 * 3 * 16 * 8, 107).reshape(2, 3, 16, 8)
    k = d(2 * 3 * 16 * 8, 108).reshape(2, 3, 16, 8)
    v = d(2 * 3 * 16 * 8, 109).reshape(2, 3, 16, 8)
    kk = d(2 * 3 * 7 * 8, 110).reshape(2, 3, 7, 8)
    vv = d(2 * 3 * 7 * 8, 111).reshape(2, 3, 7, 8)
    img = d(2 * 6 * 5 * 7, 112).reshape(2, 6, 5, 7)
    enc = d(2 * 5 * 12, 122).reshape(2, 5, 12)
    return [
        ("linear_3d", "linear_3d", (x, w, d(16, 102))),
        ("layer_norm", "layer_norm", (x, 1e-6, g, be)),
        ("rms_norm", "rms_norm", (x, 1e-5, g)),
        ("modulate", "modulate", (x, sh, sc)),
        ("linear_attention", "linear_attention", (q, k, v)),
        ("attention", "attention", (q, kk, vv, syn.attention_bias([3, 7], 7))),
        ("conv1x1", "conv1x1", (img, d(10 * 6, 113).reshape(10, 6, 1, 1), d(10, 114))),
        ("depthwise3x3", "depthwise3x3", (img, d(6 * 9, 115).reshape(6, 1, 3, 3), d(6, 116))),
        ("glumb_conv", "glumb_conv", (img, d(12 * 6, 117).reshape(12, 6, 1, 1) * np.float32(0.5), d(12, 118),
                                      d(12 * 9, 119).reshape(12, 1, 3, 3) * np.float32(0.5), d(12, 120),
                                      d(5 * 6, 121).reshape(5, 6, 1, 1))),
        ("project_caption", "project_caption", (enc, d(12 * 10, 123).reshape(12, 10) * np.float32(0.3), d(10, 124),
                                                d(10 * 10, 125).reshape(10, 10) * np.float32(0.3), d(10, 126),
                                                d(10, 127))),
    ]


def small_model_run(m, rnd):
    """The small-model cases, run on a model handle of either checker."""
    d = SMALL
    S, T, L = 2, 16, 8
    xin = syn._draw(rnd, S * T * d.hidden, 200).reshape(S, T, d.hidden)
    enc = syn.encoder_states(rnd, S, L, d.caption_dim, 201)
    mbias = syn.attention_bias([3, 8], L)
    ctx = m.project_caption(enc)
    emb, tmod = m.time_embed([999.0, 500.0])
    stages = m.block_forward(1, xin, ctx, tmod, mbias)
    lat2 = syn.latents(rnd, 2, d.latent_channels, 4, 4, 202)
    lat1 = syn.latents(rnd, 1, d.latent_channels, 4, 4, 203)
    return dict(ctx=ctx, emb=emb, tmod=tmod, after_self=stages[0], after_cross=stages[1], after_ff=stages[2],
                noise_pred=m.forward_nocfg(lat2, 999.0, ctx, mbias), loop4=m.denoise(lat1, enc, mbias, 4.5, 4))


def small(ref: Reference):
    rnd = ref.randn
    out = {name: getattr(ref, meth)(*args) for name, meth, args in ops_cases(rnd)}
    np.savez_compressed(os.path.join(HERE, "ops_small.npz"), **out)

    # --- small model: weights base seed 5, bias_std 0.02
    tensors = syn.generate_model(SMALL, rnd, base_seed=5, bias_std=0.02)
    np.savez_compressed(os.path.join(HERE, "model_small.npz"), **small_model_run(ref.model(tensors, *SMALL.as_args()), rnd))

    # --- generator: raw draws (sizes below, at and above the 16-element block)
    np.savez_compressed(os.path.join(HERE, "rng.npz"), r17_3=rnd(17, 3), r1000_42=rnd(1000, 42),
                        r100003_9=rnd(100003, 9)[-64:])

    # --- scheduler: 20-step schedule and a run over seeded model outputs
    ts, sg = ref.scheduler_schedule(20, 3.0)
    mo = syn._draw(rnd, 20 * 64, 300).reshape(20, 64)
    x0 = syn._draw(rnd, 64, 301)
    np.savez_compressed(os.path.join(HERE, "scheduler_20.npz"), timesteps=ts, sigmas=sg,
                        samples=ref.scheduler_run(mo, x0, 3.0))


# Scheduler configurations beyond the default 2M midpoint (step_sana_scheduler,
# scheduler.cpp:272-318): (num_train_timesteps, flow_shift, use_flow_sigmas, solver_order,
# lower_order_final, final_sigmas_zero, solver_heun, steps, explicit schedule). An explicit
# schedule (the configs the builder refuses: variance-preserving sigmas, a nonzero final
# sigma) is the flow schedule of the same length with its final sigma set to 0.02.
SCHEDULER_CASES = [
    (1000, 3.0, 1, 2, 1, 1, 0, 20, 0),
    (1000, 3.0, 1, 2, 1, 1, 1, 20, 0),
    (1000, 3.0, 1, 1, 1, 1, 0, 20, 0),
    (1000, 3.0, 1, 1, 0, 0, 0, 8, 1),
    (1000, 3.0, 1, 2, 0, 0, 0, 8, 1),
    (1000, 3.0, 1, 2, 0, 0, 1, 8, 1),
    (1000, 3.0, 1, 2, 0, 1, 1, 10, 0),
    (500, 3.0, 1, 2, 1, 1, 0, 20, 0),
    (37, 2.5, 1, 2, 1, 1, 1, 7, 0),
    (1000, 1.0, 1, 2, 1, 1, 0, 5, 0),
    (1000, 3.0, 0, 2, 1, 1, 0, 12, 1),
    (1000, 3.0, 0, 2, 0, 0, 1, 12, 1),
    (1000, 3.0, 0, 1, 1, 1, 0, 12, 1),
    (1000, 3.0, 1, 2, 1, 1, 0, 1, 0),
    (1000, 3.0, 1, 2, 1, 1, 1, 2, 0),
]
SCHED_KEYS = ("num_train_timesteps", "flow_shift", "use_flow_sigmas", "solver_order", "lower_order_final",
              "final_sigmas_zero", "solver_heun")
SCHED_NUMEL = 16


def scheduler_configs(ref: Reference):
    """step_sana_scheduler run over every SCHEDULER_CASES entry on the reference build:
    tests/golden/scheduler_configs.npz and, for the C++ host-layer test, the same values as
    C arrays in tests/cpp/scheduler_configs.inc."""
    rnd = ref.randn
    out = {"cases": np.array(SCHEDULER_CASES, np.float64)}
    inc = ["// Generated by tests/golden/make_golden.py scheduler from the reference build", "// (step_sana_scheduler, scheduler.cpp:272-318); do not edit.",
           f"static const int kSchedCases = {len(SCHEDULER_CASES)};",
           f"static const int kSchedNumel = {SCHED_NUMEL};"]
    cfg_rows, offs_mo, offs_out, offs_sg = [], [], [], []
    all_mo, all_x0, all_out, all_sg = [], [], [], []
    for i, case in enumerate(SCHEDULER_CASES):
        cfg = dict(zip(SCHED_KEYS, case[:7]))
        n = case[7]
        mo = syn._draw(rnd, max(16, n * SCHED_NUMEL), 600 + 2 * i)[:n * SCHED_NUMEL].reshape(n, SCHED_NUMEL)
        x0 = syn._draw(rnd, SCHED_NUMEL, 601 + 2 * i)
        sig = None
        if case[8]:
            _, sig, _ = ref.scheduler_run_config({"num_train_timesteps": case[0], "flow_shift": case[1]}, mo, x0)
            sig = sig.copy()
            sig[-1] = np.float32(0.02)
        ts, sg, samples = ref.scheduler_run_config(cfg, mo, x0, sig)
        out[f"mo_{i}"], out[f"x0_{i}"], out[f"ts_{i}"], out[f"sg_{i}"], out[f"samples_{i}"] = mo, x0, ts, sg, samples
        cfg_rows.append(case)
        offs_mo.append(sum(len(a) for a in all_mo))
        offs_sg.append(sum(len(a) for a in all_sg))
        all_mo.append(mo.reshape(-1))
        all_x0.append(x0)
        all_sg.append(np.concatenate([ts, sg]))
        all_out.append(samples.reshape(-1))
    np.savez_compressed(os.path.join(HERE, "scheduler_configs.npz"), **out)

    def lit(v):  # shortest text that reads back as the same float32, as a C float literal
        t = format(float(v), ".9g")
        return (t if any(ch in t for ch in ".e") else t + ".0") + "f"

    def arr(name, ctype, vals):
        body = ", ".join(lit(v) if ctype == "float" else str(int(v)) for v in vals)
        return f"static const {ctype} {name}[] = {{{body}}};"
    inc.append("// per case: num_train_timesteps, flow_shift x 1000, use_flow_sigmas, solver_order,")
    inc.append("// lower_order_final, final_sigmas_zero, solver_heun, steps, explicit schedule")
    inc.append(arr("kSchedCfg", "int", [int(round(v * 1000)) if j == 1 else v for c in cfg_rows for j, v in enumerate(c)]))
    inc.append(arr("kSchedMoOff", "int", offs_mo))
    inc.append(arr("kSchedSgOff", "int", offs_sg))
    inc.append(arr("kSchedModelOut", "float", np.concatenate(all_mo).view(np.float32)))
    inc.append(arr("kSchedSample0", "float", np.concatenate(all_x0)))
    inc.append("// per case: timesteps[steps] then sigmas[steps + 1]")
    inc.append(arr("kSchedSchedule", "float", np.concatenate(all_sg)))
    inc.append("// per case: the sample after every step [steps, numel]")
    inc.append(arr("kSchedSamples", "float", np.concatenate(all_out)))
    with open(os.path.join(ROOT, "tests", "cpp", "scheduler_configs.inc"), "w") as f:
        f.write("\n".join(inc) + "\n")


def _signature(a: np.ndarray) -> dict:
    """A few hundred KB stand-in for a large activation: its first 4096 values, per-row
    sums and per-row sums of squares (rows = last axis), all in float64."""
    flat = a.reshape(-1, a.shape[-1]).astype(np.float64)
    return {"head": a.reshape(-1)[:4096].copy(), "row_sum": flat.sum(1), "row_sq": (flat * flat).sum(1)}


def full_model(ref: Reference):
    t0 = time.time()
    tensors = syn.generate_model(FULL, ref.randn, base_seed=0)
    m = ref.model(tensors, *FULL.as_args())
    del tensors
    print(f"weights ready in {time.time() - t0:.1f}s", flush=True)
    return m


def full_inputs(ref: Reference, images: int):
    enc = syn.encoder_states(ref.randn, 2, 300, FULL.caption_dim, 7)
    bias = syn.attention_bias([8, 24], 300)
    lat = syn.latents(ref.randn, images, FULL.latent_channels, 32, 32, 42)
    return lat, enc, bias


def block(ref: Reference):
    m = full_model(ref)
    lat, enc, bias = full_inputs(ref, 2)
    ctx = m.project_caption(enc)
    emb, tmod = m.time_embed([999.0, 999.0])
    x = syn._draw(ref.randn, 2 * 1024 * FULL.hidden, 400).reshape(2, 1024, FULL.hidden)
    t0 = time.time()
    st = m.block_forward(0, x, ctx, tmod, bias)
    print(f"block_forward {time.time() - t0:.1f}s", flush=True)
    out = {"ctx_head": ctx.reshape(-1)[:4096].copy(), "tmod": tmod}
    for name, a in zip(("after_self", "after_cross", "after_ff"), st):
        for k, v in _signature(a).items():
            out[f"{name}_{k}"] = v
    np.savez_compressed(os.path.join(HERE, "block0_full.npz"), **out)


# Further full-size block_forward cases: config 3's 64 x 64 latent grid (4096 tokens per
# sequence, its linear-attention token split and depthwise halo) and config 2's mixed caption
# masks (four sequences with valid lengths drawn from 8..120). (name, sequences, grid side,
# valid lengths, timestep, input seed)
BLOCK_CASES = {
    "block0_4096": (2, 64, (8, 24), 999.0, 402),
    "block0_mixed": (4, 32, (17, 120, 64, 9), 500.0, 403),
}


def block_case_inputs(m, rnd, name):
    """(x, ctx, tmod, bias) of a BLOCK_CASES entry for model `m` (one block, FULL dims)."""
    S, side, lens, t, seed = BLOCK_CASES[name]
    enc = syn.encoder_states(rnd, S, 300, FULL.caption_dim, 7 + seed)
    bias = syn.attention_bias(list(lens), 300)
    ctx = m.project_caption(enc)
    _, tmod = m.time_embed([t] * S)
    x = syn._draw(rnd, S * side * side * FULL.hidden, seed).reshape(S, side * side, FULL.hidden)
    return x, ctx, tmod, bias


def blocks_more(ref: Reference):
    t0 = time.time()
    d1 = syn.ModelDims(n_blocks=1)
    m = ref.model(syn.generate_model(d1, ref.randn, base_seed=0), *d1.as_args())
    for name in BLOCK_CASES:
        x, ctx, tmod, bias = block_case_inputs(m, ref.randn, name)
        t1 = time.time()
        st = m.block_forward(0, x, ctx, tmod, bias)
        print(f"{name}: block_forward {time.time() - t1:.1f}s", flush=True)
        out = {}
        for stage, a in zip(("after_self", "after_cross", "after_ff"), st):
            for k, v in _signature(a).items():
                out[f"{stage}_{k}"] = v
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"blocks {time.time() - t0:.1f}s", flush=True)


def forward(ref: Reference):
    m = full_model(ref)
    lat, enc, bias = full_inputs(ref, 2)
    ctx = m.project_caption(enc)
    t0 = time.time()
    noise = m.forward_nocfg(lat, 999.0, ctx, bias)
    print(f"forward {time.time() - t0:.1f}s", flush=True)
    np.savez_compressed(os.path.join(HERE, "forward_full.npz"), noise_pred=noise, seconds=time.time() - t0)


def loop(ref: Reference):
    m = full_model(ref)
    lat, enc, bias = full_inputs(ref, 1)
    t0 = time.time()
    out = m.denoise(lat, enc, bias, 4.5, 20)
    print(f"loop {time.time() - t0:.1f}s", flush=True)
    np.savez_compressed(os.path.join(HERE, "loop20_full.npz"), latents=out, seconds=time.time() - t0)


VAE_SMALL_SEED, VAE_FULL_SEED = 31, 32


def vae(ref: Reference):
    """run_vae_decode (vae.cpp:243) on the small test structure (two images of 4 x 6
    latents) and on DC-AE f32c32's structure at 2 x 2 latents (a 64 x 64 image)."""
    from sana_b200 import synthetic_vae as sv
    rnd = ref.randn
    t0 = time.time()
    small_out = ref.vae_decode(sv.SMALL, sv.generate_vae(sv.SMALL, rnd, VAE_SMALL_SEED),
                               sv_latents(rnd, 2, sv.SMALL.latent_channels, 4, 6, VAE_SMALL_SEED))
    full = sv.VaeDims()
    full_out = ref.vae_decode(full, sv.generate_vae(full, rnd, VAE_FULL_SEED),
                              sv_latents(rnd, 1, full.latent_channels, 2, 2, VAE_FULL_SEED))
    print(f"vae {time.time() - t0:.1f}s", flush=True)
    np.savez_compressed(os.path.join(HERE, "vae.npz"), small=small_out, full_2x2=full_out)


def sv_latents(rnd, B, C, h, w, seed):
    return syn.latents(rnd, B, C, h, w, 1000 + seed)


if __name__ == "__main__":
    ref = Reference()
    for what in sys.argv[1:] or ["small"]:
        {"small": small, "block": block, "forward": forward, "loop": loop, "vae": vae,
         "scheduler": scheduler_configs, "blocks": blocks_more}[what](ref)
