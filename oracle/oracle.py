"""TEST INFRASTRUCTURE ONLY: ctypes bindings for the two CPU checkers.

* ``Oracle()`` loads ``oracle/liboracle_sana.so``: our plain-C restatement of the reference's
  fp32 algorithm (``sana_oracle.c``).
* ``Reference()`` loads ``oracle/_ref/libsana_ref.so``: the reference's own sources
  (cconthekeyboard/sana.cpp ``src/*.cpp``) compiled unmodified by ``oracle/Makefile``.

Both expose the same methods with the same argument meaning; arrays are numpy float32 in
the reference's layouts (activations ``[batch, tokens, hidden]``, linear weights
``[in, out]``, conv weights ``[out, in, kh, kw]``, images NCHW). Only tests, the
``smoke()`` checker and bench.py's CPU-baseline leg use this module.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle_sana.so")
REF_LIB = os.path.join(HERE, "_ref", "libsana_ref.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_sz = ctypes.c_size_t


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], "need contiguous float32"
    return a.ctypes.data_as(_f32p)


def _f32(a) -> Optional[np.ndarray]:
    if a is None:
        return None
    return np.ascontiguousarray(a, dtype=np.float32)


class CheckerError(RuntimeError):
    pass


class SchedConfig(ctypes.Structure):
    """SanaSchedulerConfig (scheduler.h:9-20) as plain fields (orc_sched_config / RefSchedConfig)."""
    _fields_ = [("num_train_timesteps", ctypes.c_int), ("flow_shift", ctypes.c_float),
                ("use_flow_sigmas", ctypes.c_int), ("solver_order", ctypes.c_int),
                ("lower_order_final", ctypes.c_int), ("final_sigmas_zero", ctypes.c_int),
                ("solver_heun", ctypes.c_int)]


SCHED_DEFAULTS = dict(num_train_timesteps=1000, flow_shift=3.0, use_flow_sigmas=1, solver_order=2,
                      lower_order_final=1, final_sigmas_zero=1, solver_heun=0)


class _Cpu:
    prefix = ""
    path = ""

    def __init__(self, path: Optional[str] = None):
        self.lib = ctypes.CDLL(path or self.path)
        getattr(self.lib, self.prefix + "last_error").restype = ctypes.c_char_p
        getattr(self.lib, self.prefix + "model_create").restype = ctypes.c_void_p
        getattr(self.lib, self.prefix + "model_destroy").argtypes = [ctypes.c_void_p]

    def _call(self, name, *args):
        fn = getattr(self.lib, self.prefix + name)
        rc = fn(*args)
        if rc != 0:
            msg = getattr(self.lib, self.prefix + "last_error")().decode()
            if rc == 1:
                raise ValueError(msg)
            raise CheckerError(msg)

    # -- VAE decoder (vae.cpp:243 run_vae_decode) ---------------------------------------
    def vae_decode(self, dims, tensors, latents):
        """dims: sana_b200.synthetic_vae.VaeDims; tensors in its upload order."""
        from sana_b200.synthetic_vae import dims_struct
        lat = _f32(latents)
        B, _, h, w = lat.shape
        ds = dims_struct(dims)
        arrs = [_f32(t) for t in tensors]
        table = (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
        up = dims.upscale()
        out = np.empty((B, dims.out_channels, h * up, w * up), np.float32)
        self._call("vae_decode", ctypes.byref(ds), table, _ptr(lat), _sz(B), _sz(h), _sz(w), _ptr(out))
        return out

    # -- primitives -------------------------------------------------------------------
    def randn(self, n: int, seed: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self._call("randn", _ptr(out), _sz(n), ctypes.c_uint64(seed))
        return out

    def linear_3d(self, x, w, bias=None):
        x, w, bias = _f32(x), _f32(w), _f32(bias)
        B, T, K = x.shape
        N = w.shape[1]
        out = np.empty((B, T, N), np.float32)
        self._call("linear_3d", _ptr(x), _sz(B), _sz(T), _sz(K), _ptr(w), _ptr(bias), _sz(N), _ptr(out))
        return out

    def layer_norm(self, x, eps, gamma=None, beta=None):
        x, gamma, beta = _f32(x), _f32(gamma), _f32(beta)
        B, T, C = x.shape
        out = np.empty_like(x)
        self._call("layer_norm", _ptr(x), _sz(B), _sz(T), _sz(C), ctypes.c_float(eps), _ptr(gamma), _ptr(beta), _ptr(out))
        return out

    def rms_norm(self, x, eps, weight=None):
        x, weight = _f32(x), _f32(weight)
        B, T, C = x.shape
        out = np.empty_like(x)
        self._call("rms_norm", _ptr(x), _sz(B), _sz(T), _sz(C), ctypes.c_float(eps), _ptr(weight), _ptr(out))
        return out

    def modulate(self, x, shift, scale):
        x, shift, scale = _f32(x), _f32(shift), _f32(scale)
        B, T, C = x.shape
        out = np.empty_like(x)
        self._call("modulate", _ptr(x), _sz(B), _sz(T), _sz(C), _ptr(shift), _ptr(scale), _ptr(out))
        return out

    def linear_attention(self, q, k, v):
        q, k, v = _f32(q), _f32(k), _f32(v)
        B, H, Tq, D = q.shape
        Tk = k.shape[2]
        out = np.empty_like(q)
        self._call("linear_attention", _ptr(q), _ptr(k), _ptr(v), _sz(B), _sz(H), _sz(Tq), _sz(Tk), _sz(D), _ptr(out))
        return out

    def attention(self, q, k, v, bias=None):
        q, k, v, bias = _f32(q), _f32(k), _f32(v), _f32(bias)
        B, H, Tq, D = q.shape
        Tk = k.shape[2]
        out = np.empty_like(q)
        self._call("attention", _ptr(q), _ptr(k), _ptr(v), _sz(B), _sz(H), _sz(Tq), _sz(Tk), _sz(D), _ptr(bias), _ptr(out))
        return out

    def conv1x1(self, x, w, bias=None):
        x, w, bias = _f32(x), _f32(w), _f32(bias)
        B, Cin, H, W = x.shape
        Cout = w.shape[0]
        out = np.empty((B, Cout, H, W), np.float32)
        self._call("conv1x1", _ptr(x), _sz(B), _sz(Cin), _sz(H), _sz(W), _ptr(w), _ptr(bias), _sz(Cout), _ptr(out))
        return out

    def depthwise3x3(self, x, w, bias=None):
        x, w, bias = _f32(x), _f32(w), _f32(bias)
        B, C, H, W = x.shape
        out = np.empty_like(x)
        self._call("depthwise3x3", _ptr(x), _sz(B), _sz(C), _sz(H), _sz(W), _ptr(w), _ptr(bias), _ptr(out))
        return out

    def glumb_conv(self, x, w_inv, b_inv, w_dw, b_dw, w_pt):
        x, w_inv, b_inv, w_dw, b_dw, w_pt = map(_f32, (x, w_inv, b_inv, w_dw, b_dw, w_pt))
        B, Cin, H, W = x.shape
        E = w_inv.shape[0]
        Cout = w_pt.shape[0]
        out = np.empty((B, Cout, H, W), np.float32)
        self._call("glumb_conv", _ptr(x), _sz(B), _sz(Cin), _sz(H), _sz(W), _ptr(w_inv), _ptr(b_inv), _sz(E),
                   _ptr(w_dw), _ptr(b_dw), _ptr(w_pt), _sz(Cout), _ptr(out))
        return out

    def project_caption(self, enc, w1, b1, w2, b2, norm_w):
        enc, w1, b1, w2, b2, norm_w = map(_f32, (enc, w1, b1, w2, b2, norm_w))
        B, L, Din = enc.shape
        C = w1.shape[1]
        out = np.empty((B, L, C), np.float32)
        self._call("project_caption", _ptr(enc), _sz(B), _sz(L), _sz(Din), _ptr(w1), _ptr(b1), _sz(C),
                   _ptr(w2), _ptr(b2), _ptr(norm_w), _ptr(out))
        return out

    def cfg(self, noise, g):
        noise = _f32(noise)
        B2, Cl, H, W = noise.shape
        out = np.empty((B2 // 2, Cl, H, W), np.float32)
        self._call("cfg", _ptr(noise), _sz(B2 // 2), _sz(Cl), _sz(H), _sz(W), ctypes.c_float(g), _ptr(out))
        return out

    def scheduler_schedule(self, n: int, flow_shift: float = 3.0):
        ts = np.empty(n, np.float32)
        sg = np.empty(n + 1, np.float32)
        self._call("scheduler_schedule", _sz(n), ctypes.c_float(flow_shift), _ptr(ts), _ptr(sg))
        return ts, sg

    def scheduler_run(self, model_outputs, sample, flow_shift: float = 3.0):
        mo = _f32(model_outputs)
        x = _f32(sample).reshape(-1)
        n = mo.shape[0]
        out = np.empty((n, x.size), np.float32)
        self._call("scheduler_run", _sz(n), ctypes.c_float(flow_shift), _ptr(mo), _ptr(x), _sz(x.size), _ptr(out))
        return out

    def scheduler_run_config(self, config: dict, model_outputs, sample, sigmas=None):
        """init_sana_scheduler_state + step_sana_scheduler over all model outputs with a
        config (the fields of the C ABI's sana_scheduler_config; missing fields take the
        reference's defaults). `sigmas` [n + 1] replaces the built schedule. Returns
        (timesteps, sigmas, samples after every step)."""
        c = SchedConfig(**{**SCHED_DEFAULTS, **config})
        mo = _f32(model_outputs)
        x = _f32(sample).reshape(-1)
        n = mo.shape[0]
        sg_in = None if sigmas is None else _f32(sigmas)
        ts = np.empty(n, np.float32)
        sg = np.empty(n + 1, np.float32)
        out = np.empty((n, x.size), np.float32)
        self._call("scheduler_run_config", ctypes.byref(c), _sz(n), _ptr(sg_in), _ptr(mo), _ptr(x), _sz(x.size),
                   _ptr(ts), _ptr(sg), _ptr(out))
        return ts, sg, out

    def attention_block(self, x, wq, bq, wk, bk, wv, bv, wo, bo, heads):
        x, wq, bq, wk, bk, wv, bv, wo, bo = map(_f32, (x, wq, bq, wk, bk, wv, bv, wo, bo))
        B, T, C = x.shape
        out = np.empty_like(x)
        self._call("attention_block", _ptr(x), _sz(B), _sz(T), _sz(C), _ptr(wq), _ptr(bq), _ptr(wk), _ptr(bk),
                   _ptr(wv), _ptr(bv), _ptr(wo), _ptr(bo), _sz(heads), _ptr(out))
        return out

    def cross_attention_block(self, x, ctx, bias, wq, bq, wk, bk, wv, bv, wo, bo, heads):
        x, ctx, bias, wq, bq, wk, bk, wv, bv, wo, bo = map(_f32, (x, ctx, bias, wq, bq, wk, bk, wv, bv, wo, bo))
        B, T, C = x.shape
        L = ctx.shape[1]
        out = np.empty_like(x)
        self._call("cross_attention_block", _ptr(x), _sz(B), _sz(T), _sz(C), _ptr(ctx), _sz(L), _ptr(bias),
                   _ptr(wq), _ptr(bq), _ptr(wk), _ptr(bk), _ptr(wv), _ptr(bv), _ptr(wo), _ptr(bo), _sz(heads),
                   _ptr(out))
        return out

    def scheduler_convert(self, sigmas, step_index, model_output, sample):
        sg, mo, x = _f32(sigmas), _f32(model_output).reshape(-1), _f32(sample).reshape(-1)
        out = np.empty_like(x)
        self._call("scheduler_convert", _ptr(sg), _sz(sg.size), _sz(step_index), _ptr(mo), _ptr(x), _sz(x.size),
                   _ptr(out))
        return out

    def scheduler_update(self, order, sigmas, step_index, m0, m1, sample):
        sg, x = _f32(sigmas), _f32(sample).reshape(-1)
        m0 = _f32(m0).reshape(-1)
        m1 = _f32(m1).reshape(-1) if m1 is not None else None
        out = np.empty_like(x)
        self._call("scheduler_update", ctypes.c_int(order), _ptr(sg), _sz(sg.size), _sz(step_index), _ptr(m0),
                   _ptr(m1), _ptr(x), _sz(x.size), _ptr(out))
        return out

    def scheduler_step(self, sigmas, step_index, lower, hist, model_output, sample):
        """Returns (new_sample, new_history[list, oldest first], new_lower_count)."""
        sg, mo, x = _f32(sigmas), _f32(model_output).reshape(-1), _f32(sample).reshape(-1)
        n = x.size
        h = np.ascontiguousarray(np.stack([np.asarray(a, np.float32).reshape(-1) for a in hist]) if hist
                                 else np.zeros((1, n), np.float32))
        out = np.empty_like(x)
        hist_out = np.empty((3, n), np.float32)
        nh, lo = ctypes.c_size_t(0), ctypes.c_size_t(0)
        self._call("scheduler_step", _ptr(sg), _sz(sg.size), _sz(step_index), _sz(lower), _ptr(h), _sz(len(hist)),
                   _ptr(mo), _ptr(x), _sz(n), _ptr(out), _ptr(hist_out), ctypes.byref(nh), ctypes.byref(lo))
        return out, [hist_out[i].copy() for i in range(nh.value)], lo.value

    # -- model ------------------------------------------------------------------------
    def model(self, tensors: Sequence[np.ndarray], n_blocks, C, Cl, Din, E, self_heads, cross_heads):
        return _CpuModel(self, tensors, n_blocks, C, Cl, Din, E, self_heads, cross_heads)


class _CpuModel:
    """A model handle; ``tensors`` is the synthetic checkpoint list in PyTorch layout."""

    def __init__(self, cpu: _Cpu, tensors, n_blocks, C, Cl, Din, E, self_heads, cross_heads):
        self.cpu = cpu
        self.C, self.Cl, self.Din, self.E = C, Cl, Din, E
        self.n_blocks = n_blocks
        self._keep = [_f32(t) for t in tensors]
        arr = (_f32p * len(self._keep))(*[_ptr(t) for t in self._keep])
        fn = getattr(cpu.lib, cpu.prefix + "model_create")
        fn.restype = ctypes.c_void_p
        self.h = fn(arr, _sz(n_blocks), _sz(C), _sz(Cl), _sz(Din), _sz(E), _sz(self_heads), _sz(cross_heads))
        if not self.h:
            raise ValueError(getattr(cpu.lib, cpu.prefix + "last_error")().decode())
        self._keep = None  # both checkers copy the weights

    def __del__(self):
        if getattr(self, "h", None):
            getattr(self.cpu.lib, self.cpu.prefix + "model_destroy")(ctypes.c_void_p(self.h))
            self.h = None

    def _call(self, name, *args):
        self.cpu._call(name, ctypes.c_void_p(self.h), *args)

    def set_cross_qk_norm(self, block, enable, q_weight=None, k_weight=None, eps=1e-6):
        """The optional RMSNorm of the cross-attention q and k projections (off = the
        reference's block)."""
        qw, kw = _f32(q_weight), _f32(k_weight)
        self._keep_norm = getattr(self, "_keep_norm", {})
        self._keep_norm[block] = (qw, kw)
        self._call("model_set_cross_qk_norm", _sz(block), ctypes.c_int(1 if enable else 0), _ptr(qw), _ptr(kw),
                   ctypes.c_float(eps))

    def set_block_extras(self, block, **kw):
        names = ["q_bias", "k_bias", "v_bias", "attn_gamma", "attn_beta", "mlp_gamma", "mlp_beta"]
        vals = [_f32(kw.get(n)) for n in names]
        self._keep_extras = vals
        self._call("model_set_block_extras", _sz(block), *[_ptr(v) for v in vals])

    def block_forward(self, block, x, ctx, tmod, bias=None):
        x, ctx, tmod, bias = map(_f32, (x, ctx, tmod, bias))
        S, T, C = x.shape
        L = ctx.shape[1]
        outs = [np.empty_like(x) for _ in range(3)]
        self._call("block_forward", _sz(block), _ptr(x), _sz(S), _sz(T), _ptr(ctx), _sz(L), _ptr(tmod), _ptr(bias),
                   *[_ptr(o) for o in outs])
        return outs

    def run_model_blocks(self, x, ctx, tmod, bias=None, begin=0, end=None):
        x, ctx, tmod, bias = map(_f32, (x, ctx, tmod, bias))
        S, T, C = x.shape
        L = ctx.shape[1]
        end = self.n_blocks if end is None else end
        out = np.empty_like(x)
        self._call("run_model_blocks", _ptr(x), _sz(S), _sz(T), _ptr(ctx), _sz(L), _ptr(tmod), _ptr(bias),
                   _sz(begin), _sz(end), _ptr(out))
        return out

    def project_caption(self, enc):
        enc = _f32(enc)
        S, L, Din = enc.shape
        out = np.empty((S, L, self.C), np.float32)
        self._call("model_project_caption", _ptr(enc), _sz(S), _sz(L), _sz(Din), _ptr(out))
        return out

    def time_embed(self, tvals):
        tv = _f32(np.asarray(tvals, np.float32).reshape(-1))
        S = tv.size
        emb = np.empty((S, self.C), np.float32)
        tmod = np.empty((S, 6 * self.C), np.float32)
        self._call("time_embed", _ptr(tv), _sz(S), _ptr(emb), _ptr(tmod))
        return emb, tmod

    def forward_nocfg(self, latents, t, ctx, bias=None):
        latents, ctx, bias = map(_f32, (latents, ctx, bias))
        S, Cl, H, W = latents.shape
        L = ctx.shape[1]
        out = np.empty_like(latents)
        self._call("forward_nocfg", _ptr(latents), _sz(S), _sz(H), _sz(W), ctypes.c_float(t), _ptr(ctx), _sz(L),
                   _ptr(bias), _ptr(out))
        return out

    def denoise(self, latents, enc, bias, guidance, num_steps, run_steps=None):
        latents, enc, bias = map(_f32, (latents, enc, bias))
        B, Cl, H, W = latents.shape
        L, Din = enc.shape[1], enc.shape[2]
        run_steps = num_steps if run_steps is None else run_steps
        out = np.empty_like(latents)
        si = ctypes.c_size_t(0)
        self._call("denoise", _ptr(latents), _sz(B), _sz(H), _sz(W), _ptr(enc), _sz(L), _sz(Din), _ptr(bias),
                   ctypes.c_float(guidance), _sz(num_steps), _sz(run_steps), _ptr(out), ctypes.byref(si))
        return out


class Oracle(_Cpu):
    # -- text-encoder output contract (gemma_encoder.cpp:51-77,177-244) -----------------
    def select_rows_first_and_last(self, x, keep):
        x = _f32(x)
        rows, cols = x.shape
        out = np.empty((keep, cols), np.float32)
        self._call("select_rows_first_and_last", _ptr(x), _sz(rows), _sz(cols), _sz(keep), _ptr(out))
        return out

    def prompt_pair_assemble(self, negative, negative_real, positive, positive_real, max_sequence_length=300):
        negative, positive = _f32(negative), _f32(positive)
        L = max_sequence_length
        hidden = positive.shape[1]
        emb = np.empty((2, L, hidden), np.float32)
        bias = np.empty((2, 1, L), np.float32)
        self._call("prompt_pair_assemble", _ptr(negative), _sz(negative.shape[0]), _sz(negative_real), _ptr(positive),
                   _sz(positive.shape[0]), _sz(positive_real), _sz(hidden), _sz(L), _ptr(emb), _ptr(bias))
        return emb, bias


    prefix = "orc_"
    path = ORACLE_LIB


class Reference(_Cpu):
    prefix = "ref_"
    path = REF_LIB

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_LIB)
